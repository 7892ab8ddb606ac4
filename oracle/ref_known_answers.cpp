/*
 * The reference's own device test cases evaluated on the reference's physics
 * compiled for the host (through refshim/carl_host_shim.h):
 *   tests/physics_regressions.cu:19-150 and tests/turtle_recovery.cu:31-78.
 * Each function makes the same calls on the same inputs as the reference test
 * and returns the quantities it checks, so the expectation tables in
 * tests/test_known_answers.py pin this oracle and the product alike.
 * TEST INFRASTRUCTURE.
 */
#include <cmath>
#include <cstring>

#include "State/GameState.cuh"
#include "State/Workspace.cuh"
#include "State/Reset.cuh"
#include "Physics/BallArena/Solve.cuh"
#include "Physics/Controls/Aerial.cuh"
#include "Physics/Controls/Drive.cuh"
#include "Physics/Goals.cuh"

extern "C" {

int refka_ball_hit_previous_tick(int hitTick, int tick) { return ballHitOnPreviousTick(hitTick, tick); }

float refka_floor_push_z(int hitAge)
{
    BallArenaContact floor{};
    floor.normal = { 0.f, 0.f, 1.f };
    floor.relPos = { 0.f, 0.f, -BALL_COLLISION_RADIUS };
    floor.depth = 30.f;
    BallArenaSolverBody body{};
    body.vel = { 0.f, 0.f, -5.f };
    body.velNoExt = body.vel;
    solveBallArenaContacts(body, &floor, 1, ballHitOnPreviousTick(100 - hitAge, 100));
    return body.pushVel.z;
}

void refka_dodge(float pitch, float yaw, float roll, int* flags, float* vel)
{
    GameState state(2, 1, 1, 42);
    Workspace space(2, 2, 4);
    state.cars.internal[0] = {};
    state.cars.vel[0] = Vec3::zero();
    CarControls controls{};
    controls.pitch = pitch;
    controls.yaw = yaw;
    controls.roll = roll;
    state.cars.controls[0] = controls;
    ControlCtx ctx{};
    ctx.state = &state;
    ctx.space = &space;
    ctx.rot = Quat::angle(0.f);
    ctx.fwd = WORLD_X;
    ctx.up = WORLD_Z;
    ctx.jumpPressed = true;
    tryStartDodge(ctx);
    flags[0] = state.cars.internal[0].hasFlipped;
    flags[1] = state.cars.internal[0].hasDoubleJumped;
    vel[0] = state.cars.vel[0].x;
    vel[1] = state.cars.vel[0].y;
    vel[2] = state.cars.vel[0].z;
}

void refka_goal_twice(int sign, int* goals, float* ball)
{
    GameState state(2, 1, 1, 42);
    state.goals[0] = {};
    state.tickCount = 5;
    const Vec3 position = { 0.f, sign * 5500.f, 200.f };
    const Vec3 velocity = { 10.f, sign * 1000.f, -50.f };
    state.ball.pos[0] = position;
    state.ball.vel[0] = velocity;
    detectGoal(&state, 0, position);
    const int firstTick = state.goals[0].tick;
    state.tickCount++;
    detectGoal(&state, 0, position);
    const GoalState g = state.goals[0];
    goals[0] = g.blueScore;
    goals[1] = g.orangeScore;
    goals[2] = g.lastScorer;
    goals[3] = g.tick;
    goals[4] = firstTick;
    ball[0] = (state.ball.pos[0] - position).lenSq();
    ball[1] = (state.ball.vel[0] - velocity).lenSq();
}

int refka_reset_ball_clears_valid()
{
    GameState state(2, 1, 1, 42);
    state.ball.integrationValid[0] = 1;
    resetBall(&state.ball, 0);
    return state.ball.integrationValid[0];
}

void refka_steer_lag(float* out)
{
    GameState state(2, 1, 1, 42);
    Workspace space(2, 2, 4);
    space.susp.steerAngle[0] = .25f;
    state.cars.controls[0] = {};
    ControlCtx ctx{};
    ctx.state = &state;
    ctx.space = &space;
    updateSteer(ctx);
    out[0] = space.susp.steerAnglePrev[0];
    out[1] = space.susp.steerAngle[0];
}

/* Per-sim reset: sim 0 has a scorer, sim 1 does not.  out: [sim][lastScorer,
 * episodeTicks, ballArenaContactTick] then [car][arenaContactTick, wheelSource x4]. */
void refka_reset_after_done(int* out)
{
    GameState state(2, 1, 1, 42);
    Workspace space(2, 2, 4);
    state.tickCount = 77;
    for (int sim = 0; sim < 2; ++sim)
    {
        state.goals[sim] = {};
        state.episodeTicks[sim] = 10;
        state.lastBallTouchTicks[sim] = 77;
        state.ballArenaContactTick[sim] = 77;
    }
    for (int car = 0; car < 4; ++car)
    {
        state.cars.arenaContactTick[car] = 77;
        for (int w = 0; w < NUM_WHEELS; ++w) state.cars.wheelSource[car * NUM_WHEELS + w] = WHEEL_SOURCE_BALL;
    }
    state.goals[0].lastScorer = 1;
    resetAfterDone(&state, &space, 0, 1200, 1200, 0);
    int k = 0;
    for (int sim = 0; sim < 2; ++sim)
    {
        out[k++] = state.goals[sim].lastScorer;
        out[k++] = state.episodeTicks[sim];
        out[k++] = state.ballArenaContactTick[sim];
    }
    for (int car = 0; car < 4; ++car)
    {
        out[k++] = state.cars.arenaContactTick[car];
        for (int w = 0; w < NUM_WHEELS; ++w) out[k++] = state.cars.wheelSource[car * NUM_WHEELS + w];
    }
}

void refka_autoflip(float yaw, float roll, int jump, int contacts, float nx, float ny, float nz, float* out)
{
    GameState state(1, 1, 1, 42);
    Workspace space(1, 2, 2);
    state.cars.internal[0] = {};
    state.cars.vel[0] = Vec3::zero();
    state.cars.ang[0] = Vec3::zero();
    space.ctMan.count[0] = contacts;
    space.ctMan.worldNormal[0] = { nx, ny, nz };
    const Quat tilt = { sinf(roll / 2), 0.f, 0.f, cosf(roll / 2) };
    const Quat rotation = Quat::angle(yaw).comp(tilt);
    ControlCtx ctx{};
    ctx.state = &state;
    ctx.space = &space;
    ctx.rot = rotation;
    ctx.fwd = rotation.toWorld(WORLD_X);
    ctx.up = rotation.toWorld(WORLD_Z);
    ctx.jumpPressed = jump != 0;
    updateAutoFlip(ctx);
    const CarInternalState r = state.cars.internal[0];
    const Vec3 ang = state.cars.ang[0];
    out[0] = (float)r.isAutoFlipping;
    out[1] = r.autoFlipTimer;
    out[2] = ang.dot(rotation.toWorld(WORLD_X));
    out[3] = ang.lenSq();
}

}  // extern "C"
