// Known-answer cases of the reference's own device tests, evaluated on the
// product's physics compiled for the host (same headers as the kernels):
//   jwmccarthy/CARL tests/physics_regressions.cu:19-110 (hit age, floor split
//   suppression, dodge vs double jump table, goal idempotence, steer lag) and
//   tests/turtle_recovery.cu:31-78 (autoflip recovery).
// Each function sets up the same inputs as the reference test and returns the
// quantities the test checks.  TEST INFRASTRUCTURE.
#include "host_intrinsics.h"

#include <cstring>

#include "../../carl_b200/csrc/cb_misc.cuh"

using namespace cb;

extern "C" {

int ka_ball_hit_previous_tick(int hitTick, int tick) { return ballHitPreviousTick(hitTick, tick); }

// Floor contact 30 uu deep, ball falling at 5 uu/s; the hit was `hitAge` ticks ago.
float ka_floor_push_z(int hitAge)
{
    BallContact floor{};
    floor.normal = V3{ 0.f, 0.f, 1.f };
    floor.relPos = V3{ 0.f, 0.f, -BALL_COLLISION_RADIUS };
    floor.depth = 30.f;
    BallBody body{};
    body.vel = V3{ 0.f, 0.f, -5.f };
    body.velNoExt = body.vel;
    solveBallArena(body, &floor, 1, ballHitPreviousTick(100 - hitAge, 100));
    return body.pushVel.z;
}

// Airborne car at rest, no flip used, jump pressed with (pitch, yaw, roll).
void ka_dodge(float pitch, float yaw, float roll, int* flags, float* vel)
{
    Internal s{};
    Susp su{};
    V3 v = v3zero(), a = v3zero();
    Controls c{};
    c.pitch = pitch;
    c.yaw = yaw;
    c.roll = roll;
    ControlCtx x{ s, su, v, a, c, Q4{ 0.f, 0.f, 0.f, 1.f }, axisVec(0), axisVec(2), 0.f, 0.f, 0, false, true, 0,
                  v3zero() };
    updateDodge(x);
    flags[0] = s.hasFlipped;
    flags[1] = s.hasDoubleJumped;
    vel[0] = v.x;
    vel[1] = v.y;
    vel[2] = v.z;
}

// Ball beyond goal line `sign`; goal detection at tick 5 and again at tick 6.
void ka_goal_twice(int sign, int* goals, float* ball)
{
    float words[NSW] = {};
    Soa<int> sims{ words, 1 };
    const V3 pos = { 0.f, sign * 5500.f, 200.f };
    const V3 vel = { 10.f, sign * 1000.f, -50.f };
    sims.setv(S_BPOS, 0, pos);
    sims.setv(S_BVEL, 0, vel);
    detectGoal(sims, 0, pos, 5);
    const int firstTick = sims.n(S_GOALS + G_TICK, 0);
    detectGoal(sims, 0, pos, 6);
    goals[0] = sims.n(S_GOALS + G_BLUE, 0);
    goals[1] = sims.n(S_GOALS + G_ORANGE, 0);
    goals[2] = sims.n(S_GOALS + G_LAST_SCORER, 0);
    goals[3] = sims.n(S_GOALS + G_TICK, 0);
    goals[4] = firstTick;
    const V3 p = sims.v(S_BPOS, 0), q = sims.v(S_BVEL, 0);
    ball[0] = lensq(p - pos);
    ball[1] = lensq(q - vel);
}

// Staged steer angle 0.25, zero input: the lagged value takes the old angle.
void ka_steer_lag(float* out)
{
    Internal s{};
    Susp su{};
    su.steer = .25f;
    V3 v = v3zero(), a = v3zero();
    Controls c{};
    ControlCtx x{ s, su, v, a, c, Q4{ 0.f, 0.f, 0.f, 1.f }, axisVec(0), axisVec(2), 0.f, 0.f, 0, false, false, 0,
                  v3zero() };
    updateSteer(x);
    out[0] = su.steerPrev;
    out[1] = su.steer;
}

// Car yawed by `yaw` and rolled by `roll`; previous manifold: `contacts` points
// with first normal n.  Returns isAutoFlipping, timer, torque about the car's
// forward axis, |angular velocity|^2.
void ka_autoflip(float yaw, float roll, int jump, int contacts, float nx, float ny, float nz, float* out)
{
    const Q4 tilt = { sinf(roll / 2), 0.f, 0.f, cosf(roll / 2) };
    const Q4 rot = qmul(qyaw(yaw), tilt);
    Internal s{};
    Susp su{};
    V3 v = v3zero(), a = v3zero();
    Controls c{};
    ControlCtx x{ s, su, v, a, c, rot, rotate(rot, axisVec(0)), rotate(rot, axisVec(2)), 0.f, 0.f, 0, false,
                  jump != 0, contacts, V3{ nx, ny, nz } };
    updateAutoFlip(x);
    out[0] = (float)s.isAutoFlipping;
    out[1] = s.autoFlipTimer;
    out[2] = dot(a, rotate(rot, axisVec(0)));
    out[3] = lensq(a);
}

}  // extern "C"
