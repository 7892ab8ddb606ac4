// Reset, state injection and output packing on the HBM-resident state.
//
// Per-sim / per-car kernels over the word-major arrays:
//   kickoff reset           include/State/Reset.cuh:8-80 (+ src/Kernels.cu:15-23)
//   auto-reset after done   include/State/Reset.cuh:82-171
//   observations            include/Physics/Observations.cuh:7-317, src/EnvIO.cu:47-80
//   canonical state         include/Physics/Observations.cuh:319-356
//   rewards / dones         include/Physics/Observations.cuh:358-397, src/EnvIO.cu:98-135
//   set ball / car / match, reset pads, restored-contact refresh
//                           src/EnvIO.cu:137-357,603-643
// with the reference's arithmetic.  Sim indices used for seeding are global
// (sim_offset + local), so a sharded run seeds exactly like a single env.
#include "envio.cuh"

#include <cuda_runtime.h>

#include "cb_misc.cuh"

namespace cb {

namespace {

// ---- kickoff ---------------------------------------------------------------------------------

__device__ void resetCarKickoff(const GView& g, long long car, int spot, bool invert)
{
    const float x = invert ? -c_tables.kickX[spot % 5] : c_tables.kickX[spot % 5];
    const float y = invert ? -c_tables.kickY[spot % 5] : c_tables.kickY[spot % 5];
    const float yaw = invert ? c_tables.kickYaw[spot % 5] + PI : c_tables.kickYaw[spot % 5];
    const V3 pos = { x, y, CAR_REST_Z };
    const Q4 rot = qyaw(yaw);
    const GlobSoa& c = g.car;
    c.setv(C_POS, car, pos);
    c.setv(C_VEL, car, v3zero());
    c.setv(C_ANG, car, v3zero());
    c.setq(C_ROT, car, rot);
    c.setv(C_CEN, car, pos + carOffsetWorld(rot));
    c.setv(C_IMP, car, v3zero());
    c.n(C_DEMOED, car) = 0;
    c.f(C_DEMO_TIMER, car) = 0.f;
    c.n(C_CONTACT_IDX, car) = -1;
    c.f(C_CONTACT_CD, car) = 0.f;
    c.n(C_BALL_HIT_TICK, car) = -1;
    c.n(C_BALL_CONTACT_TICK, car) = -1;
    for (int k = 0; k < 8; k++) g.out.n(O_CONTROLS + k, car) = 0;
    for (int w = 0; w < NUM_WHEELS; w++) g.out.n(O_WHEEL_CON + w, car) = 0;
    for (int k = 0; k < NIW; k++) c.n(C_INT + k, car) = 0;
    c.n(C_INT + I_ON_GROUND, car) = 1;
    c.f(C_INT + I_BOOST, car) = BOOST_SPAWN_AMOUNT;
}

__device__ void resetSimKickoff(const GView& g, int sim, int tick)
{
    const uint32_t seed = hash32((uint32_t)g.seed) ^ hash32((uint32_t)(g.simOffset + sim)) ^ hash32((uint32_t)tick);
    const int perm = randomIndex(seed, 120);
    g.sim.setv(S_BPOS, sim, V3{ 0.f, 0.f, BALL_REST_Z });
    g.sim.setv(S_BVEL, sim, v3zero());
    g.sim.setv(S_BANG, sim, v3zero());
    g.sim.n(S_IVALID, sim) = 0;
    for (int team = 0; team < 2; team++)
    {
        const int size = team ? g.nOrange : g.nBlue;
        for (int i = 0; i < size; i++)
        {
            const long long car = (long long)sim * g.nCars + team * g.nBlue + i;
            resetCarKickoff(g, car, c_tables.kickoffPerm[perm][i], team != 0);
        }
    }
}

__global__ void kickoffKernel(GView g, int tick)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim < g.nSim) resetSimKickoff(g, sim, tick);
}

// Fresh env state (RLEnvironment::reset / GameState::reset / Workspace::reset).
__global__ void clearKernel(GView g)
{
    const long long car = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (car < (long long)g.nSim * g.nCars)
    {
        const GlobSoa& c = g.car;
        c.setv(C_IMP, car, v3zero());
        c.n(C_DEMOED, car) = 0;
        c.f(C_DEMO_TIMER, car) = 0.f;
        c.n(C_CONTACT_IDX, car) = -1;
        c.f(C_CONTACT_CD, car) = 0.f;
        c.n(C_BALL_HIT_TICK, car) = -1;
        c.n(C_BALL_CONTACT_TICK, car) = -1;
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            g.out.n(O_WHEEL_SRC + w, car) = WHEEL_NONE;
            g.out.n(O_WHEEL_CON + w, car) = 0;
            c.f(C_LAT + w, car) = 0.f;
            c.f(C_LON + w, car) = 0.f;
        }
        g.out.n(O_ARENA_CONTACT_TICK, car) = -1;
        for (int k = 0; k < NIW; k++) c.n(C_INT + k, car) = 0;
        c.n(C_INT + I_ON_GROUND, car) = 1;
        c.f(C_INT + I_BOOST, car) = BOOST_SPAWN_AMOUNT;
        for (int k = 0; k < NSUW; k++) c.f(C_SUSP + k, car) = 0.f;
        c.n(C_MAN_COUNT, car) = 0;
    }
    const long long sim = car;
    if (sim < g.nSim)
    {
        g.sim.n(S_EP_TICKS, sim) = 0;
        g.sim.n(S_LAST_TOUCH, sim) = 0;
        g.sim.setv(S_BIMP, sim, v3zero());
        g.sim.n(S_IVALID, sim) = 0;
        for (int p = 0; p < NUM_BOOST_PADS; p++) g.sim.f(S_PADS + p, sim) = 0.f;
        for (int k = 0; k < 5; k++) g.sim.n(S_GOALS + k, sim) = 0;
        g.simOut[sim] = -1;
    }
}

// ---- auto-reset after done ------------------------------------------------------------------------

__global__ void resetDonesKernel(GView g, int tick, int maxTicks, int overtimeTicks, int noTouchTicks)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim) return;
    const GlobSoa& S = g.sim;
    const bool overtime = S.n(S_GOALS + G_OVERTIME, sim) != 0;
    const bool scored = S.n(S_GOALS + G_LAST_SCORER, sim) != 0;
    const int ep = S.n(S_EP_TICKS, sim);
    const int sinceTouch = tick - S.n(S_LAST_TOUCH, sim);
    const bool noTouch = noTouchTicks > 0 && sinceTouch >= noTouchTicks;
    const bool overtimeExpired = overtime && ep >= maxTicks + overtimeTicks;
    const bool tickTimeout = ep >= maxTicks;

    if (!overtime && !scored && !noTouch && ep >= maxTicks
        && S.n(S_GOALS + G_BLUE, sim) == S.n(S_GOALS + G_ORANGE, sim))
    {
        S.n(S_GOALS + G_OVERTIME, sim) = 1;
        return;
    }
    if (!(scored || noTouch || overtimeExpired || (!overtime && tickTimeout))) return;

    for (int k = 0; k < 5; k++) S.n(S_GOALS + k, sim) = 0;
    resetSimKickoff(g, sim, tick);
    S.n(S_EP_TICKS, sim) = 0;
    S.n(S_LAST_TOUCH, sim) = tick;
    g.simOut[sim] = -1;
    for (int k = 0; k < g.nCars; k++)
    {
        const long long car = (long long)sim * g.nCars + k;
        const GlobSoa& c = g.car;
        g.out.n(O_ARENA_CONTACT_TICK, car) = -1;
        c.n(C_MAN_COUNT, car) = 0;
        const int zeroed[] = { SU_BRAKE, SU_BRAKE_PREV, SU_THROTTLE, SU_RAW_THROTTLE, SU_HANDBRAKE,
                               SU_STEER, SU_STEER_PREV, SU_ENGINE, SU_ENGINE_PREV };
        for (int z : zeroed) c.f(C_SUSP + z, car) = 0.f;
        c.setv(C_SUSP + SU_JUMP_IMP, car, v3zero());
        c.setv(C_SUSP + SU_ANG_IMP, car, v3zero());
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            g.out.n(O_WHEEL_SRC + w, car) = WHEEL_NONE;
            g.out.n(O_WHEEL_CON + w, car) = 0;
            g.out.f(O_RAY_DIST + w, car) = 0.f;
            for (int a = 0; a < 3; a++) g.out.f(O_RAY_NORMAL + 3 * w + a, car) = 0.f;
            c.f(C_LAT + w, car) = 0.f;
            c.f(C_LON + w, car) = 0.f;
        }
    }
    for (int p = 0; p < NUM_BOOST_PADS; p++) S.f(S_PADS + p, sim) = 0.f;
}

// ---- observations -----------------------------------------------------------------------------------

__device__ __forceinline__ V3 obsVec(V3 v, bool inv) { return inv ? V3{ -v.x, -v.y, v.z } : v; }

__device__ void packCar(const GView& g, long long car, bool inv, float* o, int& k)
{
    const V3 pos = obsVec(g.car.v(C_POS, car), inv);
    const V3 vel = obsVec(g.car.v(C_VEL, car), inv);
    const V3 ang = obsVec(g.car.v(C_ANG, car), inv);
    const Q4 rot = g.car.q(C_ROT, car);
    const V3 fwd = obsVec(rotate(rot, axisVec(0)), inv);
    const V3 up = obsVec(rotate(rot, axisVec(2)), inv);
    o[k++] = pos.x; o[k++] = pos.y; o[k++] = pos.z;
    o[k++] = vel.x; o[k++] = vel.y; o[k++] = vel.z;
    o[k++] = ang.x; o[k++] = ang.y; o[k++] = ang.z;
    o[k++] = fwd.x; o[k++] = fwd.y; o[k++] = fwd.z;
    o[k++] = up.x; o[k++] = up.y; o[k++] = up.z;
    o[k++] = g.car.f(C_INT + I_BOOST, car);
    o[k++] = (float)g.car.n(C_INT + I_ON_GROUND, car);
    o[k++] = (float)(g.car.n(C_DEMOED, car) != 0);
    o[k++] = (float)g.car.n(C_INT + I_HAS_FLIPPED, car);
    o[k++] = (float)g.car.n(C_INT + I_HAS_DOUBLE_JUMPED, car);
    o[k++] = (float)g.car.n(C_INT + I_IS_BOOSTING, car);
}

__device__ void packRelative(const GView& g, long long car, V3 egoPos, V3 egoVel, bool inv, float* o, int& k)
{
    const V3 rp = obsVec(g.car.v(C_POS, car) - egoPos, inv);
    const V3 rv = obsVec(g.car.v(C_VEL, car) - egoVel, inv);
    o[k++] = rp.x; o[k++] = rp.y; o[k++] = rp.z;
    o[k++] = rv.x; o[k++] = rv.y; o[k++] = rv.z;
}

__device__ void normalizeObs(float* o, int nCars)
{
    constexpr float arenaDiagonal = 14692.54f;
    const float scale[3] = { ARENA_MAX_X, ARENA_MAX_Y, ARENA_MAX_Z };
    for (int a = 0; a < 3; a++) o[OBS_POS + a] /= scale[a];
    for (int a = 0; a < 3; a++) o[OBS_VEL + a] /= BALL_MAX_SPEED;
    for (int a = 0; a < 3; a++) o[OBS_ANG + a] /= BALL_MAX_ANG_SPEED;
    for (int car = 0; car < nCars; car++)
    {
        const int off = OBS_BALL + car * OBS_PER_CAR;
        for (int a = 0; a < 3; a++) o[off + OBS_POS + a] /= scale[a];
        for (int a = 0; a < 3; a++) o[off + OBS_VEL + a] /= CAR_MAX_SPEED;
        for (int a = 0; a < 3; a++) o[off + OBS_ANG + a] /= CAR_MAX_ANG_SPEED;
        o[off + OBS_BOOST] /= BOOST_MAX;
    }
    const int distOff = OBS_BALL + nCars * OBS_PER_CAR + NUM_BOOST_PADS;
    for (int p = 0; p < NUM_BOOST_PADS; p++) o[distOff + p] /= arenaDiagonal;
    int rel = distOff + NUM_BOOST_PADS;
    for (int a = 0; a < 3; a++)
    {
        o[rel + a] /= 2.f * scale[a];
        o[rel + OBS_VECTOR_SIZE + a] /= BALL_MAX_SPEED + CAR_MAX_SPEED;
    }
    rel += OBS_RELATIVE_EGO_BALL;
    for (int car = 1; car < nCars; car++)
    {
        for (int a = 0; a < 3; a++)
        {
            o[rel + a] /= 2.f * scale[a];
            o[rel + OBS_VECTOR_SIZE + a] /= 2.f * CAR_MAX_SPEED;
        }
        rel += OBS_RELATIVE_PER_OTHER_CAR;
    }
    for (int goal = 0; goal < 2; goal++)
        for (int a = 0; a < 3; a++) o[rel + goal * OBS_VECTOR_SIZE + a] /= 2.f * scale[a];
}

__global__ void packObsKernel(GView g, float* out, const uint8_t* mask, int obsDim, int invertOrange,
                              int normalize, int previousControls)
{
    const long long agent = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (agent >= (long long)g.nSim * g.nCars) return;
    const int sim = (int)(agent / g.nCars);
    if (mask && !mask[sim]) return;
    const int obs = (int)(agent - (long long)sim * g.nCars);
    const long long base = (long long)sim * g.nCars;
    const bool orange = obs >= g.nBlue;
    const bool inv = invertOrange && orange;
    float* o = out + agent * obsDim;
    int k = 0;

    const V3 rawBallPos = g.sim.v(S_BPOS, sim);
    const V3 rawBallVel = g.sim.v(S_BVEL, sim);
    const V3 egoPos = g.car.v(C_POS, base + obs);
    const V3 egoVel = g.car.v(C_VEL, base + obs);
    const V3 bp = obsVec(rawBallPos, inv), bv = obsVec(rawBallVel, inv), ba = obsVec(g.sim.v(S_BANG, sim), inv);
    o[k++] = bp.x; o[k++] = bp.y; o[k++] = bp.z;
    o[k++] = bv.x; o[k++] = bv.y; o[k++] = bv.z;
    o[k++] = ba.x; o[k++] = ba.y; o[k++] = ba.z;
    packCar(g, base + obs, inv, o, k);

    const int teamStart = orange ? g.nBlue : 0, teamEnd = orange ? g.nCars : g.nBlue;
    const int oppStart = orange ? 0 : g.nBlue, oppEnd = orange ? g.nBlue : g.nCars;
    for (int c = teamStart; c < teamEnd; c++)
        if (c != obs) packCar(g, base + c, inv, o, k);
    for (int c = oppStart; c < oppEnd; c++) packCar(g, base + c, inv, o, k);

    for (int p = 0; p < NUM_BOOST_PADS; p++)
    {
        const int pad = inv ? c_tables.padMirror[p] : p;
        o[k++] = g.sim.f(S_PADS + pad, sim) <= 0.f;
    }
    for (int p = 0; p < NUM_BOOST_PADS; p++)
    {
        const int pad = inv ? c_tables.padMirror[p] : p;
        o[k++] = len(egoPos - V3{ c_tables.padX[pad], c_tables.padY[pad], c_tables.padZ[pad] });
    }
    const V3 eb = obsVec(rawBallPos - egoPos, inv), ebv = obsVec(rawBallVel - egoVel, inv);
    o[k++] = eb.x; o[k++] = eb.y; o[k++] = eb.z;
    o[k++] = ebv.x; o[k++] = ebv.y; o[k++] = ebv.z;
    for (int c = teamStart; c < teamEnd; c++)
        if (c != obs) packRelative(g, base + c, egoPos, egoVel, inv, o, k);
    for (int c = oppStart; c < oppEnd; c++) packRelative(g, base + c, egoPos, egoVel, inv, o, k);

    const float ownGoalY = orange ? SOCCAR_GOAL_CENTER_Y : -SOCCAR_GOAL_CENTER_Y;
    const V3 ownGoal = { 0.f, ownGoalY, SOCCAR_GOAL_CENTER_Z };
    const V3 oppGoal = { 0.f, -ownGoalY, SOCCAR_GOAL_CENTER_Z };
    const V3 bo = obsVec(ownGoal - rawBallPos, inv), bq = obsVec(oppGoal - rawBallPos, inv);
    o[k++] = bo.x; o[k++] = bo.y; o[k++] = bo.z;
    o[k++] = bq.x; o[k++] = bq.y; o[k++] = bq.z;

    const long long ego = base + obs;
    const bool hasFlipped = g.car.n(C_INT + I_HAS_FLIPPED, ego) != 0;
    const bool hasDouble = g.car.n(C_INT + I_HAS_DOUBLE_JUMPED, ego) != 0;
    const float airSinceJump = g.car.f(C_INT + I_AIR_TIME_SINCE_JUMP, ego);
    const bool flipAvailable = !hasFlipped && !hasDouble && airSinceJump < DOUBLEJUMP_MAX_DELAY;
    o[k++] = (float)flipAvailable;
    o[k++] = flipAvailable ? fmaxf(0.f, DOUBLEJUMP_MAX_DELAY - airSinceJump) : 0.f;
    o[k++] = (float)g.car.n(C_INT + I_HAS_JUMPED, ego);
    o[k++] = (float)g.car.n(C_INT + I_IS_JUMPING, ego);
    o[k++] = (float)g.car.n(C_INT + I_IS_FLIPPING, ego);
    o[k++] = g.car.f(C_INT + I_FLIP_TIME, ego);
    o[k++] = g.car.f(C_DEMO_TIMER, ego);
    if (previousControls)
    {
        for (int c = 0; c < 5; c++) o[k++] = g.out.f(O_CONTROLS + c, ego);
        for (int c = 5; c < 8; c++) o[k++] = (float)g.out.n(O_CONTROLS + c, ego);
    }
    if (normalize) normalizeObs(o, g.nCars);
}

__global__ void packStateKernel(GView g, float* out, int stateDim, int tick, int touchWindow, const uint8_t* mask)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim || (mask && !mask[sim])) return;
    float* o = out + (long long)sim * stateDim;
    int k = 0;
    const V3 bp = g.sim.v(S_BPOS, sim), bv = g.sim.v(S_BVEL, sim), ba = g.sim.v(S_BANG, sim);
    o[k++] = bp.x; o[k++] = bp.y; o[k++] = bp.z;
    o[k++] = bv.x; o[k++] = bv.y; o[k++] = bv.z;
    o[k++] = ba.x; o[k++] = ba.y; o[k++] = ba.z;
    for (int c = 0; c < g.nCars; c++)
    {
        const long long car = (long long)sim * g.nCars + c;
        packCar(g, car, false, o, k);
        o[k++] = g.car.n(C_BALL_CONTACT_TICK, car) > tick - touchWindow;
    }
    for (int p = 0; p < NUM_BOOST_PADS; p++) o[k++] = g.sim.f(S_PADS + p, sim) <= 0.f;
}

__global__ void packRewardsDonesKernel(GView g, Outputs out, int tick, int maxTicks, int overtimeTicks, int noTouchTicks)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim) return;
    const GlobSoa& S = g.sim;
    const int blue = S.n(S_GOALS + G_BLUE, sim), orange = S.n(S_GOALS + G_ORANGE, sim);
    const int last = S.n(S_GOALS + G_LAST_SCORER, sim);
    const bool overtime = S.n(S_GOALS + G_OVERTIME, sim) != 0;
    const int ep = S.n(S_EP_TICKS, sim);
    out.rewards[sim] = (float)last;
    const bool regulationExpired = ep >= maxTicks && blue != orange;
    const bool overtimeExpired = overtime && ep >= maxTicks + overtimeTicks;
    const bool gameOver = !overtime && regulationExpired;
    const bool timeout = noTouchTicks > 0 && tick - S.n(S_LAST_TOUCH, sim) >= noTouchTicks;
    out.dones[sim] = (gameOver || overtimeExpired || timeout || last != 0) ? 1 : 0;
    out.transitionScoreDiff[sim] = blue - orange;
    out.transitionEpisodeTicks[sim] = ep;
    out.transitionOvertime[sim] = overtime ? 1 : 0;
}

__global__ void packRawMatchKernel(GView g, Outputs out, const uint8_t* mask)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim || (mask && !mask[sim])) return;
    out.scoreDiff[sim] = g.sim.n(S_GOALS + G_BLUE, sim) - g.sim.n(S_GOALS + G_ORANGE, sim);
    out.episodeTicks[sim] = g.sim.n(S_EP_TICKS, sim);
    out.overtime[sim] = g.sim.n(S_GOALS + G_OVERTIME, sim) != 0 ? 1 : 0;
}

// ---- state injection --------------------------------------------------------------------------------

__device__ __forceinline__ bool selectTarget(const GView& g, int source, const int64_t* indices, const uint8_t* mask,
                                             int& target)
{
    if (mask && !mask[source]) return false;
    const int64_t t = indices ? indices[source] : source;
    if (t < 0 || t >= g.nSim) return false;
    target = (int)t;
    return true;
}

__global__ void setBallKernel(GView g, BallInputs in, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    int sim;
    if (src >= nSelected || !selectTarget(g, src, indices, mask, sim)) return;
    g.sim.setv(S_BPOS, sim, V3{ in.pos[3 * src], in.pos[3 * src + 1], in.pos[3 * src + 2] });
    g.sim.setv(S_BVEL, sim, V3{ in.vel[3 * src], in.vel[3 * src + 1], in.vel[3 * src + 2] });
    g.sim.setv(S_BANG, sim, V3{ in.ang[3 * src], in.ang[3 * src + 1], in.ang[3 * src + 2] });
    g.sim.setv(S_BIMP, sim, v3zero());
}

__global__ void setCarKernel(GView g, CarInputs in, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    if (src >= nSelected * g.nCars) return;
    const int srcSim = src / g.nCars;
    int sim;
    if (!selectTarget(g, srcSim, indices, mask, sim)) return;
    const int local = src - srcSim * g.nCars;
    const long long car = (long long)sim * g.nCars + local;
    const GlobSoa& c = g.car;
    const float previousBoost = c.f(C_INT + I_BOOST, car);
    const V3 pos = { in.pos[3 * src], in.pos[3 * src + 1], in.pos[3 * src + 2] };
    const Q4 rot = { in.rot[4 * src], in.rot[4 * src + 1], in.rot[4 * src + 2], in.rot[4 * src + 3] };
    const int demoed = in.demoedIsByte ? (int)static_cast<const uint8_t*>(in.demoed)[src]
                                       : static_cast<const int32_t*>(in.demoed)[src];
    c.setv(C_POS, car, pos);
    c.setq(C_ROT, car, rot);
    c.setv(C_VEL, car, V3{ in.vel[3 * src], in.vel[3 * src + 1], in.vel[3 * src + 2] });
    c.setv(C_ANG, car, V3{ in.ang[3 * src], in.ang[3 * src + 1], in.ang[3 * src + 2] });
    c.setv(C_CEN, car, pos + carOffsetWorld(rot));
    c.setv(C_IMP, car, v3zero());
    c.n(C_DEMOED, car) = demoed != 0;
    c.f(C_DEMO_TIMER, car) = demoed ? DEMO_RESPAWN_TIME + PHYS_DT : 0.f;
    c.n(C_CONTACT_IDX, car) = -1;
    c.f(C_CONTACT_CD, car) = 0.f;
    c.n(C_BALL_HIT_TICK, car) = -1;
    c.n(C_BALL_CONTACT_TICK, car) = -1;
    for (int k = 0; k < 8; k++) g.out.n(O_CONTROLS + k, car) = 0;

    if (in.internal)
    {
        // CAR_INTERNAL_SIZE record (include/State/GameState.cuh:84-106 order).
        const float* v = in.internal + (long long)src * CAR_INTERNAL_SIZE;
        for (int k = 0; k < NIW; k++) c.n(C_INT + k, car) = 0;
        c.n(C_INT + I_ON_GROUND, car) = v[0] != 0.f;
        c.f(C_INT + I_AIR_TIME_SINCE_JUMP, car) = v[1];
        c.f(C_INT + I_HANDBRAKE, car) = v[2];
        c.n(C_INT + I_HAS_JUMPED, car) = v[3] != 0.f;
        c.n(C_INT + I_IS_JUMPING, car) = v[4] != 0.f;
        c.n(C_INT + I_LAST_JUMP, car) = v[5] != 0.f;
        c.f(C_INT + I_JUMP_TIME, car) = v[6];
        c.n(C_INT + I_HAS_DOUBLE_JUMPED, car) = v[7] != 0.f;
        c.n(C_INT + I_HAS_FLIPPED, car) = v[8] != 0.f;
        c.n(C_INT + I_IS_FLIPPING, car) = v[9] != 0.f;
        c.f(C_INT + I_FLIP_TIME, car) = v[10];
        c.n(C_INT + I_IS_AUTO_FLIPPING, car) = v[11] != 0.f;
        c.f(C_INT + I_AUTO_FLIP_TIMER, car) = v[12];
        c.f(C_INT + I_AUTO_FLIP_SCALE, car) = v[13];
        c.setv(C_INT + I_FLIP_TORQUE, car, V3{ v[14], v[15], v[16] });
        c.n(C_INT + I_IS_BOOSTING, car) = v[17] != 0.f;
        c.f(C_INT + I_BOOSTING_TIME, car) = v[18];
        c.f(C_INT + I_BOOST, car) = in.boost ? fminf(BOOST_MAX, fmaxf(0.f, in.boost[src])) : previousBoost;
    }
    else if (in.boost)
    {
        c.f(C_INT + I_BOOST, car) = fminf(BOOST_MAX, fmaxf(0.f, in.boost[src]));
    }
    g.out.n(O_CONTROLS + 5, car) = c.n(C_INT + I_LAST_JUMP, car);

    c.f(C_SUSP + SU_BRAKE, car) = 0.f;
    c.f(C_SUSP + SU_BRAKE_PREV, car) = 0.f;
    c.f(C_SUSP + SU_THROTTLE, car) = 0.f;
    c.f(C_SUSP + SU_RAW_THROTTLE, car) = 0.f;
    c.f(C_SUSP + SU_HANDBRAKE, car) = in.internal ? in.internal[(long long)src * CAR_INTERNAL_SIZE + 2] : 0.f;
    c.f(C_SUSP + SU_STEER, car) = 0.f;
    c.setv(C_SUSP + SU_JUMP_IMP, car, v3zero());
    c.f(C_SUSP + SU_ENGINE, car) = 0.f;
    c.f(C_SUSP + SU_ENGINE_PREV, car) = 0.f;
    c.n(C_MAN_COUNT, car) = 0;
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        g.out.n(O_WHEEL_CON + w, car) = 0;
        c.f(C_LAT + w, car) = 0.f;
        c.f(C_LON + w, car) = 0.f;
    }
}

// Serial suspension raycast of one car against its grid cell, the other cars
// and the ball (the tick kernel's flattened version gives the same hits).
__device__ void raycastCar(const GView& g, const ArenaDev& a, long long car, int sim, float* dist, V3* normal, int* src)
{
    const GlobSoa& c = g.car;
    const V3 pos = c.v(C_POS, car), vel = c.v(C_VEL, car), ang = c.v(C_ANG, car), cen = c.v(C_CEN, car);
    const Q4 rot = c.q(C_ROT, car);
    const V3 up = rotate(rot, axisVec(2));
    const V3 dir = neg(up);
    V3 start[NUM_WHEELS];
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        start[w] = cen + rotate(rot, suspConnection(w));
        dist[w] = suspRayLength(w) + 1.f;
        normal[w] = up;
        src[w] = WHEEL_NONE;
    }
    const int cell = broadphaseCell(pos, vel, ang, cen, rot);
    for (int e = a.cellStart[cell]; e < a.cellStart[cell + 1]; e++)
    {
        const int tri = a.cellTris[e];
        const float4 p0 = a.triV[3 * tri], p1 = a.triV[3 * tri + 1], p2 = a.triV[3 * tri + 2];
        const V3 v0 = { p0.x, p0.y, p0.z };
        const V3 e1 = V3{ p1.x, p1.y, p1.z } - v0;
        const V3 e2 = V3{ p2.x, p2.y, p2.z } - v0;
        const V3 pv = cross(dir, e2);
        const float det = dot(e1, pv);
        if (fabsf(det) < RAY_PARALLEL_EPS) continue;
        const float invDet = 1.f / det;
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            const V3 tv = start[w] - v0;
            const float u = invDet * dot(tv, pv);
            if (u < 0.f || u > 1.f) continue;
            const V3 qv = cross(tv, e1);
            const float v = invDet * dot(dir, qv);
            if (v < 0.f || u + v > 1.f) continue;
            const float d = invDet * dot(e2, qv);
            if (d <= 0.f || d >= dist[w]) continue;
            dist[w] = d;
            src[w] = WHEEL_ARENA;
            V3 n = cross(e1, e2);
            const float nl = lensq(n);
            if (nl > 1e-12f)
            {
                n = n * rsqrtf(nl);
                if (dot(n, dir) > 0.f) n = neg(n);
                normal[w] = n;
            }
        }
    }
    const long long base = (long long)sim * g.nCars;
    for (int k = 0; k < g.nCars; k++)
    {
        const long long o = base + k;
        if (o == car || c.n(C_DEMOED, o)) continue;
        const V3 oc = c.v(C_CEN, o);
        const Q4 orot = c.q(C_ROT, o);
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            const V3 ls = unrotate(orot, start[w] - oc);
            const V3 ld = unrotate(orot, dir);
            float entry = 0.f, exitD = suspRayLength(w);
            int hitAxis = -1;
            bool miss = false;
            for (int ax = 0; ax < 3; ax++)
            {
                const float h = vget(carHalfExtents(), ax);
                const float d = vget(ld, ax), s0 = vget(ls, ax);
                if (fabsf(d) < RAY_PARALLEL_EPS)
                {
                    if (fabsf(s0) > h) { miss = true; break; }
                    continue;
                }
                const float inv = 1.f / d;
                const float t1 = (-h - s0) * inv;
                const float t2 = (h - s0) * inv;
                const float tn = fminf(t1, t2);
                if (tn > entry) { entry = tn; hitAxis = ax; }
                exitD = fminf(exitD, fmaxf(t1, t2));
                if (entry > exitD) { miss = true; break; }
            }
            if (miss || hitAxis < 0 || entry >= dist[w]) continue;
            V3 ln = v3zero();
            vset(ln, hitAxis, vget(ld, hitAxis) > 0.f ? -1.f : 1.f);
            dist[w] = entry;
            normal[w] = rotate(orot, ln);
            src[w] = WHEEL_CAR;
        }
    }
    const V3 bp = g.sim.v(S_BPOS, sim);
    const float invR = 1.f / BALL_COLLISION_RADIUS;
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        const V3 off = start[w] - bp;
        const float b = dot(off, dir);
        const float cc = lensq(off) - BALL_COLLISION_RADIUS * BALL_COLLISION_RADIUS;
        if (cc < 0.f) continue;
        const float disc = b * b - cc;
        if (disc < 0.f) continue;
        const float d = -b - sqrtf(disc);
        if (!(d > 0.f && d <= suspRayLength(w)) || d >= dist[w]) continue;
        dist[w] = d;
        normal[w] = (start[w] + dir * d - bp) * invR;
        src[w] = WHEEL_BALL;
    }
}

__global__ void refreshContactsKernel(GView g, ArenaDev a, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    if (src >= nSelected * g.nCars) return;
    const int srcSim = src / g.nCars;
    int sim;
    if (!selectTarget(g, srcSim, indices, mask, sim)) return;
    const long long car = (long long)sim * g.nCars + (src - srcSim * g.nCars);
    float dist[NUM_WHEELS];
    V3 normal[NUM_WHEELS];
    int source[NUM_WHEELS];
    const bool demoed = g.car.n(C_DEMOED, car) != 0;
    if (demoed)
    {
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            dist[w] = suspRayLength(w) + 1.f;
            normal[w] = axisVec(2);
            source[w] = WHEEL_NONE;
        }
    }
    else
    {
        raycastCar(g, a, car, sim, dist, normal, source);
    }
    int contacts = 0;
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        const int con = source[w] != WHEEL_NONE && dist[w] <= suspRayLength(w);
        g.out.f(O_RAY_DIST + w, car) = dist[w];
        g.out.setv(O_RAY_NORMAL + 3 * w, car, normal[w]);
        g.out.n(O_WHEEL_SRC + w, car) = source[w];
        g.out.n(O_WHEEL_CON + w, car) = con;
        contacts += con;
    }
    g.car.n(C_INT + I_ON_GROUND, car) = demoed ? 0 : contacts >= 3;
}

__global__ void setMatchKernel(GView g, const int32_t* blue, const int32_t* orange, const int32_t* ticks, int nSelected,
                               const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    int sim;
    if (src >= nSelected || !selectTarget(g, src, indices, mask, sim)) return;
    g.sim.n(S_GOALS + G_BLUE, sim) = blue[src];
    g.sim.n(S_GOALS + G_ORANGE, sim) = orange[src];
    g.sim.n(S_GOALS + G_LAST_SCORER, sim) = 0;
    g.sim.n(S_GOALS + G_OVERTIME, sim) = 0;
    g.sim.n(S_EP_TICKS, sim) = ticks[src];
}

__global__ void resetPadsKernel(GView g, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    int sim;
    if (src >= nSelected || !selectTarget(g, src, indices, mask, sim)) return;
    for (int p = 0; p < NUM_BOOST_PADS; p++) g.sim.f(S_PADS + p, sim) = 0.f;
}

inline int blocks(long long n, int t) { return (int)((n + t - 1) / t); }

}  // namespace

int uploadEnvioTables(const Tables& t) { return (int)cudaMemcpyToSymbol(c_tables, &t, sizeof(Tables)); }

void launchClear(const GView& g, cudaStream_t s)
{
    const long long n = (long long)g.nSim * g.nCars;
    clearKernel<<<blocks(n > g.nSim ? n : g.nSim, 256), 256, 0, s>>>(g);
}
void launchKickoff(const GView& g, int tick, cudaStream_t s) { kickoffKernel<<<blocks(g.nSim, 128), 128, 0, s>>>(g, tick); }
void launchResetDones(const GView& g, int tick, int maxTicks, int ot, int nt, cudaStream_t s)
{
    resetDonesKernel<<<blocks(g.nSim, 128), 128, 0, s>>>(g, tick, maxTicks, ot, nt);
}
void launchPackObs(const GView& g, float* out, const uint8_t* mask, int obsDim, bool invert, bool normalize, bool prev,
                   cudaStream_t s)
{
    packObsKernel<<<blocks((long long)g.nSim * g.nCars, 128), 128, 0, s>>>(g, out, mask, obsDim, invert, normalize, prev);
}
void launchPackState(const GView& g, float* out, int stateDim, int tick, int touchWindow, const uint8_t* mask, cudaStream_t s)
{
    packStateKernel<<<blocks(g.nSim, 128), 128, 0, s>>>(g, out, stateDim, tick, touchWindow, mask);
}
void launchPackRewardsDones(const GView& g, const Outputs& o, int tick, int maxTicks, int ot, int nt, cudaStream_t s)
{
    packRewardsDonesKernel<<<blocks(g.nSim, 128), 128, 0, s>>>(g, o, tick, maxTicks, ot, nt);
}
void launchPackRawMatch(const GView& g, const Outputs& o, const uint8_t* mask, cudaStream_t s)
{
    packRawMatchKernel<<<blocks(g.nSim, 128), 128, 0, s>>>(g, o, mask);
}
void launchSetBall(const GView& g, const BallInputs& in, int n, const int64_t* idx, const uint8_t* mask, cudaStream_t s)
{
    if (n > 0) setBallKernel<<<blocks(n, 128), 128, 0, s>>>(g, in, n, idx, mask);
}
void launchSetCar(const GView& g, const ArenaDev& a, const CarInputs& in, int n, const int64_t* idx, const uint8_t* mask,
                  cudaStream_t s)
{
    if (n <= 0) return;
    setCarKernel<<<blocks((long long)n * g.nCars, 256), 256, 0, s>>>(g, in, n, idx, mask);
    refreshContactsKernel<<<blocks((long long)n * g.nCars, 256), 256, 0, s>>>(g, a, n, idx, mask);
}
void launchSetMatch(const GView& g, const int32_t* b, const int32_t* o, const int32_t* t, int n, const int64_t* idx,
                    const uint8_t* mask, cudaStream_t s)
{
    if (n > 0) setMatchKernel<<<blocks(n, 128), 128, 0, s>>>(g, b, o, t, n, idx, mask);
}
void launchResetPads(const GView& g, int n, const int64_t* idx, const uint8_t* mask, cudaStream_t s)
{
    if (n > 0) resetPadsKernel<<<blocks(n, 128), 128, 0, s>>>(g, n, idx, mask);
}

}  // namespace cb
