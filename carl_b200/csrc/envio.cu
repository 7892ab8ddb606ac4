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

// Auto-reset of one sim after its episode ended (src/RLEnvironment.cu:192-219,
// State/Reset.cuh resetAfterDone): overtime starts on a tied regulation end,
// otherwise a scored, timed-out or untouched episode restarts from a kickoff.
__device__ void resetDoneSim(const GView& g, int sim, int tick, int maxTicks, int overtimeTicks, int noTouchTicks)
{
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

__global__ void resetDonesKernel(GView g, int tick, int maxTicks, int overtimeTicks, int noTouchTicks)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim) return;
    resetDoneSim(g, sim, tick, maxTicks, overtimeTicks, noTouchTicks);
}

// ---- observations -----------------------------------------------------------------------------------

__device__ __forceinline__ V3 obsVec(V3 v, bool inv) { return inv ? V3{ -v.x, -v.y, v.z } : v; }

// Output rows (obs, state) are produced by one row function per kind, written
// through an emitter: put(v) appends v, putN(v, d) appends v / d when the row is
// normalised (the division the reference applies in place after packing,
// Observations.cuh normalizeObservations), else v.

// Emitter writing a row straight to memory (one thread per row).
struct DirectRow
{
    float* o;
    int k;
    bool normalize;
    __device__ void put(float v) { o[k++] = v; }
    __device__ void putN(float v, float d) { o[k++] = normalize ? v / d : v; }
};

// Emitter of a warp that writes 32 rows of rowLen floats lying back to back in
// memory (row r at out + r * rowLen, lane r produces row r).  Values go to a
// per-warp tile, 32 columns at a time; a full tile is written as 32 runs of
// consecutive floats, one row each, so every store of the warp is one coalesced
// run instead of 32 scattered words.  All 32 lanes must emit the same number of
// values in the same order; rows whose bit in `rows` is clear are not written.
struct WarpRows
{
    float (*tile)[33];
    float* out;
    int rowLen, lane, k;
    unsigned rows;
    bool normalize;
    __device__ void put(float v)
    {
        tile[lane][k & 31] = v;
        if ((++k & 31) == 0) flush(32);
    }
    __device__ void putN(float v, float d) { put(normalize ? v / d : v); }
    __device__ void finish()
    {
        if (k & 31) flush(k & 31);
    }
    __device__ void flush(int n)
    {
        __syncwarp();
        const int c0 = k - n;
        if (lane < n)
        {
            #pragma unroll 4
            for (int r = 0; r < 32; r++)
                if ((rows >> r) & 1u) out[(long long)r * rowLen + c0 + lane] = tile[r][lane];
        }
        __syncwarp();
    }
};

constexpr float OBS_ARENA_DIAGONAL = 14692.54f;

__device__ __forceinline__ float arenaScale(int a) { return a == 0 ? ARENA_MAX_X : a == 1 ? ARENA_MAX_Y : ARENA_MAX_Z; }

// Every segment of a row loads its words before it emits anything: an emitter
// may store to global memory, and a load placed after a store it might alias
// cannot be hoisted, so loads interleaved with emits would each wait a full
// memory round trip.

// One car block (OBS_PER_CAR values): pose, velocities, axes, boost and flags.
template <class E>
__device__ void emitCar(const GView& g, long long car, bool inv, E& e)
{
    const V3 rawPos = g.car.v(C_POS, car), rawVel = g.car.v(C_VEL, car), rawAng = g.car.v(C_ANG, car);
    const Q4 rot = g.car.q(C_ROT, car);
    const float boost = g.car.f(C_INT + I_BOOST, car);
    const int onGround = g.car.n(C_INT + I_ON_GROUND, car), demoed = g.car.n(C_DEMOED, car);
    const int flipped = g.car.n(C_INT + I_HAS_FLIPPED, car), doubled = g.car.n(C_INT + I_HAS_DOUBLE_JUMPED, car);
    const int boosting = g.car.n(C_INT + I_IS_BOOSTING, car);
    const V3 pos = obsVec(rawPos, inv), vel = obsVec(rawVel, inv), ang = obsVec(rawAng, inv);
    const V3 fwd = obsVec(rotate(rot, axisVec(0)), inv);
    const V3 up = obsVec(rotate(rot, axisVec(2)), inv);
    e.putN(pos.x, arenaScale(0)); e.putN(pos.y, arenaScale(1)); e.putN(pos.z, arenaScale(2));
    e.putN(vel.x, CAR_MAX_SPEED); e.putN(vel.y, CAR_MAX_SPEED); e.putN(vel.z, CAR_MAX_SPEED);
    e.putN(ang.x, CAR_MAX_ANG_SPEED); e.putN(ang.y, CAR_MAX_ANG_SPEED); e.putN(ang.z, CAR_MAX_ANG_SPEED);
    e.put(fwd.x); e.put(fwd.y); e.put(fwd.z);
    e.put(up.x); e.put(up.y); e.put(up.z);
    e.putN(boost, BOOST_MAX);
    e.put((float)onGround);
    e.put((float)(demoed != 0));
    e.put((float)flipped);
    e.put((float)doubled);
    e.put((float)boosting);
}

// The sim's pad cooldowns in emission order (mirrored for an inverted row).
__device__ __forceinline__ void loadPads(const GView& g, int sim, bool inv, float* cd)
{
    #pragma unroll
    for (int p = 0; p < NUM_BOOST_PADS; p++) cd[p] = g.sim.f(S_PADS + (inv ? c_tables.padMirror[p] : p), sim);
}

// j-th other car of `obs` (0 <= j < nCars - 1): its teammates in car order, then
// the opponents in car order.
__device__ __forceinline__ int otherCar(const GView& g, int obs, int j)
{
    const bool orange = obs >= g.nBlue;
    const int teamStart = orange ? g.nBlue : 0, teamSize = orange ? g.nCars - g.nBlue : g.nBlue;
    const int oppStart = orange ? 0 : g.nBlue;
    if (j < teamSize - 1)
    {
        const int c = teamStart + j;
        return c >= obs ? c + 1 : c;
    }
    return oppStart + (j - (teamSize - 1));
}

// Observation row of car `obs` of `sim` (src/EnvIO.cu:47-80, Observations.cuh:97-317).
template <class E>
__device__ void emitObsRow(const GView& g, E& e, int invertOrange, int previousControls, int sim, int obs)
{
    const long long base = (long long)sim * g.nCars;
    const bool orange = obs >= g.nBlue;
    const bool inv = invertOrange && orange;
    const V3 rawBallPos = g.sim.v(S_BPOS, sim);
    const V3 rawBallVel = g.sim.v(S_BVEL, sim);
    const V3 egoPos = g.car.v(C_POS, base + obs);
    const V3 egoVel = g.car.v(C_VEL, base + obs);
    const V3 bp = obsVec(rawBallPos, inv), bv = obsVec(rawBallVel, inv), ba = obsVec(g.sim.v(S_BANG, sim), inv);
    e.putN(bp.x, arenaScale(0)); e.putN(bp.y, arenaScale(1)); e.putN(bp.z, arenaScale(2));
    e.putN(bv.x, BALL_MAX_SPEED); e.putN(bv.y, BALL_MAX_SPEED); e.putN(bv.z, BALL_MAX_SPEED);
    e.putN(ba.x, BALL_MAX_ANG_SPEED); e.putN(ba.y, BALL_MAX_ANG_SPEED); e.putN(ba.z, BALL_MAX_ANG_SPEED);
    emitCar(g, base + obs, inv, e);
    for (int j = 0; j < g.nCars - 1; j++) emitCar(g, base + otherCar(g, obs, j), inv, e);

    float cd[NUM_BOOST_PADS];
    loadPads(g, sim, inv, cd);
    #pragma unroll
    for (int p = 0; p < NUM_BOOST_PADS; p++) e.put(cd[p] <= 0.f);
    for (int p = 0; p < NUM_BOOST_PADS; p++)
    {
        const int pad = inv ? c_tables.padMirror[p] : p;
        e.putN(len(egoPos - V3{ c_tables.padX[pad], c_tables.padY[pad], c_tables.padZ[pad] }), OBS_ARENA_DIAGONAL);
    }
    const V3 eb = obsVec(rawBallPos - egoPos, inv), ebv = obsVec(rawBallVel - egoVel, inv);
    e.putN(eb.x, 2.f * arenaScale(0)); e.putN(eb.y, 2.f * arenaScale(1)); e.putN(eb.z, 2.f * arenaScale(2));
    e.putN(ebv.x, BALL_MAX_SPEED + CAR_MAX_SPEED); e.putN(ebv.y, BALL_MAX_SPEED + CAR_MAX_SPEED);
    e.putN(ebv.z, BALL_MAX_SPEED + CAR_MAX_SPEED);
    for (int j = 0; j < g.nCars - 1; j++)
    {
        const long long car = base + otherCar(g, obs, j);
        const V3 op = g.car.v(C_POS, car), ov = g.car.v(C_VEL, car);
        const V3 rp = obsVec(op - egoPos, inv);
        const V3 rv = obsVec(ov - egoVel, inv);
        e.putN(rp.x, 2.f * arenaScale(0)); e.putN(rp.y, 2.f * arenaScale(1)); e.putN(rp.z, 2.f * arenaScale(2));
        e.putN(rv.x, 2.f * CAR_MAX_SPEED); e.putN(rv.y, 2.f * CAR_MAX_SPEED); e.putN(rv.z, 2.f * CAR_MAX_SPEED);
    }

    const long long ego = base + obs;
    const bool hasFlipped = g.car.n(C_INT + I_HAS_FLIPPED, ego) != 0;
    const bool hasDouble = g.car.n(C_INT + I_HAS_DOUBLE_JUMPED, ego) != 0;
    const float airSinceJump = g.car.f(C_INT + I_AIR_TIME_SINCE_JUMP, ego);
    const int hasJumped = g.car.n(C_INT + I_HAS_JUMPED, ego), isJumping = g.car.n(C_INT + I_IS_JUMPING, ego);
    const int isFlipping = g.car.n(C_INT + I_IS_FLIPPING, ego);
    const float flipTime = g.car.f(C_INT + I_FLIP_TIME, ego), demoTimer = g.car.f(C_DEMO_TIMER, ego);
    float prev[8];
    if (previousControls)
    {
        #pragma unroll
        for (int c = 0; c < 5; c++) prev[c] = g.out.f(O_CONTROLS + c, ego);
        #pragma unroll
        for (int c = 5; c < 8; c++) prev[c] = (float)g.out.n(O_CONTROLS + c, ego);
    }

    const float ownGoalY = orange ? SOCCAR_GOAL_CENTER_Y : -SOCCAR_GOAL_CENTER_Y;
    const V3 ownGoal = { 0.f, ownGoalY, SOCCAR_GOAL_CENTER_Z };
    const V3 oppGoal = { 0.f, -ownGoalY, SOCCAR_GOAL_CENTER_Z };
    const V3 bo = obsVec(ownGoal - rawBallPos, inv), bq = obsVec(oppGoal - rawBallPos, inv);
    e.putN(bo.x, 2.f * arenaScale(0)); e.putN(bo.y, 2.f * arenaScale(1)); e.putN(bo.z, 2.f * arenaScale(2));
    e.putN(bq.x, 2.f * arenaScale(0)); e.putN(bq.y, 2.f * arenaScale(1)); e.putN(bq.z, 2.f * arenaScale(2));

    const bool flipAvailable = !hasFlipped && !hasDouble && airSinceJump < DOUBLEJUMP_MAX_DELAY;
    e.put((float)flipAvailable);
    e.put(flipAvailable ? fmaxf(0.f, DOUBLEJUMP_MAX_DELAY - airSinceJump) : 0.f);
    e.put((float)hasJumped);
    e.put((float)isJumping);
    e.put((float)isFlipping);
    e.put(flipTime);
    e.put(demoTimer);
    if (previousControls)
    {
        #pragma unroll
        for (int c = 0; c < 8; c++) e.put(prev[c]);
    }
}

// Canonical state row of `sim` (Observations.cuh:320-356): ball, each car's
// block and ball-touch flag (a touch within `touchWindow` ticks), pad states.
template <class E>
__device__ void emitStateRow(const GView& g, E& e, int tick, int touchWindow, int sim)
{
    const V3 bp = g.sim.v(S_BPOS, sim), bv = g.sim.v(S_BVEL, sim), ba = g.sim.v(S_BANG, sim);
    e.put(bp.x); e.put(bp.y); e.put(bp.z);
    e.put(bv.x); e.put(bv.y); e.put(bv.z);
    e.put(ba.x); e.put(ba.y); e.put(ba.z);
    for (int c = 0; c < g.nCars; c++)
    {
        const long long car = (long long)sim * g.nCars + c;
        const int touchTick = g.car.n(C_BALL_CONTACT_TICK, car);
        emitCar(g, car, false, e);
        e.put(touchTick > tick - touchWindow);
    }
    float cd[NUM_BOOST_PADS];
    loadPads(g, sim, false, cd);
    #pragma unroll
    for (int p = 0; p < NUM_BOOST_PADS; p++) e.put(cd[p] <= 0.f);
}

__device__ void packObsAgent(const GView& g, float* out, int obsDim, int invertOrange, int normalize,
                             int previousControls, int sim, int obs)
{
    DirectRow e{ out + ((long long)sim * g.nCars + obs) * obsDim, 0, normalize != 0 };
    emitObsRow(g, e, invertOrange, previousControls, sim, obs);
}

__device__ void packStateSim(const GView& g, float* out, int stateDim, int tick, int touchWindow, int sim)
{
    DirectRow e{ out + (long long)sim * stateDim, 0, false };
    emitStateRow(g, e, tick, touchWindow, sim);
}

constexpr int PACK_THREADS = 128;

// One thread per row, written directly.
__global__ void packObsKernel(GView g, float* out, const uint8_t* mask, int obsDim, int invertOrange,
                              int normalize, int previousControls)
{
    const long long agent = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (agent >= (long long)g.nSim * g.nCars) return;
    const int sim = (int)(agent / g.nCars);
    if (mask && !mask[sim]) return;
    packObsAgent(g, out, obsDim, invertOrange, normalize, previousControls, sim, (int)(agent - (long long)sim * g.nCars));
}

__global__ void packStateKernel(GView g, float* out, int stateDim, int tick, int touchWindow, const uint8_t* mask)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim || (mask && !mask[sim])) return;
    packStateSim(g, out, stateDim, tick, touchWindow, sim);
}

// A warp per 32 consecutive rows, written through the warp's staging tile.
// Lanes past the end or outside the mask produce a clamped row that is not
// written; a warp with no row to write returns at once.
__global__ void __launch_bounds__(PACK_THREADS, 6) packObsWarpKernel(GView g, float* out, const uint8_t* mask, int obsDim,
                                                                  int invertOrange, int normalize, int previousControls)
{
    __shared__ float tile[PACK_THREADS / 32][32][33];
    const long long n = (long long)g.nSim * g.nCars;
    const long long agent = blockIdx.x * (long long)PACK_THREADS + threadIdx.x;
    const long long a = agent < n ? agent : n - 1;
    const int sim = (int)(a / g.nCars);
    const bool write = agent < n && (!mask || mask[sim]);
    const unsigned rows = __ballot_sync(0xffffffffu, write);
    if (!rows) return;
    const int lane = threadIdx.x & 31;
    WarpRows e{ tile[threadIdx.x >> 5], out + (agent - lane) * obsDim, obsDim, lane, 0, rows, normalize != 0 };
    emitObsRow(g, e, invertOrange, previousControls, sim, (int)(a - (long long)sim * g.nCars));
    e.finish();
}

__global__ void __launch_bounds__(PACK_THREADS) packStateWarpKernel(GView g, float* out, int stateDim, int tick,
                                                                    int touchWindow, const uint8_t* mask)
{
    __shared__ float tile[PACK_THREADS / 32][32][33];
    const int s = blockIdx.x * PACK_THREADS + threadIdx.x;
    const int sim = s < g.nSim ? s : g.nSim - 1;
    const bool write = s < g.nSim && (!mask || mask[sim]);
    const unsigned rows = __ballot_sync(0xffffffffu, write);
    if (!rows) return;
    const int lane = threadIdx.x & 31;
    WarpRows e{ tile[threadIdx.x >> 5], out + (long long)(s - lane) * stateDim, stateDim, lane, 0, rows, false };
    emitStateRow(g, e, tick, touchWindow, sim);
    e.finish();
}

// Whether a sim's episode is over (Observations.cuh:360-397 packDones): a goal,
// regulation time with a winner, expired overtime or the no-touch timeout.
__device__ bool simDone(const GView& g, int sim, int tick, int maxTicks, int overtimeTicks, int noTouchTicks)
{
    const GlobSoa& S = g.sim;
    const int blue = S.n(S_GOALS + G_BLUE, sim), orange = S.n(S_GOALS + G_ORANGE, sim);
    const int last = S.n(S_GOALS + G_LAST_SCORER, sim);
    const bool overtime = S.n(S_GOALS + G_OVERTIME, sim) != 0;
    const int ep = S.n(S_EP_TICKS, sim);
    const bool regulationExpired = ep >= maxTicks && blue != orange;
    const bool overtimeExpired = overtime && ep >= maxTicks + overtimeTicks;
    const bool gameOver = !overtime && regulationExpired;
    const bool timeout = noTouchTicks > 0 && tick - S.n(S_LAST_TOUCH, sim) >= noTouchTicks;
    return gameOver || overtimeExpired || timeout || last != 0;
}

// Reward, done and transition match outputs of one sim (Observations.cuh:360-397).
__device__ void packRewardsDonesSim(const GView& g, const Outputs& out, int sim, int tick, int maxTicks,
                                    int overtimeTicks, int noTouchTicks)
{
    const GlobSoa& S = g.sim;
    const int blue = S.n(S_GOALS + G_BLUE, sim), orange = S.n(S_GOALS + G_ORANGE, sim);
    const bool overtime = S.n(S_GOALS + G_OVERTIME, sim) != 0;
    const int ep = S.n(S_EP_TICKS, sim);
    out.rewards[sim] = (float)S.n(S_GOALS + G_LAST_SCORER, sim);
    out.dones[sim] = simDone(g, sim, tick, maxTicks, overtimeTicks, noTouchTicks) ? 1 : 0;
    out.transitionScoreDiff[sim] = blue - orange;
    out.transitionEpisodeTicks[sim] = ep;
    out.transitionOvertime[sim] = overtime ? 1 : 0;
}

__global__ void packRewardsDonesKernel(GView g, Outputs out, int tick, int maxTicks, int overtimeTicks, int noTouchTicks)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim) return;
    packRewardsDonesSim(g, out, sim, tick, maxTicks, overtimeTicks, noTouchTicks);
}

__device__ void packRawMatchSim(const GView& g, const Outputs& out, int sim)
{
    out.scoreDiff[sim] = g.sim.n(S_GOALS + G_BLUE, sim) - g.sim.n(S_GOALS + G_ORANGE, sim);
    out.episodeTicks[sim] = g.sim.n(S_EP_TICKS, sim);
    out.overtime[sim] = g.sim.n(S_GOALS + G_OVERTIME, sim) != 0 ? 1 : 0;
}

__global__ void packRawMatchKernel(GView g, Outputs out, const uint8_t* mask)
{
    const int sim = blockIdx.x * blockDim.x + threadIdx.x;
    if (sim >= g.nSim || (mask && !mask[sim])) return;
    packRawMatchSim(g, out, sim);
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

// Input row `src` written to `sim` (src/EnvIO.cu:137-318,603-680).
__device__ void setBallSim(const GView& g, const BallInputs& in, int src, int sim)
{
    g.sim.setv(S_BPOS, sim, V3{ in.pos[3 * src], in.pos[3 * src + 1], in.pos[3 * src + 2] });
    g.sim.setv(S_BVEL, sim, V3{ in.vel[3 * src], in.vel[3 * src + 1], in.vel[3 * src + 2] });
    g.sim.setv(S_BANG, sim, V3{ in.ang[3 * src], in.ang[3 * src + 1], in.ang[3 * src + 2] });
    g.sim.setv(S_BIMP, sim, v3zero());
}

__global__ void setBallKernel(GView g, BallInputs in, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    int sim;
    if (src >= nSelected || !selectTarget(g, src, indices, mask, sim)) return;
    setBallSim(g, in, src, sim);
}

// Input row `src` (= input sim × nCars + local) written to car `local` of `sim`.
__device__ void setCarOne(const GView& g, const CarInputs& in, int src, int sim, int local)
{
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

__global__ void setCarKernel(GView g, CarInputs in, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    if (src >= nSelected * g.nCars) return;
    const int srcSim = src / g.nCars;
    int sim;
    if (!selectTarget(g, srcSim, indices, mask, sim)) return;
    setCarOne(g, in, src, sim, src - srcSim * g.nCars);
}

// Wheel ray set-up of one car: ray starts, direction (-up), the car's up axis
// and its broadphase cell.
struct CarRays
{
    V3 start[NUM_WHEELS];
    V3 dir, up;
    int cell;
};

__device__ CarRays carRays(const GView& g, long long car)
{
    const GlobSoa& c = g.car;
    const V3 pos = c.v(C_POS, car), vel = c.v(C_VEL, car), ang = c.v(C_ANG, car), cen = c.v(C_CEN, car);
    const Q4 rot = c.q(C_ROT, car);
    CarRays r;
    r.up = rotate(rot, axisVec(2));
    r.dir = neg(r.up);
    for (int w = 0; w < NUM_WHEELS; w++) r.start[w] = cen + rotate(rot, suspConnection(w));
    r.cell = broadphaseCell(pos, vel, ang, cen, rot);
    return r;
}

// Möller–Trumbore hit distance of a wheel ray against a triangle given by v0
// and its edges (pv = dir × e2, invDet = 1 / (e1 · pv)); false when missed or
// not closer than `limit`.
__device__ __forceinline__ bool wheelTriHit(V3 start, V3 dir, V3 v0, V3 e1, V3 e2, V3 pv, float invDet, float limit,
                                            float& d)
{
    const V3 tv = start - v0;
    const float u = invDet * dot(tv, pv);
    if (u < 0.f || u > 1.f) return false;
    const V3 qv = cross(tv, e1);
    const float v = invDet * dot(dir, qv);
    if (v < 0.f || u + v > 1.f) return false;
    d = invDet * dot(e2, qv);
    return !(d <= 0.f || d >= limit);
}

// Serial arena pass of the wheel rays over the cell's triangles in candidate
// order (a strictly closer hit replaces the previous one; a degenerate winning
// triangle keeps the previous normal).  Wheels outside [w0, w1) are untouched.
__device__ void arenaRaysSerial(const ArenaDev& a, const CarRays& r, int w0, int w1, float* dist, V3* normal, int* src)
{
    for (int e = a.cellStart[r.cell]; e < a.cellStart[r.cell + 1]; e++)
    {
        const int tri = a.cellTris[e];
        const float4 p0 = a.triV[3 * tri], p1 = a.triV[3 * tri + 1], p2 = a.triV[3 * tri + 2];
        const V3 v0 = { p0.x, p0.y, p0.z };
        const V3 e1 = V3{ p1.x, p1.y, p1.z } - v0;
        const V3 e2 = V3{ p2.x, p2.y, p2.z } - v0;
        const V3 pv = cross(r.dir, e2);
        const float det = dot(e1, pv);
        if (fabsf(det) < RAY_PARALLEL_EPS) continue;
        const float invDet = 1.f / det;
        for (int w = w0; w < w1; w++)
        {
            float d;
            if (!wheelTriHit(r.start[w], r.dir, v0, e1, e2, pv, invDet, dist[w], d)) continue;
            dist[w] = d;
            src[w] = WHEEL_ARENA;
            V3 n = cross(e1, e2);
            const float nl = lensq(n);
            if (nl > 1e-12f)
            {
                n = n * rsqrtf(nl);
                if (dot(n, r.dir) > 0.f) n = neg(n);
                normal[w] = n;
            }
        }
    }
}

__device__ void initWheelRays(const CarRays& r, float* dist, V3* normal, int* src)
{
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        dist[w] = suspRayLength(w) + 1.f;
        normal[w] = r.up;
        src[w] = WHEEL_NONE;
    }
}

// The wheel rays against the sim's other cars (in car order) and the ball,
// after the arena pass.
__device__ void carBallRays(const GView& g, long long car, int sim, const CarRays& r, float* dist, V3* normal, int* src)
{
    const GlobSoa& c = g.car;
    const V3* start = r.start;
    const V3 dir = r.dir;
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

// Serial suspension raycast of one car against its grid cell, the other cars
// and the ball (the tick kernel's flattened version gives the same hits).
__device__ void raycastCar(const GView& g, const ArenaDev& a, long long car, int sim, float* dist, V3* normal, int* src)
{
    const CarRays r = carRays(g, car);
    initWheelRays(r, dist, normal, src);
    arenaRaysSerial(a, r, 0, NUM_WHEELS, dist, normal, src);
    carBallRays(g, car, sim, r, dist, normal, src);
}

// Stores the wheel ray results and the on-ground flag of a restored car.
__device__ void storeRefresh(const GView& g, long long car, bool demoed, const float* dist, const V3* normal,
                             const int* source)
{
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

__device__ void demoedWheelRays(float* dist, V3* normal, int* source)
{
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        dist[w] = suspRayLength(w) + 1.f;
        normal[w] = axisVec(2);
        source[w] = WHEEL_NONE;
    }
}

// Wheel contacts and on-ground flag of a restored car (refreshRestoredCarContacts).
__device__ void refreshCarOne(const GView& g, const ArenaDev& a, int sim, int local)
{
    const long long car = (long long)sim * g.nCars + local;
    float dist[NUM_WHEELS];
    V3 normal[NUM_WHEELS];
    int source[NUM_WHEELS];
    const bool demoed = g.car.n(C_DEMOED, car) != 0;
    if (demoed) demoedWheelRays(dist, normal, source);
    else raycastCar(g, a, car, sim, dist, normal, source);
    storeRefresh(g, car, demoed, dist, normal, source);
}

__global__ void refreshContactsKernel(GView g, ArenaDev a, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    if (src >= nSelected * g.nCars) return;
    const int srcSim = src / g.nCars;
    int sim;
    if (!selectTarget(g, srcSim, indices, mask, sim)) return;
    refreshCarOne(g, a, sim, src - srcSim * g.nCars);
}

__device__ void setMatchSim(const GView& g, const int32_t* blue, const int32_t* orange, const int32_t* ticks, int src,
                            int sim)
{
    g.sim.n(S_GOALS + G_BLUE, sim) = blue[src];
    g.sim.n(S_GOALS + G_ORANGE, sim) = orange[src];
    g.sim.n(S_GOALS + G_LAST_SCORER, sim) = 0;
    g.sim.n(S_GOALS + G_OVERTIME, sim) = 0;
    g.sim.n(S_EP_TICKS, sim) = ticks[src];
}

__global__ void setMatchKernel(GView g, const int32_t* blue, const int32_t* orange, const int32_t* ticks, int nSelected,
                               const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    int sim;
    if (src >= nSelected || !selectTarget(g, src, indices, mask, sim)) return;
    setMatchSim(g, blue, orange, ticks, src, sim);
}

__device__ void resetPadsSim(const GView& g, int sim)
{
    for (int p = 0; p < NUM_BOOST_PADS; p++) g.sim.f(S_PADS + p, sim) = 0.f;
}

__global__ void resetPadsKernel(GView g, int nSelected, const int64_t* indices, const uint8_t* mask)
{
    const int src = blockIdx.x * blockDim.x + threadIdx.x;
    int sim;
    if (src >= nSelected || !selectTarget(g, src, indices, mask, sim)) return;
    resetPadsSim(g, sim);
}

// Emitter of a warp that writes 32 rows of rowLen floats at per-lane row
// addresses (lane r's row at `row`), through the same per-warp tile as WarpRows:
// each store of the warp is a run of consecutive floats of one row.  All lanes
// emit the same sequence; rows whose bit in `rows` is clear are not written.
struct WarpRowsAt
{
    float (*tile)[33];
    float* row;
    int lane, k;
    unsigned rows;
    bool normalize;
    __device__ void put(float v)
    {
        tile[lane][k & 31] = v;
        if ((++k & 31) == 0) flush(32);
    }
    __device__ void putN(float v, float d) { put(normalize ? v / d : v); }
    __device__ void finish()
    {
        if (k & 31) flush(k & 31);
    }
    __device__ void flush(int n)
    {
        __syncwarp();
        const int c0 = k - n;
        for (int r = 0; r < 32; r++)
        {
            float* dst = reinterpret_cast<float*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(row), r));
            if (((rows >> r) & 1u) && lane < n) dst[c0 + lane] = tile[r][lane];
        }
        __syncwarp();
    }
};

// Masked apply_reset_state in one launch (python/carl.cu:508-666 with reset_mask:
// pads, ball, cars, contact refresh, match state, then obs / state / raw match
// outputs of the masked sims).  Each CTA owns a chunk of RESET_CHUNK sims: it
// lists the chunk's selected sims (ascending), then steps them in rounds of
// whole sims, one thread per car, so the refresh (which casts against the sim's
// other cars and ball) and the packing (which reads the whole sim) follow the
// writes after a CTA barrier.  With few selected sims every CTA is resident in
// one wave and does one short round.  Each phase runs the same per-item code as
// the separate kernels.
constexpr int RESET_THREADS = 128;
constexpr int RESET_CHUNK = 512;  // sims per CTA (a multiple of RESET_THREADS)

__device__ __forceinline__ unsigned long long wheelKey(float dist, unsigned cand)
{
    return ((unsigned long long)__float_as_uint(dist) << 32) | cand;
}

__global__ void __launch_bounds__(RESET_THREADS) resetMaskedKernel(GView g, ArenaDev a, BallInputs ball, CarInputs cars,
                                                                  MatchInputs match, const uint8_t* mask, PackTargets pk)
{
    __shared__ int selS[RESET_CHUNK];
    __shared__ int warpCountS[RESET_THREADS / 32];
    __shared__ unsigned long long keyS[NUM_WHEELS][RESET_THREADS];
    __shared__ float startS[15][RESET_THREADS];  // wheel ray starts (12), direction (3)
    __shared__ int firstS[RESET_THREADS], endS[RESET_THREADS], warpSumS[RESET_THREADS / 32];
    __shared__ float obsTile[RESET_THREADS / 32][32][33];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // The chunk's selected sims in ascending order.
    int nSel = 0;
    for (int part = 0; part < RESET_CHUNK / RESET_THREADS; part++)
    {
        const long long s = (long long)blockIdx.x * RESET_CHUNK + part * RESET_THREADS + tid;
        const bool pick = s < g.nSim && mask[s] != 0;
        const unsigned bits = __ballot_sync(0xffffffffu, pick);
        if (lane == 0) warpCountS[warp] = __popc(bits);
        __syncthreads();
        int before = nSel;
        for (int w = 0; w < warp; w++) before += warpCountS[w];
        if (pick) selS[before + __popc(bits & ((1u << lane) - 1u))] = (int)s;
        for (int w = 0; w < RESET_THREADS / 32; w++) nSel += warpCountS[w];
        __syncthreads();
    }
    if (nSel == 0) return;

    const int perRound = RESET_THREADS / g.nCars;
    const int slot = tid / g.nCars;
    const int local = tid - slot * g.nCars;
    for (int round = 0; round < nSel; round += perRound)
    {
        const bool on = slot < perRound && round + slot < nSel;
        const int sim = selS[on ? round + slot : round];  // threads with no car read a valid sim
        if (on)
        {
            if (local == 0)
            {
                resetPadsSim(g, sim);
                setBallSim(g, ball, sim, sim);
            }
            setCarOne(g, cars, sim * g.nCars + local, sim, local);
            if (local == 0 && match.blue) setMatchSim(g, match.blue, match.orange, match.ticks, sim, sim);
        }
        __syncthreads();
        // Contact refresh.  The arena pass of the wheel rays is flattened over the
        // CTA: every (car, cell triangle) item of the CTA's restored cars is one unit
        // of work, and a wheel's winner is the least (distance bits, candidate) key,
        // which is the serial pass's first strictly closest hit.
        const long long car = (long long)sim * g.nCars + local;
        const bool demoed = on && g.car.n(C_DEMOED, car) != 0;
        const bool cast = on && !demoed;
        CarRays r;
        if (cast)
        {
            r = carRays(g, car);
            for (int w = 0; w < NUM_WHEELS; w++)
            {
                keyS[w][threadIdx.x] = wheelKey(suspRayLength(w) + 1.f, 0xffffffffu);
                startS[3 * w][threadIdx.x] = r.start[w].x;
                startS[3 * w + 1][threadIdx.x] = r.start[w].y;
                startS[3 * w + 2][threadIdx.x] = r.start[w].z;
            }
            startS[12][threadIdx.x] = r.dir.x;
            startS[13][threadIdx.x] = r.dir.y;
            startS[14][threadIdx.x] = r.dir.z;
            firstS[threadIdx.x] = a.cellStart[r.cell];
        }
        const int count = cast ? a.cellStart[r.cell + 1] - firstS[threadIdx.x] : 0;
        // Block inclusive scan of the item counts.
        {
            int v = count;
            const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
            for (int o = 1; o < 32; o <<= 1)
            {
                const int n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += n;
            }
            if (lane == 31) warpSumS[warp] = v;
            __syncthreads();
            if (warp == 0)
            {
                int t = lane < RESET_THREADS / 32 ? warpSumS[lane] : 0;
                for (int o = 1; o < 32; o <<= 1)
                {
                    const int n = __shfl_up_sync(0xffffffffu, t, o);
                    if (lane >= o) t += n;
                }
                if (lane < RESET_THREADS / 32) warpSumS[lane] = t;
            }
            __syncthreads();
            endS[threadIdx.x] = v + (warp > 0 ? warpSumS[warp - 1] : 0);
            __syncthreads();
        }
        const int items = endS[RESET_THREADS - 1];
        for (int it = threadIdx.x; it < items; it += RESET_THREADS)
        {
            // Owner: the first thread whose inclusive end exceeds the item.
            int lo = 0, hi = RESET_THREADS - 1;
            while (lo < hi)
            {
                const int mid = (lo + hi) >> 1;
                if (endS[mid] > it) hi = mid;
                else lo = mid + 1;
            }
            const int cand = it - (lo > 0 ? endS[lo - 1] : 0);
            const int tri = a.cellTris[firstS[lo] + cand];
            const float4 p0 = a.triV[3 * tri], p1 = a.triV[3 * tri + 1], p2 = a.triV[3 * tri + 2];
            const V3 v0 = { p0.x, p0.y, p0.z };
            const V3 e1 = V3{ p1.x, p1.y, p1.z } - v0;
            const V3 e2 = V3{ p2.x, p2.y, p2.z } - v0;
            const V3 dir = { startS[12][lo], startS[13][lo], startS[14][lo] };
            const V3 pv = cross(dir, e2);
            const float det = dot(e1, pv);
            if (fabsf(det) < RAY_PARALLEL_EPS) continue;
            const float invDet = 1.f / det;
            for (int w = 0; w < NUM_WHEELS; w++)
            {
                const V3 st = { startS[3 * w][lo], startS[3 * w + 1][lo], startS[3 * w + 2][lo] };
                float d;
                if (wheelTriHit(st, dir, v0, e1, e2, pv, invDet, suspRayLength(w) + 1.f, d))
                    atomicMin(&keyS[w][lo], wheelKey(d, (unsigned)cand));
            }
        }
        __syncthreads();
        if (on)
        {
            float dist[NUM_WHEELS];
            V3 normal[NUM_WHEELS];
            int source[NUM_WHEELS];
            if (demoed)
            {
                demoedWheelRays(dist, normal, source);
            }
            else
            {
                initWheelRays(r, dist, normal, source);
                for (int w = 0; w < NUM_WHEELS; w++)
                {
                    const unsigned long long key = keyS[w][threadIdx.x];
                    const unsigned cand = (unsigned)(key & 0xffffffffu);
                    if (cand == 0xffffffffu) continue;
                    const int tri = a.cellTris[firstS[threadIdx.x] + (int)cand];
                    const float4 p0 = a.triV[3 * tri], p1 = a.triV[3 * tri + 1], p2 = a.triV[3 * tri + 2];
                    const V3 v0 = { p0.x, p0.y, p0.z };
                    V3 n = cross(V3{ p1.x, p1.y, p1.z } - v0, V3{ p2.x, p2.y, p2.z } - v0);
                    const float nl = lensq(n);
                    if (nl > 1e-12f)
                    {
                        dist[w] = __uint_as_float((unsigned)(key >> 32));
                        source[w] = WHEEL_ARENA;
                        n = n * rsqrtf(nl);
                        if (dot(n, r.dir) > 0.f) n = neg(n);
                        normal[w] = n;
                    }
                    else
                    {
                        // A degenerate winner keeps an earlier hit's normal: replay the serial pass.
                        arenaRaysSerial(a, r, w, w + 1, dist, normal, source);
                    }
                }
                carBallRays(g, car, sim, r, dist, normal, source);
            }
            storeRefresh(g, car, demoed, dist, normal, source);
        }
        __syncthreads();
        // Obs rows through the warp's staging tile, one row per car thread.
        {
            WarpRowsAt e{ obsTile[warp], pk.obs + ((long long)sim * g.nCars + local) * pk.obsDim, lane, 0,
                          __ballot_sync(0xffffffffu, on), pk.normalize != 0 };
            emitObsRow(g, e, pk.invertOrange, pk.previousControls, sim, local);
            e.finish();
        }
        if (on && local == 0)
        {
            packStateSim(g, pk.state, pk.stateDim, pk.tick, 1, sim);
            packRawMatchSim(g, pk.outputs, sim);
        }
        __syncthreads();
    }
}

// Action mask of each observation row (python/carl/gymnasium/action.py:17-37,
// CARLActionCodec.mask): every logit allowed except powerslide (on ground),
// boost (boost > 0) and jump (on ground, or a flip available with more than one
// tick of dodge window left).  Flags read as the reference's torch ops do:
// `.bool()` is `!= 0` (NaN counts as set), comparisons are false for NaN.
// A warp's 32 mask rows are 576 contiguous bytes: they are assembled in shared
// memory and written as 144 four-byte words (the mask must be 4-byte aligned;
// a warp holding the last rows writes bytes).
constexpr int MASK_THREADS = 256;

__global__ void __launch_bounds__(MASK_THREADS) actionMaskKernel(const float* obs, long long rows, int obsDim,
                                                                 int controlsSize, uint8_t* mask)
{
    __shared__ __align__(4) uint8_t rowsS[MASK_THREADS / 32][32 * ACTION_LOGITS];
    const long long r = blockIdx.x * (long long)MASK_THREADS + threadIdx.x;
    const int lane = threadIdx.x & 31;
    uint8_t* m = rowsS[threadIdx.x >> 5] + lane * ACTION_LOGITS;
    if (r < rows)
    {
        const float* o = obs + r * obsDim;
        const bool onGround = o[OBS_BALL + OBS_ON_GROUND] != 0.f;
        const bool hasBoost = o[OBS_BALL + OBS_BOOST] > 0.f;
        const bool flipAvailable = o[obsDim + OBS_EGO_FLIP_INDEX - controlsSize] != 0.f;
        const bool jump = onGround || (flipAvailable && o[obsDim + OBS_EGO_DODGE_TIME_INDEX - controlsSize] > PHYS_DT);
        for (int k = 0; k < ACTION_LOGITS; k++) m[k] = 1;
        m[ACTION_POWERSLIDE_LOGIT] = onGround;
        m[ACTION_BOOST_LOGIT] = hasBoost;
        m[ACTION_JUMP_LOGIT] = jump;
    }
    __syncwarp();
    const long long r0 = r - lane;
    if (r0 >= rows) return;
    const long long n = rows - r0 < 32 ? rows - r0 : 32;
    uint8_t* dst = mask + r0 * ACTION_LOGITS;
    const uint8_t* src = rowsS[threadIdx.x >> 5];
    if (n == 32)
    {
        const unsigned* s32 = reinterpret_cast<const unsigned*>(src);
        unsigned* d32 = reinterpret_cast<unsigned*>(dst);
        for (int w = lane; w < 32 * ACTION_LOGITS / 4; w += 32) d32[w] = s32[w];
    }
    else
    {
        for (int b = lane; b < n * ACTION_LOGITS; b += 32) dst[b] = src[b];
    }
}

// The env step's outputs after the ticks in one launch (python/carl.cu:312-370:
// rewards and dones, transition state, transition obs of the done sims,
// auto-reset, raw match state, obs, state).  A CTA owns EPI_AGENTS / nCars whole
// sims: its agent warps hold a car each, its sim warps a sim each.  Every phase
// only touches the CTA's own sims, so the per-sim order of the separate kernels
// is kept with two CTA barriers:
//   1. sim warps: rewards, dones, transition state rows; agent warps: transition
//      obs rows of the done sims (each evaluates its sim's done flag itself);
//   2. sim warps: auto-reset of the done sims;
//   3. agent warps: obs rows; sim warps: raw match state and state rows.
// Rows are written through the warps' staging tiles (a warp's agents, and its
// sims, are consecutive rows).
constexpr int EPI_AGENTS = 128;               // agent threads per CTA (4 warps)
constexpr int EPI_MAX_WARPS = 8;              // 4 agent warps + up to 4 sim warps (one car per sim)

__global__ void __launch_bounds__(EPI_MAX_WARPS * 32, 3) stepEpilogueKernel(GView g, Outputs o, StepOutputs a)
{
    extern __shared__ float tileMem[];  // [warps][32][33]
    float(*tile)[32][33] = reinterpret_cast<float(*)[32][33]>(tileMem);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int simsPerCta = EPI_AGENTS / g.nCars;
    const int sim0 = blockIdx.x * simsPerCta;
    const int nS = min(simsPerCta, g.nSim - sim0);
    const int agents = nS * g.nCars;
    const long long agent0 = (long long)sim0 * g.nCars;
    const bool agentWarp = tid < EPI_AGENTS;
    // Agent role: agent index inside the CTA; sim role: sim index inside the CTA.
    const int idx = agentWarp ? tid : tid - EPI_AGENTS;
    const bool live = agentWarp ? idx < agents : idx < nS;
    const int first = agentWarp ? (warp * 32) : (warp - EPI_AGENTS / 32) * 32;  // index of lane 0
    const bool warpLive = first < (agentWarp ? agents : nS);
    int sim, local = 0;
    if (agentWarp)
    {
        const long long ag = agent0 + min(idx, agents - 1);
        sim = (int)(ag / g.nCars);
        local = (int)(ag - (long long)sim * g.nCars);
    }
    else
    {
        sim = sim0 + min(idx, nS - 1);
    }

    if (!agentWarp)
    {
        if (live) packRewardsDonesSim(g, o, sim, a.tick, a.maxTicks, a.overtimeTicks, a.noTouchTicks);
        if (warpLive)
        {
            WarpRows e{ tile[warp], a.tstate + (long long)(sim0 + first) * a.stateDim, a.stateDim, lane, 0,
                        __ballot_sync(0xffffffffu, live), false };
            emitStateRow(g, e, a.tick, a.frameskip, sim);
            e.finish();
        }
    }
    else if (warpLive)
    {
        const bool done = live && simDone(g, sim, a.tick, a.maxTicks, a.overtimeTicks, a.noTouchTicks);
        const unsigned rows = __ballot_sync(0xffffffffu, done);
        if (rows)
        {
            WarpRows e{ tile[warp], a.tobs + (agent0 + first) * a.obsDim, a.obsDim, lane, 0, rows, a.normalize != 0 };
            emitObsRow(g, e, a.invertOrange, a.previousControls, sim, local);
            e.finish();
        }
    }
    __syncthreads();
    if (!agentWarp && live) resetDoneSim(g, sim, a.tick, a.maxTicks, a.overtimeTicks, a.noTouchTicks);
    __syncthreads();
    if (agentWarp)
    {
        if (warpLive)
        {
            WarpRows e{ tile[warp], a.obs + (agent0 + first) * a.obsDim, a.obsDim, lane, 0,
                        __ballot_sync(0xffffffffu, live), a.normalize != 0 };
            emitObsRow(g, e, a.invertOrange, a.previousControls, sim, local);
            e.finish();
        }
    }
    else
    {
        if (live) packRawMatchSim(g, o, sim);
        if (warpLive)
        {
            WarpRows e{ tile[warp], a.state + (long long)(sim0 + first) * a.stateDim, a.stateDim, lane, 0,
                        __ballot_sync(0xffffffffu, live), false };
            emitStateRow(g, e, a.tick, 1, sim);
            e.finish();
        }
    }
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
    const long long n = (long long)g.nSim * g.nCars;
    if (n <= 0) return;
    if (g.stagedPack)
        packObsWarpKernel<<<blocks(n, PACK_THREADS), PACK_THREADS, 0, s>>>(g, out, mask, obsDim, invert, normalize, prev);
    else
        packObsKernel<<<blocks(n, 128), 128, 0, s>>>(g, out, mask, obsDim, invert, normalize, prev);
}
void launchPackState(const GView& g, float* out, int stateDim, int tick, int touchWindow, const uint8_t* mask, cudaStream_t s)
{
    if (g.nSim <= 0) return;
    if (g.stagedPack)
        packStateWarpKernel<<<blocks(g.nSim, PACK_THREADS), PACK_THREADS, 0, s>>>(g, out, stateDim, tick, touchWindow, mask);
    else
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
void launchActionMask(const float* obs, long long rows, int obsDim, bool previousControls, uint8_t* mask, cudaStream_t s)
{
    if (rows > 0)
        actionMaskKernel<<<blocks(rows, MASK_THREADS), MASK_THREADS, 0, s>>>(obs, rows, obsDim,
                                                                            previousControls ? OBS_PREVIOUS_CONTROLS : 0,
                                                                            mask);
}
void launchStepEpilogue(const GView& g, const Outputs& o, const StepOutputs& a, cudaStream_t s)
{
    if (g.nSim <= 0) return;
    const int simsPerCta = EPI_AGENTS / g.nCars;
    const int threads = EPI_AGENTS + 32 * ((simsPerCta + 31) / 32);
    const size_t smem = (size_t)(threads / 32) * 32 * 33 * sizeof(float);
    stepEpilogueKernel<<<blocks(g.nSim, simsPerCta), threads, smem, s>>>(g, o, a);
}
void launchResetMasked(const GView& g, const ArenaDev& a, const BallInputs& ball, const CarInputs& cars,
                       const MatchInputs& match, const uint8_t* mask, const PackTargets& pk, cudaStream_t s)
{
    if (g.nSim <= 0) return;
    resetMaskedKernel<<<blocks(g.nSim, RESET_CHUNK), RESET_THREADS, 0, s>>>(g, a, ball, cars, match, mask, pk);
}

}  // namespace cb
