/*
 * CPU oracle: the reference's own physics (jwmccarthy/CARL include/Physics/**,
 * include/State/**, include/Arena/**, src/ArenaMesh.cu, src/RLConstants.cu)
 * compiled as host C++ through refshim/carl_host_shim.h, driven by a host loop
 * that reproduces the stage order of the reference's tick.
 *
 *   tick order            src/RLEnvironment.cu:166-211, kernels src/Kernels.cu:15-202
 *   env step              python/carl.cu:312-370 (EnvWrapper::step / stepContinuous)
 *   construction, reset   python/carl.cu:286-310, src/RLEnvironment.cu:192-198
 *   obs / state packing   src/EnvIO.cu:47-135
 *
 * Differences from the reference's GPU build, by construction of the shim:
 * rsqrtf is exact, __sincosf / sinf / cosf / atan2f / powf are the host libm
 * versions, and SAT slots are assigned in (car, candidate) order instead of
 * atomicAdd order.  Per-car and per-sim stages run under OpenMP
 * (schedule(static)); sims never interact, so the result does not depend on the
 * thread count.
 * TEST INFRASTRUCTURE: only tests, smoke() and bench.py's CPU baseline use it.
 */
#include <omp.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "State/GameState.cuh"
#include "State/Workspace.cuh"
#include "State/Reset.cuh"
#include "State/Controls.cuh"
#include "Arena/ArenaMesh.cuh"
#include "Cuda/DLPack.h"
#include "Physics/CarArena/BroadPhase.cuh"
#include "Physics/CarArena/SAT.cuh"
#include "Physics/CarArena/Clip.cuh"
#include "Physics/CarArena/Solve.cuh"
#include "Physics/BallArena/Solve.cuh"
#include "Physics/BoostPads.cuh"
#include "Physics/CarCar/Solve.cuh"
#include "Physics/Controls.cuh"
#include "Physics/FinishTick.cuh"
#include "Physics/SuspensionRaycast.cuh"
#include "Physics/Observations.cuh"

#include "ref_fields.h"

static_assert(sizeof(bool) == 1, "dones are packed as one byte per sim");

namespace {

thread_local std::string g_error;

struct RefCpu
{
    GameState state;
    Workspace space;
    ArenaMesh arena;

    int frameskip;
    bool invertOrange, normalize, previousControls;
    int maxTicks = REGULATION_TICKS;
    int overtimeTimeoutTicks = REGULATION_TICKS;
    int noTouchTimeoutTicks = 0;
    int obsDim, stateDim;

    std::vector<float> obs, transitionObs, packed, transitionPacked, rewards;
    std::vector<uint8_t> dones, overtime, transitionOvertime;
    std::vector<int> scoreDiff, episodeTicks, transitionScoreDiff, transitionEpisodeTicks;

    RefCpu(int nSim, int nBlue, int nOrange, int seed, int fs, bool inv, bool norm, bool prev)
        : state(nSim, nBlue, nOrange, seed)
        , space(nSim, nBlue + nOrange, nSim * (nBlue + nOrange))
        , arena()
        , frameskip(fs), invertOrange(inv), normalize(norm), previousControls(prev)
        , obsDim(observationDim(nBlue + nOrange, prev))
        , stateDim(packedStateDim(nBlue + nOrange))
    {
        const int n = state.nTotalCars;
        state.cars.controls.fill(0);
        obs.assign((size_t)n * obsDim, 0.f);
        transitionObs.assign((size_t)n * obsDim, 0.f);
        packed.assign((size_t)nSim * stateDim, 0.f);
        transitionPacked.assign((size_t)nSim * stateDim, 0.f);
        rewards.assign(nSim, 0.f);
        dones.assign(nSim, 0);
        overtime.assign(nSim, 0);
        transitionOvertime.assign(nSim, 0);
        scoreDiff.assign(nSim, 0);
        episodeTicks.assign(nSim, 0);
        transitionScoreDiff.assign(nSim, 0);
        transitionEpisodeTicks.assign(nSim, 0);
    }

    // --- RLEnvironment::reset (src/RLEnvironment.cu:192-198, src/Kernels.cu:15-23)
    void resetAll()
    {
        state.reset();
        space.reset();
        GameState* S = &state;
        state.tickCount = 0;
        #pragma omp parallel for schedule(static)
        for (int sim = 0; sim < S->nSim; sim++) resetToKickoff(S, sim);
    }

    // --- one physics tick (src/RLEnvironment.cu:179-211), optionally stopping
    // after stage `lastStage` (0 begin, 1 broadphase, 2 scan, 3 raycast,
    // 4 controls, 5 SAT, 6 clip, 7 solve, 8 car-car + ball, 9 integrate,
    // 10 impulse cache, 11 boost pads).
    void tick(int kind, const void* actions, int lastStage = 11)
    {
        GameState* S = &state;
        Workspace* W = &space;
        ArenaMesh* A = &arena;
        const int n = S->nTotalCars;

        // beginStepKernel (src/Kernels.cu:42-55)
        S->tickCount++;
        #pragma omp parallel for schedule(static)
        for (int sim = 0; sim < S->nSim; sim++) S->episodeTicks[sim]++;
        if (lastStage < 1) return;

        // stepBroadSusp: broadphase, exclusive scan, raycast (src/RLEnvironment.cu:96-106)
        #pragma omp parallel for schedule(static)
        for (int car = 0; car < n; car++) carArenaBroadPhase(S, W, A, car);
        if (lastStage < 2) return;
        {
            int run = 0;
            for (int i = 0; i <= n; i++)
            {
                W->bp.triPrefix[i] = run;
                run += W->bp.numTris[i];
            }
        }
        if (lastStage < 3) return;
        #pragma omp parallel for schedule(static)
        for (int car = 0; car < n; car++) raycastCarSuspension(S, W, A, car);
        if (lastStage < 4) return;

        // stepControls (src/Kernels.cu:68-90,112-122)
        #pragma omp parallel for schedule(static)
        for (int car = 0; car < n; car++)
        {
            if (kind == CARLB_ACTIONS_DISCRETE)
                S->cars.controls[car] = static_cast<const DiscreteControls*>(actions)[car].decode();
            else if (kind == CARLB_ACTIONS_CONTINUOUS)
                S->cars.controls[car] = static_cast<const ContinuousControls*>(actions)[car].decode();
            else
                S->cars.controls[car] = static_cast<const CarControls*>(actions)[car];
            processCarControls(S, W, car);
        }
        if (lastStage < 5) return;

        // stepNarrow: SAT per candidate in (car, candidate) order, then clip
        #pragma omp parallel for schedule(static)
        for (int car = 0; car < n; car++)
        {
            const int count = W->bp.numTris[car];
            for (int offset = 0; offset < count; offset++)
                writeCarTriPairResult(S, W, A, car, offset);
        }
        if (lastStage < 6) return;
        #pragma omp parallel for schedule(static)
        for (int hit = 0; hit < W->ctNrw.maxCarTriPairs; hit++) carArenaClip(A, W, hit);
        if (lastStage < 7) return;

        // stepCarManifoldSolve (src/Kernels.cu:148-160)
        #pragma omp parallel for schedule(static)
        for (int car = 0; car < n; car++) solveCarArena(S, W, A, car);
        if (lastStage < 8) return;

        // stepCarCarSolve: car-car then ball per sim (src/Kernels.cu:162-172)
        #pragma omp parallel for schedule(static)
        for (int sim = 0; sim < S->nSim; sim++)
        {
            solveCarCarForSim(S, W, sim);
            solveBallForSim(S, A, sim);
        }
        if (lastStage < 9) return;

        // integrateCars (src/Kernels.cu:174-180)
        #pragma omp parallel for schedule(static)
        for (int car = 0; car < n; car++) integrateCar(S, car);
        if (lastStage < 10) return;

        // applyImpulseCache (src/Kernels.cu:182-190)
        const int finishCount = n > S->nSim ? n : S->nSim;
        #pragma omp parallel for schedule(static)
        for (int idx = 0; idx < finishCount; idx++)
        {
            if (idx < S->nSim) finishBallTick(S, idx);
            if (idx < n) finishCarTick(S, idx);
        }
        if (lastStage < 11) return;

        // stepBoostPad (src/Kernels.cu:192-202)
        #pragma omp parallel for schedule(static)
        for (int slot = 0; slot < S->nSim * NUM_BOOST_PADS; slot++) processBoostPad(S, slot);
    }

    void resetDones()
    {
        GameState* S = &state;
        Workspace* W = &space;
        #pragma omp parallel for schedule(static)
        for (int sim = 0; sim < S->nSim; sim++)
            resetAfterDone(S, W, sim, maxTicks, overtimeTimeoutTicks, noTouchTimeoutTicks);
    }

    // --- EnvIO packing (src/EnvIO.cu:47-135)
    void packObs(float* out, const uint8_t* mask)
    {
        GameState* S = &state;
        const int nCars = S->nCars;
        #pragma omp parallel for schedule(static)
        for (int agent = 0; agent < S->nTotalCars; agent++)
        {
            const int sim = agent / nCars;
            if (mask && !mask[sim]) continue;
            float* o = out + (size_t)agent * obsDim;
            packObservations(S, sim, agent % nCars, nCars, invertOrange, o, previousControls);
            if (normalize) normalizeObservations(o, nCars);
        }
    }

    void packStateInto(float* out, int touchWindow, const uint8_t* mask)
    {
        GameState* S = &state;
        #pragma omp parallel for schedule(static)
        for (int sim = 0; sim < S->nSim; sim++)
        {
            if (mask && !mask[sim]) continue;
            ::packState(S, sim, S->nCars, touchWindow, out + (size_t)sim * stateDim);
        }
    }

    void packRawMatch(int* score, int* ticks, uint8_t* ot, const uint8_t* mask)
    {
        GameState* S = &state;
        for (int sim = 0; sim < S->nSim; sim++)
        {
            if (mask && !mask[sim]) continue;
            const GoalState goal = S->goals[sim];
            score[sim] = goal.blueScore - goal.orangeScore;
            ticks[sim] = S->episodeTicks[sim];
            ot[sim] = goal.overtime ? 1 : 0;
        }
    }

    void packRewardsDones()
    {
        GameState* S = &state;
        for (int sim = 0; sim < S->nSim; sim++)
        {
            packRewards(S, sim, rewards.data());
            packDones(S, sim, maxTicks, overtimeTimeoutTicks, noTouchTimeoutTicks,
                      reinterpret_cast<bool*>(dones.data()));
        }
        packRawMatch(transitionScoreDiff.data(), transitionEpisodeTicks.data(),
                     transitionOvertime.data(), nullptr);
    }

    void initialPack()
    {
        packObs(obs.data(), nullptr);
        packStateInto(packed.data(), 1, nullptr);
        packStateInto(transitionPacked.data(), 1, nullptr);
        packRewardsDones();
        packRawMatch(scoreDiff.data(), episodeTicks.data(), overtime.data(), nullptr);
    }

    // --- EnvWrapper::step (python/carl.cu:312-344)
    void envStep(int kind, const void* actions)
    {
        for (int t = 0; t < frameskip; t++) tick(kind, actions);
        packRewardsDones();
        packStateInto(transitionPacked.data(), frameskip, nullptr);
        packObs(transitionObs.data(), dones.data());
        resetDones();
        packRawMatch(scoreDiff.data(), episodeTicks.data(), overtime.data(), nullptr);
        packObs(obs.data(), nullptr);
        packStateInto(packed.data(), 1, nullptr);
    }
};

RefCopy hostCopy()
{
    return [](void* d, const void* s, size_t b) { if (b) std::memcpy(d, s, b); };
}

}  // namespace

extern "C" {

const char* carlref_error() { return g_error.c_str(); }

int carlref_set_threads(int threads)
{
    if (threads > 0) omp_set_num_threads(threads);
    return omp_get_max_threads();
}

void* carlref_create(int nSim, int nBlue, int nOrange, int seed, int frameskip,
                     int invertOrange, int normalize, int previousControls)
{
    try
    {
        if (nSim < 1 || nBlue < 0 || nOrange < 0 || nBlue + nOrange < 1 || frameskip < 1)
        {
            g_error = "invalid dimensions";
            return nullptr;
        }
        auto* env = new RefCpu(nSim, nBlue, nOrange, seed, frameskip,
                               invertOrange != 0, normalize != 0, previousControls != 0);
        env->resetAll();
        env->initialPack();
        return env;
    }
    catch (const std::exception& e)
    {
        g_error = e.what();
        return nullptr;
    }
}

void carlref_destroy(void* h) { delete static_cast<RefCpu*>(h); }

int carlref_dims(void* h, int* dims)
{
    auto* e = static_cast<RefCpu*>(h);
    dims[0] = e->state.nSim;
    dims[1] = e->state.nCars;
    dims[2] = e->obsDim;
    dims[3] = e->state.nCars * ACT_PER_CAR;
    dims[4] = e->stateDim;
    return 0;
}

int carlref_set_limits(void* h, int maxTicks, int overtimeTicks, int noTouchTicks, int frameskip)
{
    auto* e = static_cast<RefCpu*>(h);
    if (maxTicks > 0) e->maxTicks = maxTicks;
    if (overtimeTicks > 0) e->overtimeTimeoutTicks = overtimeTicks;
    if (noTouchTicks >= 0) e->noTouchTimeoutTicks = noTouchTicks;
    if (frameskip > 0) e->frameskip = frameskip;
    return 0;
}

int carlref_reset(void* h)
{
    auto* e = static_cast<RefCpu*>(h);
    e->resetAll();
    e->initialPack();
    return 0;
}

int carlref_ticks(void* h, int kind, const void* actions, int nTicks)
{
    auto* e = static_cast<RefCpu*>(h);
    for (int t = 0; t < nTicks; t++) e->tick(kind, actions);
    return 0;
}

int carlref_tick_partial(void* h, int kind, const void* actions, int lastStage)
{
    static_cast<RefCpu*>(h)->tick(kind, actions, lastStage);
    return 0;
}

int carlref_env_step(void* h, int kind, const void* actions)
{
    static_cast<RefCpu*>(h)->envStep(kind, actions);
    return 0;
}

int carlref_reset_dones(void* h)
{
    static_cast<RefCpu*>(h)->resetDones();
    return 0;
}

/* Re-pack obs / state / raw match outputs from the current state. */
int carlref_repack(void* h)
{
    auto* e = static_cast<RefCpu*>(h);
    e->packObs(e->obs.data(), nullptr);
    e->packStateInto(e->packed.data(), 1, nullptr);
    e->packRawMatch(e->scoreDiff.data(), e->episodeTicks.data(), e->overtime.data(), nullptr);
    return 0;
}

/* Copies an output buffer (numbering of carlb_buffer) into host memory. */
int carlref_get_buffer(void* h, int which, void* out)
{
    auto* e = static_cast<RefCpu*>(h);
    auto cp = [&](const auto& v) {
        std::memcpy(out, v.data(), v.size() * sizeof(v[0]));
        return 0;
    };
    switch (which)
    {
    case CARLB_BUF_OBS: return cp(e->obs);
    case CARLB_BUF_TRANSITION_OBS: return cp(e->transitionObs);
    case CARLB_BUF_STATE: return cp(e->packed);
    case CARLB_BUF_TRANSITION_STATE: return cp(e->transitionPacked);
    case CARLB_BUF_REWARDS: return cp(e->rewards);
    case CARLB_BUF_DONES: return cp(e->dones);
    case CARLB_BUF_SCORE_DIFFERENCE: return cp(e->scoreDiff);
    case CARLB_BUF_EPISODE_TICKS: return cp(e->episodeTicks);
    case CARLB_BUF_TRANSITION_SCORE_DIFFERENCE: return cp(e->transitionScoreDiff);
    case CARLB_BUF_TRANSITION_EPISODE_TICKS: return cp(e->transitionEpisodeTicks);
    case CARLB_BUF_OVERTIME: return cp(e->overtime);
    case CARLB_BUF_TRANSITION_OVERTIME: return cp(e->transitionOvertime);
    default: g_error = "unknown buffer"; return 1;
    }
}

int carlref_field_shape(void* h, int field, int64_t* rows, int* width)
{
    auto* e = static_cast<RefCpu*>(h);
    const RefField f = refField(e->state, e->space, field, &e->state.tickCount);
    if (f.rows < 0) { g_error = "unknown field"; return 1; }
    *rows = f.rows;
    *width = f.width;
    return 0;
}

int carlref_read_field(void* h, int field, void* out)
{
    auto* e = static_cast<RefCpu*>(h);
    const RefField f = refField(e->state, e->space, field, &e->state.tickCount);
    if (f.rows < 0) { g_error = "unknown field"; return 1; }
    uint32_t* words = static_cast<uint32_t*>(out);
    if (field == CARLB_F_DIAG_SAT_PAIRS)
    {
        for (int car = 0; car < e->state.nTotalCars; car++)
        {
            const int hits = e->space.ctHit.carHitCount[car];
            const int count = hits < MAX_CAR_TRI_PAIRS ? hits : MAX_CAR_TRI_PAIRS;
            uint32_t* row = words + (size_t)car * f.width;
            std::memset(row, 0xff, sizeof(uint32_t) * f.width);
            row[0] = (uint32_t)count;
            for (int s = 0; s < count; s++)
                row[1 + s] = (uint32_t)e->space.ctNrw.triIdx[car * MAX_CAR_TRI_PAIRS + s];
        }
        return 0;
    }
    refReadField(f, words, hostCopy());
    return 0;
}

int carlref_write_field(void* h, int field, const void* in)
{
    auto* e = static_cast<RefCpu*>(h);
    const RefField f = refField(e->state, e->space, field, &e->state.tickCount);
    if (f.rows < 0 || f.readOnly) { g_error = "field is unknown or read-only"; return 1; }
    refWriteField(f, static_cast<const uint32_t*>(in), hostCopy(), hostCopy());
    return 0;
}

/* The reference's kickoff permutation table (src/RLConstants.cu:4-29). */
int carlref_kickoff_table(int* out)
{
    for (int r = 0; r < 120; r++)
        for (int k = 0; k < 4; k++) out[4 * r + k] = KICKOFF_PERMUTATIONS[r][k];
    return 0;
}

/* Arena tables for the arena-build parity test. */
int carlref_arena_sizes(void* h, int* sizes)
{
    auto* e = static_cast<RefCpu*>(h);
    sizes[0] = e->arena.nVerts;
    sizes[1] = e->arena.nTris;
    sizes[2] = e->arena.nCells;
    sizes[3] = e->arena.prefix[e->arena.nCells];
    return 0;
}

int carlref_arena_tables(void* h, float* verts, int* tris, int* prefix, int* triIdx,
                         float* edgeAngles, int* ballTriIdx)
{
    auto* e = static_cast<RefCpu*>(h);
    const ArenaMesh& a = e->arena;
    for (int i = 0; i < a.nVerts; i++)
    {
        verts[3 * i] = a.verts[i].x;
        verts[3 * i + 1] = a.verts[i].y;
        verts[3 * i + 2] = a.verts[i].z;
    }
    for (int i = 0; i < a.nTris; i++)
    {
        tris[3 * i] = a.tris[i].x;
        tris[3 * i + 1] = a.tris[i].y;
        tris[3 * i + 2] = a.tris[i].z;
        edgeAngles[3 * i] = a.triAngs[i].x;
        edgeAngles[3 * i + 1] = a.triAngs[i].y;
        edgeAngles[3 * i + 2] = a.triAngs[i].z;
    }
    const int refs = a.prefix[a.nCells];
    for (int c = 0; c <= a.nCells; c++) prefix[c] = a.prefix[c];
    for (int r = 0; r < refs; r++)
    {
        triIdx[r] = a.carTriIdx[r];
        ballTriIdx[r] = a.ballTriIdx[r];
    }
    return 0;
}

}  // extern "C"
