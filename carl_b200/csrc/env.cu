// carlb_env: one env on one CUDA device behind the C ABI of include/carlb.h.
//
// Host orchestration of an RL step (jwmccarthy/CARL python/carl.cu:312-370):
//   copy actions -> stage kernels of frameskip ticks (one graph replay) ->
//   rewards/dones -> transition state / obs -> auto-reset -> obs, state.
// Everything is enqueued on the env's own non-blocking stream; the host keeps
// the tick counter.  Errors are returned as carlb_status with a message; no
// entry point exits the process.
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/carlb.h"
#include "arena.hpp"
#include "envio.cuh"
#include "tick.cuh"

using namespace cb;

namespace {

thread_local std::string g_createError;

std::string libraryDir()
{
    Dl_info info{};
    if (dladdr(reinterpret_cast<void*>(&libraryDir), &info) && info.dli_fname)
    {
        std::string p = info.dli_fname;
        const size_t slash = p.rfind('/');
        return slash == std::string::npos ? std::string(".") : p.substr(0, slash);
    }
    return ".";
}

// Host arena tables, built once per process, mesh path and metadata path.
std::shared_ptr<const ArenaHost> hostArena(const std::string& path, const std::string& metadata, std::string& err)
{
    static std::mutex mu;
    static std::map<std::string, std::shared_ptr<const ArenaHost>> cache;
    std::lock_guard<std::mutex> lock(mu);
    const std::string key = path + '\n' + metadata;
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    auto a = std::make_shared<ArenaHost>();
    err = buildArena(path, *a);
    if (err.empty() && !metadata.empty()) err = loadNativeMetadata(metadata, *a);
    if (!err.empty()) return nullptr;
    cache[key] = a;
    return a;
}

}  // namespace

struct carlb_env
{
    carlb_config cfg{};
    int nCars = 0;
    long long nCarTotal = 0;
    long long carStride = 0, simStride = 0;
    int obsDim = 0, stateDim = 0, actDim = 0;
    cudaStream_t stream = nullptr;

    float* car = nullptr;
    float* sim = nullptr;
    float* carOut = nullptr;
    int* simOut = nullptr;
    int* diagCar = nullptr;
    int* diagSim = nullptr;
    bool diagnostics = false;

    float4* triV = nullptr;
    float4* triAng = nullptr;
    float4* cellSph = nullptr;
    float4* cellV = nullptr;
    float4 ballGrid{};
    int ballDims[3] = { 0, 0, 0 };
    int* ballCellStart = nullptr;
    int* ballCellTris = nullptr;
    float4* ballCellSph = nullptr;
    int hasNative = 0;
    float4 *nativeV = nullptr, *nativeAng = nullptr;
    float carReach = 0.f;
    int* cellStart = nullptr;
    int* cellTris = nullptr;
    int hitWords = 1;

    // Scratch of the stage kernels.
    StageScratch scratch{};
    int groups = 2;
    cudaStream_t groupStream[8] = {};
    cudaEvent_t groupJoin[8] = {};
    cudaEvent_t evFork = nullptr;
    bool stageTiming = false;
    bool stageTimed = false;  // the last launch recorded stage events
    cudaEvent_t stageEv[2 * STAGE_KERNELS] = {};
    bool ballSide = true;  // ball arena stage on a side stream per slice (CARLB_BALL_STREAM=0 disables)
    cudaStream_t ballStream[8] = {};
    // Arena tables in one allocation with an L2 persisting access-policy window on
    // the stage kernels (CARLB_L2_WINDOW=1; off by default): the tables' device
    // pointers and sizes as allocated, then the pool they were moved into.
    bool l2Window = false;
    std::vector<std::pair<void**, size_t>> arenaTables;
    void* arenaPool = nullptr;
    size_t arenaPoolBytes = 0;
    cudaEvent_t tickStart[8] = {}, ballDone[8] = {};
    bool phaseOffset = true;  // slices alternate their wide stages (CARLB_PHASE_OFFSET=0 disables)
    cudaEvent_t wideDone[8] = {};
    // Staged launches replayed from instantiated graphs (CARLB_GRAPH=0 disables): one per
    // (action kind, tick count, diagnostics, stage timing); the tick count before
    // each launch is written to tickDev, which the captured stage kernels read.
    bool useGraph = true;
    // Masked apply_reset_state in one fused kernel (CARLB_FUSED_RESET=0: one kernel per part).
    bool fusedReset = true;
    // Obs / state rows written through per-warp staging tiles (CARLB_STAGED_PACK=0: a thread per row).
    bool stagedPack = true;
    // An env step's packing and auto-reset in one kernel (CARLB_FUSED_EPILOGUE=1); the
    // default runs the seven grid-wide kernels, which measured faster.
    bool fusedEpilogue = false;
    int* tickDev = nullptr;
    // Host actions of carlb_ticks_host copied slice by slice on their own stream, each
    // slice's controls stage waiting for its rows (CARLB_OVERLAP_COPY=0: one copy on the
    // env stream before the launch).  Created on first use.
    bool overlapCopy = true;
    cudaStream_t copyStream = nullptr;
    cudaEvent_t actionsIn = nullptr;
    cudaEvent_t actionsReady[8] = {};
    struct TickGraph { int kind, nTicks; bool diag, timing, hostIn; cudaGraphExec_t exec; };
    std::vector<TickGraph> graphs;

    float *obs = nullptr, *tobs = nullptr, *packed = nullptr, *tpacked = nullptr, *rewards = nullptr;
    uint8_t *dones = nullptr, *overtime = nullptr, *tovertime = nullptr;
    int *scoreDiff = nullptr, *episodeTicks = nullptr, *tScoreDiff = nullptr, *tEpisodeTicks = nullptr;
    void* actions = nullptr;
    size_t actionCapacity = 0;

    int tick = 0;
    int maxTicks = REGULATION_TICKS;
    int overtimeTicks = REGULATION_TICKS;
    int noTouchTicks = 0;

    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float lastTickMs = 0.f;
    std::string error;

    std::vector<void*> allocations;

    GView view() const
    {
        GView g;
        g.car = GlobSoa{ car, carStride };
        g.out = GlobSoa{ carOut, carStride };
        g.sim = GlobSoa{ sim, simStride };
        g.simOut = simOut;
        g.nSim = cfg.n_sim;
        g.nCars = nCars;
        g.stagedPack = stagedPack;
        g.nBlue = cfg.n_blue;
        g.nOrange = cfg.n_orange;
        g.seed = cfg.seed;
        g.simOffset = cfg.sim_offset;
        return g;
    }
    StageStreams stageStreams(bool hostIn = false) const
    {
        StageStreams s{};
        for (int g = 0; g < 8; g++) s.actionsReady[g] = hostIn ? actionsReady[g] : nullptr;
        s.groups = groups;
        for (int g = 0; g < 8; g++)
        {
            s.streams[g] = groupStream[g];
            s.join[g] = groupJoin[g];
        }
        s.fork = evFork;
        for (int k = 0; k < 2 * STAGE_KERNELS; k++) s.stageEvents[k] = stageTiming ? stageEv[k] : nullptr;
        for (int g = 0; g < 8; g++)
        {
            s.ballStreams[g] = ballSide ? ballStream[g] : nullptr;
            s.tickStart[g] = tickStart[g];
            s.ballDone[g] = ballDone[g];
            s.wideDone[g] = phaseOffset ? wideDone[g] : nullptr;
        }
        return s;
    }
    ArenaDev arena() const { return ArenaDev{ triV, triAng, cellStart, cellTris, hitWords, cellSph, carReach, cellV, ballGrid, ballDims[0], ballDims[1],
                         ballDims[2], ballCellStart, ballCellTris, ballCellSph, hasNative, nativeV, nativeAng }; }
    Outputs outputs() const
    {
        return Outputs{ rewards, dones, scoreDiff, episodeTicks, tScoreDiff, tEpisodeTicks, overtime, tovertime };
    }
};

namespace {

carlb_status fail(carlb_env* e, carlb_status s, const std::string& msg)
{
    if (e) e->error = msg;
    else g_createError = msg;
    return s;
}

carlb_status cudaFail(carlb_env* e, cudaError_t err, const char* what)
{
    return fail(e, CARLB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

#define ECHECK(e, call)                                            \
    do {                                                           \
        cudaError_t err_ = (call);                                 \
        if (err_ != cudaSuccess) return cudaFail((e), err_, #call); \
    } while (0)

template <class T>
cudaError_t allocZero(carlb_env* e, T** p, size_t count)
{
    void* v = nullptr;
    cudaError_t err = cudaMalloc(&v, count * sizeof(T) > 0 ? count * sizeof(T) : 16);
    if (err != cudaSuccess) return err;
    e->allocations.push_back(v);
    *p = static_cast<T*>(v);
    return cudaMemsetAsync(v, 0, count * sizeof(T), e->stream);
}

// An arena table (read-only after set-up): remembered so that it can be moved
// into the one pool an L2 access-policy window covers.
template <class T>
cudaError_t allocArena(carlb_env* e, T** p, size_t count)
{
    const cudaError_t err = allocZero(e, p, count);
    if (err == cudaSuccess) e->arenaTables.push_back({ reinterpret_cast<void**>(p), count * sizeof(T) });
    return err;
}

// Moves the arena tables into one allocation and reserves persisting L2 lines
// for it (a limit of this process's context; it ends with the process).
cudaError_t poolArenaTables(carlb_env* e)
{
    size_t total = 0;
    for (const auto& t : e->arenaTables) total += (t.second + 255) & ~(size_t)255;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    int maxWindow = 0, maxPersist = 0;
    cudaDeviceGetAttribute(&maxWindow, cudaDevAttrMaxAccessPolicyWindowSize, dev);
    cudaDeviceGetAttribute(&maxPersist, cudaDevAttrMaxPersistingL2CacheSize, dev);
    if (total == 0 || (size_t)maxWindow < total || (size_t)maxPersist < total) return cudaSuccess;  // no window
    err = cudaMalloc(&e->arenaPool, total);
    if (err != cudaSuccess) return err;
    e->allocations.push_back(e->arenaPool);
    size_t off = 0;
    for (const auto& t : e->arenaTables)
    {
        char* dst = static_cast<char*>(e->arenaPool) + off;
        err = cudaMemcpyAsync(dst, *t.first, t.second, cudaMemcpyDeviceToDevice, e->stream);
        if (err != cudaSuccess) return err;
        *t.first = dst;
        off += (t.second + 255) & ~(size_t)255;
    }
    e->arenaPoolBytes = total;
    size_t current = 0;
    cudaDeviceGetLimit(&current, cudaLimitPersistingL2CacheSize);
    if (current < total) err = cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, total);
    return err;
}

cudaAccessPolicyWindow arenaWindow(const carlb_env* e)
{
    cudaAccessPolicyWindow w{};
    w.base_ptr = e->arenaPool;
    w.num_bytes = e->arenaPoolBytes;
    w.hitRatio = 1.f;
    w.hitProp = cudaAccessPropertyPersisting;
    w.missProp = cudaAccessPropertyStreaming;
    return w;
}

// Sets the arena window on every kernel node of a captured tick graph.
cudaError_t applyArenaWindow(const carlb_env* e, cudaGraph_t graph)
{
    if (!e->arenaPool) return cudaSuccess;
    size_t n = 0;
    cudaError_t err = cudaGraphGetNodes(graph, nullptr, &n);
    if (err != cudaSuccess) return err;
    std::vector<cudaGraphNode_t> nodes(n);
    err = cudaGraphGetNodes(graph, nodes.data(), &n);
    if (err != cudaSuccess) return err;
    cudaKernelNodeAttrValue v{};
    v.accessPolicyWindow = arenaWindow(e);
    for (cudaGraphNode_t node : nodes)
    {
        cudaGraphNodeType type;
        if ((err = cudaGraphNodeGetType(node, &type)) != cudaSuccess) return err;
        if (type != cudaGraphNodeTypeKernel) continue;
        if ((err = cudaGraphKernelNodeSetAttribute(node, cudaKernelNodeAttributeAccessPolicyWindow, &v)) != cudaSuccess)
            return err;
    }
    return cudaSuccess;
}

size_t actionRowBytes(carlb_action_kind kind) { return kind == CARLB_ACTIONS_DIRECT ? 32 : 28; }

// hostIn: the actions are being copied in per slice on the copy stream
// (stageHostActionsSliced), so each slice's controls stage waits for its rows.
carlb_status launchTicks(carlb_env* e, carlb_action_kind kind, int nTicks, bool hostIn = false)
{
    TickParams p{};
    p.car = e->car;
    p.sim = e->sim;
    p.carOut = e->carOut;
    p.diagCar = e->diagnostics ? e->diagCar : nullptr;
    p.diagSim = e->diagnostics ? e->diagSim : nullptr;
    p.actions = e->actions;
    p.carStride = e->carStride;
    p.simStride = e->simStride;
    p.globalCarBase = e->cfg.sim_offset * e->nCars;
    p.actionKind = (int)kind;
    p.nSim = e->cfg.n_sim;
    p.nCars = e->nCars;
    p.nBlue = e->cfg.n_blue;
    p.seed = e->cfg.seed;
    p.tick0 = e->tick;
    p.nTicks = nTicks;
    p.compatFlags = e->cfg.compat_flags;
    // A caller capturing the env stream into its own graph gets the kernels in that capture.
    cudaStreamCaptureStatus outer = cudaStreamCaptureStatusNone;
    ECHECK(e, cudaStreamIsCapturing(e->stream, &outer));
    if (e->useGraph && nTicks > 0 && outer == cudaStreamCaptureStatusNone)
    {
        cudaGraphExec_t exec = nullptr;
        for (const auto& g : e->graphs)
            if (g.kind == (int)kind && g.nTicks == nTicks && g.diag == e->diagnostics && g.timing == e->stageTiming &&
                g.hostIn == hostIn)
                exec = g.exec;
        if (!exec && e->graphs.size() < 16)
        {
            // Capture the launch once; every replay reads the tick count from tickDev.
            const int serr = stagedSetup();
            if (serr) return cudaFail(e, (cudaError_t)serr, "staged tick setup");
            TickParams q = p;
            q.tickDev = e->tickDev;
            ECHECK(e, cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
            const int lerr = launchTickStaged(q, e->arena(), e->scratch, e->stream, e->stageStreams(hostIn));
            cudaGraph_t graph = nullptr;
            const cudaError_t cerr = cudaStreamEndCapture(e->stream, &graph);
            if (lerr || cerr != cudaSuccess)
            {
                if (graph) cudaGraphDestroy(graph);
                return cudaFail(e, lerr ? (cudaError_t)lerr : cerr, "tick graph capture");
            }
            const cudaError_t werr = applyArenaWindow(e, graph);
            if (werr != cudaSuccess)
            {
                cudaGraphDestroy(graph);
                return cudaFail(e, werr, "tick graph access-policy window");
            }
            const cudaError_t ierr = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            if (ierr != cudaSuccess) return cudaFail(e, ierr, "tick graph instantiate");
            e->graphs.push_back({ (int)kind, nTicks, e->diagnostics, e->stageTiming, hostIn, exec });
        }
        if (exec)
        {
            ECHECK(e, cudaEventRecord(e->ev0, e->stream));
            const int serr = launchSetTick(e->tickDev, e->tick, e->stream);
            if (serr) return cudaFail(e, (cudaError_t)serr, "tick counter");
            ECHECK(e, cudaGraphLaunch(exec, e->stream));
            e->stageTimed = e->stageTiming;
            ECHECK(e, cudaEventRecord(e->ev1, e->stream));
            e->tick += nTicks;
            return CARLB_OK;
        }
    }
    ECHECK(e, cudaEventRecord(e->ev0, e->stream));
    const int err = launchTickStaged(p, e->arena(), e->scratch, e->stream, e->stageStreams(hostIn));
    if (err) return cudaFail(e, (cudaError_t)err, "tick kernel launch");
    e->stageTimed = e->stageTiming && nTicks > 0;
    ECHECK(e, cudaEventRecord(e->ev1, e->stream));
    e->tick += nTicks;
    return CARLB_OK;
}

carlb_status stageActions(carlb_env* e, carlb_action_kind kind, const void* src, cudaMemcpyKind dir)
{
    if (kind != CARLB_ACTIONS_DISCRETE && kind != CARLB_ACTIONS_CONTINUOUS && kind != CARLB_ACTIONS_DIRECT)
        return fail(e, CARLB_ERR_VALUE, "unknown action kind");
    if (!src) return fail(e, CARLB_ERR_VALUE, "actions pointer is null");
    const size_t bytes = (size_t)e->nCarTotal * actionRowBytes(kind);
    ECHECK(e, cudaMemcpyAsync(e->actions, src, bytes, dir, e->stream));
    return CARLB_OK;
}

// Number of non-empty sim slices of a staged launch.
int sliceCount(const carlb_env* e)
{
    int n = 0;
    for (int g = 0; g < 8; g++)
    {
        int s0 = 0, ns = 0;
        stageSlice(e->cfg.n_sim, e->groups, g, &s0, &ns);
        if (ns <= 0) break;
        n++;
    }
    return n;
}

// Host actions for a staged launch, copied slice by slice on the copy stream after
// the work already queued on the env stream (which covers the last launch's reads of
// the action buffer); actionsReady[g] marks slice g's rows.  The caller launches with
// hostIn, so each slice's controls stage waits for its own rows only.
carlb_status stageHostActionsSliced(carlb_env* e, carlb_action_kind kind, const void* src)
{
    if (kind != CARLB_ACTIONS_DISCRETE && kind != CARLB_ACTIONS_CONTINUOUS && kind != CARLB_ACTIONS_DIRECT)
        return fail(e, CARLB_ERR_VALUE, "unknown action kind");
    if (!src) return fail(e, CARLB_ERR_VALUE, "actions pointer is null");
    if (!e->copyStream)
    {
        ECHECK(e, cudaStreamCreateWithFlags(&e->copyStream, cudaStreamNonBlocking));
        ECHECK(e, cudaEventCreateWithFlags(&e->actionsIn, cudaEventDisableTiming));
        for (int g = 0; g < 8; g++) ECHECK(e, cudaEventCreateWithFlags(&e->actionsReady[g], cudaEventDisableTiming));
    }
    ECHECK(e, cudaEventRecord(e->actionsIn, e->stream));
    ECHECK(e, cudaStreamWaitEvent(e->copyStream, e->actionsIn, 0));
    const size_t rowBytes = (size_t)e->nCars * actionRowBytes(kind);
    for (int g = 0; g < 8; g++)
    {
        int s0 = 0, ns = 0;
        stageSlice(e->cfg.n_sim, e->groups, g, &s0, &ns);
        if (ns <= 0) break;
        ECHECK(e, cudaMemcpyAsync(static_cast<char*>(e->actions) + (size_t)s0 * rowBytes,
                                  static_cast<const char*>(src) + (size_t)s0 * rowBytes, (size_t)ns * rowBytes,
                                  cudaMemcpyHostToDevice, e->copyStream));
        ECHECK(e, cudaEventRecord(e->actionsReady[g], e->copyStream));
    }
    return CARLB_OK;
}

// Output packing after a reset / state injection (current outputs only).
void packCurrent(carlb_env* e, const uint8_t* mask)
{
    const GView g = e->view();
    launchPackObs(g, e->obs, mask, e->obsDim, e->cfg.invert_orange, e->cfg.normalize, e->cfg.previous_controls, e->stream);
    launchPackState(g, e->packed, e->stateDim, e->tick, 1, mask, e->stream);
    launchPackRawMatch(g, e->outputs(), mask, e->stream);
}

carlb_status resetEnv(carlb_env* e)
{
    const GView g = e->view();
    e->tick = 0;
    launchClear(g, e->stream);
    launchKickoff(g, 0, e->stream);
    launchPackObs(g, e->obs, nullptr, e->obsDim, e->cfg.invert_orange, e->cfg.normalize, e->cfg.previous_controls, e->stream);
    launchPackState(g, e->packed, e->stateDim, e->tick, 1, nullptr, e->stream);
    launchPackState(g, e->tpacked, e->stateDim, e->tick, 1, nullptr, e->stream);
    launchPackRewardsDones(g, e->outputs(), e->tick, e->maxTicks, e->overtimeTicks, e->noTouchTicks, e->stream);
    launchPackRawMatch(g, e->outputs(), nullptr, e->stream);
    ECHECK(e, cudaGetLastError());
    return CARLB_OK;
}

struct FieldMap
{
    void* base = nullptr;
    long long stride = 0;
    long long rows = 0;
    int word = 0, width = 0;
    bool readOnly = false;
    bool host = false;  // tick counter
};

bool mapField(carlb_env* e, int field, FieldMap& m)
{
    const long long n = e->nCarTotal, ns = e->cfg.n_sim;
    auto carW = [&](int w, int width) { m.base = e->car; m.stride = e->carStride; m.rows = n; m.word = w; m.width = width; };
    auto outW = [&](int w, int width) { m.base = e->carOut; m.stride = e->carStride; m.rows = n; m.word = w; m.width = width; };
    auto simW = [&](int w, int width) { m.base = e->sim; m.stride = e->simStride; m.rows = ns; m.word = w; m.width = width; };
    switch (field)
    {
    case CARLB_F_CAR_POS: carW(C_POS, 3); return true;
    case CARLB_F_CAR_VEL: carW(C_VEL, 3); return true;
    case CARLB_F_CAR_ANG: carW(C_ANG, 3); return true;
    case CARLB_F_CAR_ROT: carW(C_ROT, 4); return true;
    case CARLB_F_CAR_CEN: carW(C_CEN, 3); return true;
    case CARLB_F_CAR_IMP: carW(C_IMP, 3); return true;
    case CARLB_F_CAR_IS_DEMOED: carW(C_DEMOED, 1); return true;
    case CARLB_F_CAR_DEMO_TIMER: carW(C_DEMO_TIMER, 1); return true;
    case CARLB_F_CAR_CONTACT_IDX: carW(C_CONTACT_IDX, 1); return true;
    case CARLB_F_CAR_CONTACT_COOLDOWN: carW(C_CONTACT_CD, 1); return true;
    case CARLB_F_CAR_BALL_HIT_TICK: carW(C_BALL_HIT_TICK, 1); return true;
    case CARLB_F_CAR_BALL_CONTACT_TICK: carW(C_BALL_CONTACT_TICK, 1); return true;
    case CARLB_F_CAR_WHEEL_SOURCE: outW(O_WHEEL_SRC, 4); return true;
    case CARLB_F_CAR_WHEEL_CONTACT: outW(O_WHEEL_CON, 4); return true;
    case CARLB_F_CAR_ARENA_CONTACT_TICK: outW(O_ARENA_CONTACT_TICK, 1); return true;
    case CARLB_F_CAR_CONTROLS: outW(O_CONTROLS, 8); return true;
    case CARLB_F_CAR_INTERNAL: carW(C_INT, CARLB_INT_WORDS); return true;
    case CARLB_F_SUSP_SCALARS: carW(C_SUSP, CARLB_SUSP_WORDS); return true;
    case CARLB_F_SUSP_RAY_DIST: outW(O_RAY_DIST, 4); return true;
    case CARLB_F_SUSP_RAY_NORMAL: outW(O_RAY_NORMAL, 12); return true;
    case CARLB_F_SUSP_LAT_FRICTION: carW(C_LAT, 4); return true;
    case CARLB_F_SUSP_LON_FRICTION: carW(C_LON, 4); return true;
    case CARLB_F_MAN_COUNT: carW(C_MAN_COUNT, 1); return true;
    case CARLB_F_MAN_NORMAL0: carW(C_MAN_N0, 3); return true;
    case CARLB_F_BALL_POS: simW(S_BPOS, 3); return true;
    case CARLB_F_BALL_VEL: simW(S_BVEL, 3); return true;
    case CARLB_F_BALL_ANG: simW(S_BANG, 3); return true;
    case CARLB_F_BALL_IMP: simW(S_BIMP, 3); return true;
    case CARLB_F_BALL_INT_POS: simW(S_IPOS, 3); return true;
    case CARLB_F_BALL_INT_VEL: simW(S_IVEL, 3); return true;
    case CARLB_F_BALL_EXP_POS: simW(S_EPOS, 3); return true;
    case CARLB_F_BALL_EXP_VEL: simW(S_EVEL, 3); return true;
    case CARLB_F_BALL_INT_VALID: simW(S_IVALID, 1); return true;
    case CARLB_F_EPISODE_TICKS: simW(S_EP_TICKS, 1); return true;
    case CARLB_F_LAST_TOUCH_TICKS: simW(S_LAST_TOUCH, 1); return true;
    case CARLB_F_BALL_ARENA_CONTACT_TICK:
        m.base = e->simOut; m.stride = e->simStride; m.rows = ns; m.word = 0; m.width = 1; return true;
    case CARLB_F_GOALS: simW(S_GOALS, 5); return true;
    case CARLB_F_PAD_COOLDOWNS: simW(S_PADS, NUM_BOOST_PADS); return true;
    case CARLB_F_TICK_COUNT: m.rows = 1; m.width = 1; m.host = true; return true;
    case CARLB_F_DIAG_CELL_IDX:
        m.base = e->diagCar; m.stride = e->carStride; m.rows = n; m.word = 0; m.width = 1; m.readOnly = true; return true;
    case CARLB_F_DIAG_NUM_TRIS:
        m.base = e->diagCar; m.stride = e->carStride; m.rows = n; m.word = 1; m.width = 1; m.readOnly = true; return true;
    case CARLB_F_DIAG_SAT_PAIRS:
        m.base = e->diagCar; m.stride = e->carStride; m.rows = n; m.word = 2; m.width = 1 + MAX_CAR_TRI_PAIRS;
        m.readOnly = true; return true;
    case CARLB_F_DIAG_CC_COUNT:
    {
        const int pairs = e->nCars * (e->nCars - 1) / 2;
        m.base = e->diagSim; m.stride = e->simStride; m.rows = ns; m.word = 0; m.width = pairs > 0 ? pairs : 1;
        m.readOnly = true; return true;
    }
    default:
        return false;
    }
}

}  // namespace

extern "C" {

carlb_status carlb_destroy(carlb_env* e);

static carlb_status initEnv(carlb_env* p, const carlb_config* cfg)
{
    std::string err;
    const auto host = hostArena(arenaObjPath(libraryDir() + "/_data/arena.obj"), arenaMetadataPath(), err);
    if (!host) return fail(p, CARLB_ERR_STATE, err);

    p->cfg = *cfg;
    p->nCars = cfg->n_blue + cfg->n_orange;
    p->nCarTotal = (long long)cfg->n_sim * p->nCars;
    p->obsDim = observationDim(p->nCars, cfg->previous_controls != 0);
    p->stateDim = packedStateDim(p->nCars);
    p->actDim = p->nCars * ACT_PER_CAR;
    p->hitWords = (host->maxCellTris + 31) / 32;
    // Rows padded to whole warps of sims (and 4 words), so every per-word row is
    // 16-byte aligned.
    const long long simPad = ((long long)cfg->n_sim + 31) / 32 * 32;
    p->simStride = simPad;
    p->carStride = (simPad * p->nCars + 3) / 4 * 4;

    ECHECK(p, cudaSetDevice(cfg->device));
    ECHECK(p, cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking));
    ECHECK(p, cudaEventCreate(&p->ev0));
    ECHECK(p, cudaEventCreate(&p->ev1));

    ECHECK(p, allocZero(p, &p->car, (size_t)NCW * p->carStride));
    ECHECK(p, allocZero(p, &p->sim, (size_t)NSW * p->simStride));
    ECHECK(p, allocZero(p, &p->carOut, (size_t)NOW * p->carStride));
    ECHECK(p, allocZero(p, &p->simOut, (size_t)NSOW * p->simStride));
    ECHECK(p, allocZero(p, &p->obs, (size_t)p->nCarTotal * p->obsDim));
    ECHECK(p, allocZero(p, &p->tobs, (size_t)p->nCarTotal * p->obsDim));
    ECHECK(p, allocZero(p, &p->packed, (size_t)cfg->n_sim * p->stateDim));
    ECHECK(p, allocZero(p, &p->tpacked, (size_t)cfg->n_sim * p->stateDim));
    ECHECK(p, allocZero(p, &p->rewards, (size_t)cfg->n_sim));
    ECHECK(p, allocZero(p, &p->dones, (size_t)cfg->n_sim));
    ECHECK(p, allocZero(p, &p->overtime, (size_t)cfg->n_sim));
    ECHECK(p, allocZero(p, &p->tovertime, (size_t)cfg->n_sim));
    ECHECK(p, allocZero(p, &p->scoreDiff, (size_t)cfg->n_sim));
    ECHECK(p, allocZero(p, &p->episodeTicks, (size_t)cfg->n_sim));
    ECHECK(p, allocZero(p, &p->tScoreDiff, (size_t)cfg->n_sim));
    ECHECK(p, allocZero(p, &p->tEpisodeTicks, (size_t)cfg->n_sim));
    if (const char* fr = std::getenv("CARLB_FUSED_RESET")) p->fusedReset = std::atoi(fr) != 0;
    if (const char* sp = std::getenv("CARLB_STAGED_PACK")) p->stagedPack = std::atoi(sp) != 0;
    if (const char* fe = std::getenv("CARLB_FUSED_EPILOGUE")) p->fusedEpilogue = std::atoi(fe) != 0;
    {
        if (const char* g = std::getenv("CARLB_GROUPS")) p->groups = std::max(1, std::min(8, std::atoi(g)));
        // Slices of fewer than ~4k sims would leave the wide stages too small.
        p->groups = std::max(1, std::min(p->groups, cfg->n_sim / 4096));
        if (const char* b = std::getenv("CARLB_BALL_STREAM")) p->ballSide = std::atoi(b) != 0;
        if (const char* o = std::getenv("CARLB_PHASE_OFFSET")) p->phaseOffset = std::atoi(o) != 0;
        if (const char* gr = std::getenv("CARLB_GRAPH")) p->useGraph = std::atoi(gr) != 0;
        if (const char* oc = std::getenv("CARLB_OVERLAP_COPY")) p->overlapCopy = std::atoi(oc) != 0;
        if (const char* lw = std::getenv("CARLB_L2_WINDOW")) p->l2Window = std::atoi(lw) != 0;
        if (p->useGraph) ECHECK(p, allocZero(p, &p->tickDev, (size_t)1));
        for (int g = 0; g < p->groups; g++)
        {
            ECHECK(p, cudaStreamCreateWithFlags(&p->groupStream[g], cudaStreamNonBlocking));
            ECHECK(p, cudaEventCreateWithFlags(&p->groupJoin[g], cudaEventDisableTiming));
            ECHECK(p, cudaEventCreateWithFlags(&p->wideDone[g], cudaEventDisableTiming));
            if (p->ballSide)
            {
                ECHECK(p, cudaStreamCreateWithFlags(&p->ballStream[g], cudaStreamNonBlocking));
                ECHECK(p, cudaEventCreateWithFlags(&p->tickStart[g], cudaEventDisableTiming));
                ECHECK(p, cudaEventCreateWithFlags(&p->ballDone[g], cudaEventDisableTiming));
            }
        }
        ECHECK(p, cudaEventCreateWithFlags(&p->evFork, cudaEventDisableTiming));
        ECHECK(p, allocZero(p, &p->scratch.first, (size_t)p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.cnt, (size_t)p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.ray, (size_t)16 * p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.hits, (size_t)p->hitWords * p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.wheelBits, (size_t)p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.keys, (size_t)4 * p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.heavyBody, (size_t)18 * p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.heavyList, (size_t)HEAVY_CLASSES * p->carStride));
        ECHECK(p, allocZero(p, &p->scratch.heavyCount, (size_t)8 * HEAVY_CLASSES));
        ECHECK(p, allocZero(p, &p->scratch.ball, (size_t)15 * p->simStride));
        ECHECK(p, allocZero(p, &p->scratch.ballList, (size_t)p->simStride));
        ECHECK(p, allocZero(p, &p->scratch.ballCount, (size_t)8));
        ECHECK(p, allocZero(p, &p->scratch.ccCount, (size_t)8));
        ECHECK(p, allocZero(p, &p->scratch.stats, (size_t)8 * STAGE_WORK));
    }
    p->actionCapacity = (size_t)p->nCarTotal * 32;
    {
        uint8_t* a = nullptr;
        ECHECK(p, allocZero(p, &a, p->actionCapacity));
        p->actions = a;
    }

    // Arena tables: vertices expanded per triangle (flags in vertex 0's w).
    const int nTris = host->nTris();
    std::vector<float4> triV((size_t)nTris * 3), triAng(nTris);
    for (int t = 0; t < nTris; t++)
    {
        for (int k = 0; k < 3; k++)
        {
            const int v = host->tris[3 * t + k];
            float w = 0.f;
            if (k == 0) std::memcpy(&w, &host->triFlags[t], 4);
            triV[3 * t + k] = make_float4(host->verts[3 * v], host->verts[3 * v + 1], host->verts[3 * v + 2], w);
        }
        triAng[t] = make_float4(host->edgeAngles[3 * t], host->edgeAngles[3 * t + 1], host->edgeAngles[3 * t + 2], 0.f);
    }
    // Bounding spheres for the candidate culls, stored per cell-list entry so a
    // reject costs one load: a triangle whose sphere is farther than carReach
    // from a car's box centre can neither overlap the box (SAT) nor meet a wheel
    // ray, and one farther than the contact radius from the ball cannot touch
    // it, so skipping it leaves every result unchanged.
    std::vector<float4> triSph(nTris);
    for (int t = 0; t < nTris; t++)
    {
        double c[3] = { 0, 0, 0 };
        for (int k = 0; k < 3; k++)
            for (int d = 0; d < 3; d++) c[d] += (double)host->verts[3 * host->tris[3 * t + k] + d] / 3.0;
        double r2 = 0;
        for (int k = 0; k < 3; k++)
        {
            double q = 0;
            for (int d = 0; d < 3; d++)
            {
                const double e = (double)host->verts[3 * host->tris[3 * t + k] + d] - c[d];
                q += e * e;
            }
            r2 = std::max(r2, q);
        }
        triSph[t] = make_float4((float)c[0], (float)c[1], (float)c[2], (float)(std::sqrt(r2) * (1.0 + 1e-6) + 1e-2));
    }
    {
        double reach = std::sqrt((double)CAR_HALF_X * CAR_HALF_X + (double)CAR_HALF_Y * CAR_HALF_Y +
                                 (double)CAR_HALF_Z * CAR_HALF_Z);
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            const V3 conn = suspConnection(w);
            const double arm = std::sqrt((double)conn.x * conn.x + (double)conn.y * conn.y + (double)conn.z * conn.z);
            reach = std::max(reach, arm + (double)suspRayLength(w) + 1.0);
        }
        p->carReach = (float)(reach + 2.0);  // 2 uu margin over float rounding
    }
    std::vector<float4> cellSph(host->cellTris.size());
    for (size_t e = 0; e < cellSph.size(); e++) cellSph[e] = triSph[host->cellTris[e]];
    // Vertices per cell-list entry too, so a candidate's geometry is one load
    // away from its entry index rather than behind the triangle index.
    std::vector<float4> cellV(3 * host->cellTris.size());
    for (size_t e = 0; e < host->cellTris.size(); e++)
        for (int k = 0; k < 3; k++) cellV[3 * e + k] = triV[3 * (size_t)host->cellTris[e] + k];
    // Margin of the flat stage's plane pre-test per triangle, in distance units
    // times |n| (n = cross(v1 - v0, v2 - v0), the unnormalised normal the test
    // uses).  A box centre that passed the reach cull lies within D = 2r + carReach
    // of every vertex (r: the bounding-sphere radius).  The car-frame SAT projects
    // vertices at most D away onto a normal built from edges at least Lmin long,
    // so its rounding is bounded by a few ulp of D plus the normal's direction
    // error times D, about 1e-7 * D * D / Lmin.  The margin takes 100 times those
    // terms, plus 0.05 uu.  Degenerate triangles get an infinite margin (no skip).
    {
        std::vector<float> marginN(nTris);
        for (int t = 0; t < nTris; t++)
        {
            double v[3][3];
            for (int k = 0; k < 3; k++)
                for (int d = 0; d < 3; d++) v[k][d] = (double)host->verts[3 * host->tris[3 * t + k] + d];
            double e1[3], e2[3], e3[3];
            for (int d = 0; d < 3; d++)
            {
                e1[d] = v[1][d] - v[0][d];
                e2[d] = v[2][d] - v[0][d];
                e3[d] = v[2][d] - v[1][d];
            }
            const double n[3] = { e1[1] * e2[2] - e1[2] * e2[1], e1[2] * e2[0] - e1[0] * e2[2],
                                  e1[0] * e2[1] - e1[1] * e2[0] };
            const double nl = std::sqrt(n[0] * n[0] + n[1] * n[1] + n[2] * n[2]);
            auto len = [](const double* a) { return std::sqrt(a[0] * a[0] + a[1] * a[1] + a[2] * a[2]); };
            const double lmin = std::min(len(e1), std::min(len(e2), len(e3)));
            const double D = 2.0 * (double)triSph[t].w + (double)p->carReach;
            if (nl < 1e-3 || lmin < 1e-3)
            {
                marginN[t] = INFINITY;
                continue;
            }
            const double margin = 0.05 + 1e-4 * D + 1e-5 * D * D / lmin;
            marginN[t] = (float)(margin * nl * (1.0 + 1e-6));
        }
        for (size_t e = 0; e < host->cellTris.size(); e++) cellV[3 * e + 1].w = marginN[host->cellTris[e]];
    }
    ECHECK(p, allocArena(p, &p->cellV, cellV.size()));
    ECHECK(p, cudaMemcpyAsync(p->cellV, cellV.data(), cellV.size() * sizeof(float4), cudaMemcpyHostToDevice,
                              p->stream));
    {
        std::vector<float4> bsph(host->ballCellTris.size());
        for (size_t k = 0; k < bsph.size(); k++) bsph[k] = triSph[host->ballCellTris[k]];
        p->ballGrid = make_float4(host->ballOrigin[0], host->ballOrigin[1], host->ballOrigin[2], 1.f / host->ballCell);
        for (int k = 0; k < 3; k++) p->ballDims[k] = host->ballDims[k];
        ECHECK(p, allocArena(p, &p->ballCellStart, host->ballCellStart.size()));
        ECHECK(p, allocArena(p, &p->ballCellTris, std::max<size_t>(1, host->ballCellTris.size())));
        ECHECK(p, allocArena(p, &p->ballCellSph, std::max<size_t>(1, bsph.size())));
        ECHECK(p, cudaMemcpyAsync(p->ballCellStart, host->ballCellStart.data(), host->ballCellStart.size() * 4,
                                  cudaMemcpyHostToDevice, p->stream));
        ECHECK(p, cudaMemcpyAsync(p->ballCellTris, host->ballCellTris.data(), host->ballCellTris.size() * 4,
                                  cudaMemcpyHostToDevice, p->stream));
        ECHECK(p, cudaMemcpyAsync(p->ballCellSph, bsph.data(), bsph.size() * sizeof(float4), cudaMemcpyHostToDevice,
                                  p->stream));
        ECHECK(p, cudaStreamSynchronize(p->stream));  // the host vectors go out of scope
    }
    if (host->hasNative)
    {
        std::vector<float4> nv((size_t)nTris * 3), na(nTris);
        for (int t = 0; t < nTris; t++)
        {
            for (int k = 0; k < 3; k++)
            {
                float w = 0.f;
                if (k == 0) std::memcpy(&w, &host->nativeMesh[t], 4);
                const float* v = &host->nativeVerts[9 * (size_t)t + 3 * k];
                nv[3 * t + k] = make_float4(v[0], v[1], v[2], w);
            }
            float fw = 0.f;
            std::memcpy(&fw, &host->nativeFlags[t], 4);
            na[t] = make_float4(host->nativeAngles[3 * t], host->nativeAngles[3 * t + 1], host->nativeAngles[3 * t + 2], fw);
        }
        ECHECK(p, allocArena(p, &p->nativeV, nv.size()));
        ECHECK(p, allocArena(p, &p->nativeAng, na.size()));
        ECHECK(p, cudaMemcpyAsync(p->nativeV, nv.data(), nv.size() * sizeof(float4), cudaMemcpyHostToDevice, p->stream));
        ECHECK(p, cudaMemcpyAsync(p->nativeAng, na.data(), na.size() * sizeof(float4), cudaMemcpyHostToDevice,
                                  p->stream));
        ECHECK(p, cudaStreamSynchronize(p->stream));
        p->hasNative = 1;
    }
    ECHECK(p, allocArena(p, &p->cellSph, cellSph.size()));
    ECHECK(p, cudaMemcpyAsync(p->cellSph, cellSph.data(), cellSph.size() * sizeof(float4), cudaMemcpyHostToDevice,
                              p->stream));
    ECHECK(p, allocArena(p, &p->triV, triV.size()));
    ECHECK(p, allocArena(p, &p->triAng, triAng.size()));
    ECHECK(p, allocArena(p, &p->cellStart, host->cellStart.size()));
    ECHECK(p, allocArena(p, &p->cellTris, host->cellTris.size()));
    ECHECK(p, cudaMemcpyAsync(p->triV, triV.data(), triV.size() * sizeof(float4), cudaMemcpyHostToDevice, p->stream));
    ECHECK(p, cudaMemcpyAsync(p->triAng, triAng.data(), triAng.size() * sizeof(float4), cudaMemcpyHostToDevice, p->stream));
    ECHECK(p, cudaMemcpyAsync(p->cellStart, host->cellStart.data(), host->cellStart.size() * 4, cudaMemcpyHostToDevice, p->stream));
    ECHECK(p, cudaMemcpyAsync(p->cellTris, host->cellTris.data(), host->cellTris.size() * 4, cudaMemcpyHostToDevice, p->stream));

    if (p->l2Window)
    {
        ECHECK(p, poolArenaTables(p));
        if (p->arenaPool)
        {
            cudaStreamAttrValue v{};
            v.accessPolicyWindow = arenaWindow(p);
            for (int g = 0; g < 8; g++)
                for (cudaStream_t st : { p->groupStream[g], p->ballStream[g] })
                    if (st) ECHECK(p, cudaStreamSetAttribute(st, cudaStreamAttributeAccessPolicyWindow, &v));
            ECHECK(p, cudaStreamSetAttribute(p->stream, cudaStreamAttributeAccessPolicyWindow, &v));
        }
    }

    Tables tables;
    buildTables(tables);
    ECHECK(p, (cudaError_t)uploadTickTables(tables));
    ECHECK(p, (cudaError_t)uploadEnvioTables(tables));
    {
        // Set-up for carlb_ticks_static_scratch, once per device: look up the fixed
        // scratch array and load the stage kernels, so that entry point's calls
        // allocate nothing.
        void* base = nullptr;
        void* lastUse = nullptr;
        size_t capacity = 0;
        if (const int serr = staticScratchAddress(&base, &capacity, &lastUse))
            return cudaFail(p, (cudaError_t)serr, "static scratch set-up");
    }

    const carlb_status st = resetEnv(p);
    if (st != CARLB_OK) return st;
    ECHECK(p, cudaStreamSynchronize(p->stream));
    return CARLB_OK;
}

carlb_status carlb_create(const carlb_config* cfg, carlb_env** out)
{
    if (!out) return fail(nullptr, CARLB_ERR_VALUE, "out is null");
    *out = nullptr;
    if (!cfg) return fail(nullptr, CARLB_ERR_VALUE, "config is null");
    if (cfg->n_sim < 1) return fail(nullptr, CARLB_ERR_VALUE, "n_sim must be at least 1");
    if (cfg->n_blue < 0 || cfg->n_orange < 0 || cfg->n_blue + cfg->n_orange < 1)
        return fail(nullptr, CARLB_ERR_VALUE, "team sizes must be non-negative with at least one car");
    if (cfg->n_blue > 4 || cfg->n_orange > 4)
        return fail(nullptr, CARLB_ERR_VALUE, "at most 4 cars per team (4 kickoff spots per team)");
    if (cfg->frameskip < 1) return fail(nullptr, CARLB_ERR_VALUE, "frameskip must be at least 1");
    if (cfg->sim_offset < 0) return fail(nullptr, CARLB_ERR_VALUE, "sim_offset must be non-negative");
    if (cfg->compat_flags & ~CARLB_SOURCE_LAGGED_LATERAL_FRICTION)
        return fail(nullptr, CARLB_ERR_VALUE, "unknown compat_flags bits");

    carlb_env* p = new carlb_env;
    const carlb_status st = initEnv(p, cfg);
    if (st != CARLB_OK)
    {
        g_createError = p->error;
        carlb_destroy(p);
        return st;
    }
    *out = p;
    return CARLB_OK;
}

carlb_status carlb_destroy(carlb_env* e)
{
    if (!e) return CARLB_OK;
    cudaSetDevice(e->cfg.device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    for (int g = 0; g < 8; g++)
    {
        if (e->groupStream[g]) cudaStreamSynchronize(e->groupStream[g]);
        if (e->ballStream[g]) cudaStreamSynchronize(e->ballStream[g]);
    }
    for (const auto& g : e->graphs) cudaGraphExecDestroy(g.exec);
    for (void* v : e->allocations) cudaFree(v);
    if (e->ev0) cudaEventDestroy(e->ev0);
    if (e->ev1) cudaEventDestroy(e->ev1);
    for (int g = 0; g < 8; g++)
    {
        if (e->groupJoin[g]) cudaEventDestroy(e->groupJoin[g]);
        if (e->groupStream[g]) cudaStreamDestroy(e->groupStream[g]);
        if (e->tickStart[g]) cudaEventDestroy(e->tickStart[g]);
        if (e->ballDone[g]) cudaEventDestroy(e->ballDone[g]);
        if (e->wideDone[g]) cudaEventDestroy(e->wideDone[g]);
        if (e->ballStream[g]) cudaStreamDestroy(e->ballStream[g]);
    }
    if (e->evFork) cudaEventDestroy(e->evFork);
    if (e->copyStream)
    {
        cudaStreamSynchronize(e->copyStream);
        cudaStreamDestroy(e->copyStream);
    }
    if (e->actionsIn) cudaEventDestroy(e->actionsIn);
    for (int g = 0; g < 8; g++)
        if (e->actionsReady[g]) cudaEventDestroy(e->actionsReady[g]);
    for (int k = 0; k < 2 * STAGE_KERNELS; k++)
        if (e->stageEv[k]) cudaEventDestroy(e->stageEv[k]);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return CARLB_OK;
}

const char* carlb_last_error(const carlb_env* e) { return e ? e->error.c_str() : g_createError.c_str(); }

carlb_status carlb_ticks(carlb_env* e, carlb_action_kind kind, const void* actions, int32_t n)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (n < 0) return fail(e, CARLB_ERR_VALUE, "n_ticks must be non-negative");
    carlb_status s = stageActions(e, kind, actions, cudaMemcpyDeviceToDevice);
    if (s != CARLB_OK) return s;
    return launchTicks(e, kind, n);
}

carlb_status carlb_ticks_static_scratch(carlb_env* e, carlb_action_kind kind, const void* actions, int32_t n)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (n < 0) return fail(e, CARLB_ERR_VALUE, "n_ticks must be non-negative");
    // The caller's current device is restored on return (the address lookup and
    // the launches need the env's device current).
    int callerDevice = -1;
    ECHECK(e, cudaGetDevice(&callerDevice));
    struct RestoreDevice
    {
        int dev;
        ~RestoreDevice() { cudaSetDevice(dev); }
    } restore{ callerDevice };
    ECHECK(e, cudaSetDevice(e->cfg.device));
    void* base = nullptr;
    void* lastUse = nullptr;
    size_t capacity = 0;
    const int aerr = staticScratchAddress(&base, &capacity, &lastUse);
    if (aerr) return cudaFail(e, (cudaError_t)aerr, "static scratch lookup");

    // Carve the stage scratch out of the fixed array (each part 256-byte aligned).
    const size_t cs = (size_t)e->carStride, ss = (size_t)e->simStride;
    size_t off = 0;
    auto take = [&](size_t bytes) -> size_t {
        const size_t at = (off + 255) & ~(size_t)255;
        off = at + bytes;
        return at;
    };
    const size_t oFirst = take(cs * 4), oCnt = take(cs * 4), oRay = take(16 * cs * 4);
    const size_t oHits = take((size_t)e->hitWords * cs * 4), oWheel = take(cs * 4), oKeys = take(4 * cs * 8);
    const size_t oHeavyBody = take(18 * cs * 4), oHeavyList = take((size_t)HEAVY_CLASSES * cs * 4);
    const size_t oHeavyCount = take(8 * HEAVY_CLASSES * 4), oBall = take(15 * ss * 4), oBallList = take(ss * 4);
    const size_t oBallCount = take(8 * 4), oCcCount = take(8 * 4), oStats = take(8 * STAGE_WORK * 4);
    if (off > capacity)
        return fail(e, CARLB_ERR_VALUE,
                    "env needs " + std::to_string(off) + " bytes of stage scratch; the static scratch holds " +
                        std::to_string(capacity));
    char* b = static_cast<char*>(base);
    StageScratch x{};
    x.first = reinterpret_cast<int*>(b + oFirst);
    x.cnt = reinterpret_cast<int*>(b + oCnt);
    x.ray = reinterpret_cast<float*>(b + oRay);
    x.hits = reinterpret_cast<unsigned*>(b + oHits);
    x.wheelBits = reinterpret_cast<unsigned*>(b + oWheel);
    x.keys = reinterpret_cast<unsigned long long*>(b + oKeys);
    x.heavyBody = reinterpret_cast<float*>(b + oHeavyBody);
    x.heavyList = reinterpret_cast<int*>(b + oHeavyList);
    x.heavyCount = reinterpret_cast<int*>(b + oHeavyCount);
    x.ball = reinterpret_cast<float*>(b + oBall);
    x.ballList = reinterpret_cast<int*>(b + oBallList);
    x.ballCount = reinterpret_cast<int*>(b + oBallCount);
    x.ccCount = reinterpret_cast<int*>(b + oCcCount);
    x.stats = reinterpret_cast<int*>(b + oStats);

    carlb_status s = stageActions(e, kind, actions, cudaMemcpyDeviceToDevice);
    if (s != CARLB_OK) return s;
    // One call at a time uses the array: the env stream waits for the end of the
    // work the previous call enqueued (any env, any stream), and this call's end
    // is recorded in its place.  The lock keeps the wait and the record of
    // concurrent host threads in one order.
    static std::mutex order;
    std::lock_guard<std::mutex> guard(order);
    ECHECK(e, cudaStreamWaitEvent(e->stream, (cudaEvent_t)lastUse, 0));
    // The work-list counters start at zero (every other scratch word is written
    // before it is read within a tick).
    ECHECK(e, cudaMemsetAsync(x.heavyCount, 0, 8 * HEAVY_CLASSES * 4, e->stream));
    ECHECK(e, cudaMemsetAsync(x.ballCount, 0, 8 * 4, e->stream));
    ECHECK(e, cudaMemsetAsync(x.ccCount, 0, 8 * 4, e->stream));

    TickParams p{};
    p.car = e->car;
    p.sim = e->sim;
    p.carOut = e->carOut;
    p.diagCar = e->diagnostics ? e->diagCar : nullptr;
    p.diagSim = e->diagnostics ? e->diagSim : nullptr;
    p.actions = e->actions;
    p.carStride = e->carStride;
    p.simStride = e->simStride;
    p.globalCarBase = e->cfg.sim_offset * e->nCars;
    p.actionKind = (int)kind;
    p.nSim = e->cfg.n_sim;
    p.nCars = e->nCars;
    p.nBlue = e->cfg.n_blue;
    p.seed = e->cfg.seed;
    p.tick0 = e->tick;
    p.nTicks = n;
    p.compatFlags = e->cfg.compat_flags;
    StageStreams streams = e->stageStreams();
    for (int k = 0; k < 2 * STAGE_KERNELS; k++) streams.stageEvents[k] = nullptr;
    ECHECK(e, cudaEventRecord(e->ev0, e->stream));
    const int err = launchTickStaged(p, e->arena(), x, e->stream, streams);
    e->stageTimed = false;  // this call records no stage events
    if (err) return cudaFail(e, (cudaError_t)err, "tick kernel launch");
    ECHECK(e, cudaEventRecord(e->ev1, e->stream));
    // Every stage kernel of the launch has joined the env stream by here.
    ECHECK(e, cudaEventRecord((cudaEvent_t)lastUse, e->stream));
    e->tick += n;
    return CARLB_OK;
}

carlb_status carlb_ticks_host(carlb_env* e, carlb_action_kind kind, const void* hostActions, int32_t n,
                              float* hostRewards)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (n < 0) return fail(e, CARLB_ERR_VALUE, "n_ticks must be non-negative");
    cudaStreamCaptureStatus outer = cudaStreamCaptureStatusNone;
    ECHECK(e, cudaStreamIsCapturing(e->stream, &outer));
    const bool sliced = e->overlapCopy && n > 0 && outer == cudaStreamCaptureStatusNone;
    carlb_status s = sliced ? stageHostActionsSliced(e, kind, hostActions)
                            : stageActions(e, kind, hostActions, cudaMemcpyHostToDevice);
    if (s != CARLB_OK) return s;
    s = launchTicks(e, kind, n, sliced);
    if (s != CARLB_OK) return s;
    // The slices' controls stages already waited for their rows; this orders the
    // env stream after the last copy as well, whatever the launch read.
    if (sliced) ECHECK(e, cudaStreamWaitEvent(e->stream, e->actionsReady[sliceCount(e) - 1], 0));
    if (hostRewards)
    {
        launchPackRewardsDones(e->view(), e->outputs(), e->tick, e->maxTicks, e->overtimeTicks, e->noTouchTicks, e->stream);
        ECHECK(e, cudaMemcpyAsync(hostRewards, e->rewards, (size_t)e->cfg.n_sim * 4, cudaMemcpyDeviceToHost, e->stream));
    }
    ECHECK(e, cudaStreamSynchronize(e->stream));
    return CARLB_OK;
}

carlb_status carlb_env_step(carlb_env* e, carlb_action_kind kind, const void* actions)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (kind == CARLB_ACTIONS_DIRECT) return fail(e, CARLB_ERR_VALUE, "env_step takes discrete or continuous actions");
    carlb_status s = stageActions(e, kind, actions, cudaMemcpyDeviceToDevice);
    if (s != CARLB_OK) return s;
    s = launchTicks(e, kind, e->cfg.frameskip);
    if (s != CARLB_OK) return s;
    const GView g = e->view();
    const Outputs o = e->outputs();
    if (e->fusedEpilogue)
    {
        const StepOutputs a{ e->obs, e->tobs, e->packed, e->tpacked, e->obsDim, e->stateDim, e->cfg.invert_orange,
                             e->cfg.normalize, e->cfg.previous_controls, e->tick, e->cfg.frameskip, e->maxTicks,
                             e->overtimeTicks, e->noTouchTicks };
        launchStepEpilogue(g, o, a, e->stream);
        ECHECK(e, cudaGetLastError());
        return CARLB_OK;
    }
    launchPackRewardsDones(g, o, e->tick, e->maxTicks, e->overtimeTicks, e->noTouchTicks, e->stream);
    launchPackState(g, e->tpacked, e->stateDim, e->tick, e->cfg.frameskip, nullptr, e->stream);
    launchPackObs(g, e->tobs, e->dones, e->obsDim, e->cfg.invert_orange, e->cfg.normalize, e->cfg.previous_controls, e->stream);
    launchResetDones(g, e->tick, e->maxTicks, e->overtimeTicks, e->noTouchTicks, e->stream);
    launchPackRawMatch(g, o, nullptr, e->stream);
    launchPackObs(g, e->obs, nullptr, e->obsDim, e->cfg.invert_orange, e->cfg.normalize, e->cfg.previous_controls, e->stream);
    launchPackState(g, e->packed, e->stateDim, e->tick, 1, nullptr, e->stream);
    ECHECK(e, cudaGetLastError());
    return CARLB_OK;
}

carlb_status carlb_reset(carlb_env* e)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    return resetEnv(e);
}

carlb_status carlb_reset_dones(carlb_env* e)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    launchResetDones(e->view(), e->tick, e->maxTicks, e->overtimeTicks, e->noTouchTicks, e->stream);
    ECHECK(e, cudaGetLastError());
    return CARLB_OK;
}

carlb_status carlb_apply_reset_state(carlb_env* e, int32_t n, const float* ballPos, const float* ballVel,
                                     const float* ballAng, const float* carPos, const float* carRot,
                                     const float* carVel, const float* carAng, const void* demoed, int32_t demoedIsByte,
                                     const float* boost, const float* internal, const int32_t* blue,
                                     const int32_t* orange, const int32_t* ticks, const int64_t* indices,
                                     const uint8_t* mask)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (mask && indices) return fail(e, CARLB_ERR_VALUE, "specify reset_mask or simulation_indices, not both");
    if (mask) n = e->cfg.n_sim;
    if (n < 0 || n > e->cfg.n_sim) return fail(e, CARLB_ERR_VALUE, "too many simulation_indices");
    if (!ballPos || !ballVel || !ballAng || !carPos || !carRot || !carVel || !carAng || !demoed)
        return fail(e, CARLB_ERR_VALUE, "ball and car inputs are required");
    if ((blue == nullptr) != (orange == nullptr) || (blue == nullptr) != (ticks == nullptr))
        return fail(e, CARLB_ERR_VALUE, "blue_score, orange_score and episode_ticks must be supplied together");
    if (n == 0) return CARLB_OK;
    const GView g = e->view();
    const BallInputs ball{ ballPos, ballVel, ballAng };
    const CarInputs cars{ carPos, carRot, carVel, carAng, demoed, demoedIsByte, boost, internal };
    if (mask && e->fusedReset)
    {
        const PackTargets pk{ e->obs, e->obsDim, e->cfg.invert_orange, e->cfg.normalize, e->cfg.previous_controls,
                              e->packed, e->stateDim, e->tick, e->outputs() };
        launchResetMasked(g, e->arena(), ball, cars, MatchInputs{ blue, orange, ticks }, mask, pk, e->stream);
        ECHECK(e, cudaGetLastError());
        return CARLB_OK;
    }
    launchResetPads(g, n, indices, mask, e->stream);
    launchSetBall(g, ball, n, indices, mask, e->stream);
    launchSetCar(g, e->arena(), cars, n, indices, mask, e->stream);
    if (blue) launchSetMatch(g, blue, orange, ticks, n, indices, mask, e->stream);
    packCurrent(e, mask);
    ECHECK(e, cudaGetLastError());
    return CARLB_OK;
}

carlb_status carlb_set_ball(carlb_env* e, int32_t n, const float* pos, const float* vel, const float* ang,
                            const int64_t* indices)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (n < 0 || n > e->cfg.n_sim) return fail(e, CARLB_ERR_VALUE, "too many simulation_indices");
    if (!pos || !vel || !ang) return fail(e, CARLB_ERR_VALUE, "ball inputs are required");
    const GView g = e->view();
    launchSetBall(g, BallInputs{ pos, vel, ang }, n, indices, nullptr, e->stream);
    launchPackObs(g, e->obs, nullptr, e->obsDim, e->cfg.invert_orange, e->cfg.normalize, e->cfg.previous_controls, e->stream);
    launchPackState(g, e->packed, e->stateDim, e->tick, 1, nullptr, e->stream);
    launchPackState(g, e->tpacked, e->stateDim, e->tick, 1, nullptr, e->stream);
    ECHECK(e, cudaGetLastError());
    ECHECK(e, cudaStreamSynchronize(e->stream));
    return CARLB_OK;
}

carlb_status carlb_set_car(carlb_env* e, int32_t n, const float* pos, const float* rot, const float* vel,
                           const float* ang, const void* demoed, int32_t demoedIsByte, const float* boost,
                           const float* internal, const int64_t* indices)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (n < 0 || n > e->cfg.n_sim) return fail(e, CARLB_ERR_VALUE, "too many simulation_indices");
    if (!pos || !rot || !vel || !ang || !demoed) return fail(e, CARLB_ERR_VALUE, "car inputs are required");
    const GView g = e->view();
    launchSetCar(g, e->arena(), CarInputs{ pos, rot, vel, ang, demoed, demoedIsByte, boost, internal }, n, indices,
                 nullptr, e->stream);
    launchPackObs(g, e->obs, nullptr, e->obsDim, e->cfg.invert_orange, e->cfg.normalize, e->cfg.previous_controls, e->stream);
    launchPackState(g, e->packed, e->stateDim, e->tick, 1, nullptr, e->stream);
    launchPackState(g, e->tpacked, e->stateDim, e->tick, 1, nullptr, e->stream);
    ECHECK(e, cudaGetLastError());
    ECHECK(e, cudaStreamSynchronize(e->stream));
    return CARLB_OK;
}

carlb_status carlb_set_match_state(carlb_env* e, int32_t n, const int32_t* blue, const int32_t* orange,
                                   const int32_t* ticks, const int64_t* indices)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (n < 0 || n > e->cfg.n_sim) return fail(e, CARLB_ERR_VALUE, "too many simulation_indices");
    if (!blue || !orange || !ticks) return fail(e, CARLB_ERR_VALUE, "score and tick inputs are required");
    launchSetMatch(e->view(), blue, orange, ticks, n, indices, nullptr, e->stream);
    ECHECK(e, cudaGetLastError());
    return CARLB_OK;
}

carlb_status carlb_reset_boost_pads(carlb_env* e, int32_t n, const int64_t* indices)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (n < 0 || n > e->cfg.n_sim) return fail(e, CARLB_ERR_VALUE, "too many simulation_indices");
    launchResetPads(e->view(), n, indices, nullptr, e->stream);
    ECHECK(e, cudaGetLastError());
    ECHECK(e, cudaStreamSynchronize(e->stream));
    return CARLB_OK;
}

carlb_status carlb_get_buffer(carlb_env* e, carlb_buffer which, void** data, int64_t shape[3], int32_t* ndim,
                              carlb_dtype* dtype)
{
    if (!e || !data || !shape || !ndim || !dtype) return fail(e, CARLB_ERR_VALUE, "null argument");
    const int64_t ns = e->cfg.n_sim;
    shape[0] = ns;
    shape[1] = shape[2] = 0;
    *ndim = 1;
    switch (which)
    {
    case CARLB_BUF_OBS:
    case CARLB_BUF_TRANSITION_OBS:
        *data = which == CARLB_BUF_OBS ? e->obs : e->tobs;
        shape[1] = e->nCars; shape[2] = e->obsDim; *ndim = 3; *dtype = CARLB_F32; return CARLB_OK;
    case CARLB_BUF_STATE:
    case CARLB_BUF_TRANSITION_STATE:
        *data = which == CARLB_BUF_STATE ? e->packed : e->tpacked;
        shape[1] = e->stateDim; *ndim = 2; *dtype = CARLB_F32; return CARLB_OK;
    case CARLB_BUF_REWARDS: *data = e->rewards; *dtype = CARLB_F32; return CARLB_OK;
    case CARLB_BUF_DONES: *data = e->dones; *dtype = CARLB_BOOL; return CARLB_OK;
    case CARLB_BUF_SCORE_DIFFERENCE: *data = e->scoreDiff; *dtype = CARLB_I32; return CARLB_OK;
    case CARLB_BUF_EPISODE_TICKS: *data = e->episodeTicks; *dtype = CARLB_I32; return CARLB_OK;
    case CARLB_BUF_TRANSITION_SCORE_DIFFERENCE: *data = e->tScoreDiff; *dtype = CARLB_I32; return CARLB_OK;
    case CARLB_BUF_TRANSITION_EPISODE_TICKS: *data = e->tEpisodeTicks; *dtype = CARLB_I32; return CARLB_OK;
    case CARLB_BUF_OVERTIME: *data = e->overtime; *dtype = CARLB_BOOL; return CARLB_OK;
    case CARLB_BUF_TRANSITION_OVERTIME: *data = e->tovertime; *dtype = CARLB_BOOL; return CARLB_OK;
    default: return fail(e, CARLB_ERR_VALUE, "unknown buffer");
    }
}

carlb_status carlb_set_limit(carlb_env* e, carlb_limit which, int32_t v)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    switch (which)
    {
    case CARLB_LIMIT_MAX_TICKS:
        if (v < 1) return fail(e, CARLB_ERR_VALUE, "max_ticks must be at least 1");
        e->maxTicks = v; return CARLB_OK;
    case CARLB_LIMIT_OVERTIME_TIMEOUT_TICKS:
        if (v < 1) return fail(e, CARLB_ERR_VALUE, "overtime_timeout_ticks must be at least 1");
        e->overtimeTicks = v; return CARLB_OK;
    case CARLB_LIMIT_NO_TOUCH_TIMEOUT_TICKS:
        if (v < 0) return fail(e, CARLB_ERR_VALUE, "no_touch_timeout_ticks must be non-negative");
        e->noTouchTicks = v; return CARLB_OK;
    case CARLB_LIMIT_FRAMESKIP:
        if (v < 1) return fail(e, CARLB_ERR_VALUE, "frameskip must be at least 1");
        e->cfg.frameskip = v; return CARLB_OK;
    default: return fail(e, CARLB_ERR_VALUE, "unknown limit");
    }
}

carlb_status carlb_get_limit(const carlb_env* e, carlb_limit which, int32_t* v)
{
    if (!e || !v) return CARLB_ERR_VALUE;
    switch (which)
    {
    case CARLB_LIMIT_MAX_TICKS: *v = e->maxTicks; return CARLB_OK;
    case CARLB_LIMIT_OVERTIME_TIMEOUT_TICKS: *v = e->overtimeTicks; return CARLB_OK;
    case CARLB_LIMIT_NO_TOUCH_TIMEOUT_TICKS: *v = e->noTouchTicks; return CARLB_OK;
    case CARLB_LIMIT_FRAMESKIP: *v = e->cfg.frameskip; return CARLB_OK;
    default: return CARLB_ERR_VALUE;
    }
}

carlb_status carlb_dims(const carlb_env* e, int32_t dims[5])
{
    if (!e || !dims) return CARLB_ERR_VALUE;
    dims[0] = e->cfg.n_sim;
    dims[1] = e->nCars;
    dims[2] = e->obsDim;
    dims[3] = e->actDim;
    dims[4] = e->stateDim;
    return CARLB_OK;
}

void* carlb_stream(const carlb_env* e) { return e ? (void*)e->stream : nullptr; }

carlb_status carlb_synchronize(carlb_env* e)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    ECHECK(e, cudaStreamSynchronize(e->stream));
    return CARLB_OK;
}

carlb_status carlb_field_shape(const carlb_env* e, carlb_field field, int64_t* rows, int32_t* width)
{
    if (!e || !rows || !width) return CARLB_ERR_VALUE;
    FieldMap m;
    if (!mapField(const_cast<carlb_env*>(e), field, m)) return CARLB_ERR_VALUE;
    *rows = m.rows;
    *width = m.width;
    return CARLB_OK;
}

carlb_status carlb_read_field(carlb_env* e, carlb_field field, void* out)
{
    if (!e || !out) return fail(e, CARLB_ERR_VALUE, "null argument");
    FieldMap m;
    if (!mapField(e, field, m)) return fail(e, CARLB_ERR_VALUE, "unknown field");
    ECHECK(e, cudaStreamSynchronize(e->stream));
    uint32_t* dst = static_cast<uint32_t*>(out);
    if (m.host)
    {
        dst[0] = (uint32_t)e->tick;
        return CARLB_OK;
    }
    std::vector<uint32_t> col((size_t)m.rows);
    for (int k = 0; k < m.width; k++)
    {
        const uint32_t* src = static_cast<const uint32_t*>(m.base) + (long long)(m.word + k) * m.stride;
        ECHECK(e, cudaMemcpy(col.data(), src, (size_t)m.rows * 4, cudaMemcpyDeviceToHost));
        for (long long r = 0; r < m.rows; r++) dst[r * m.width + k] = col[r];
    }
    return CARLB_OK;
}

carlb_status carlb_write_field(carlb_env* e, carlb_field field, const void* in)
{
    if (!e || !in) return fail(e, CARLB_ERR_VALUE, "null argument");
    FieldMap m;
    if (!mapField(e, field, m)) return fail(e, CARLB_ERR_VALUE, "unknown field");
    if (m.readOnly) return fail(e, CARLB_ERR_VALUE, "field is read-only");
    ECHECK(e, cudaStreamSynchronize(e->stream));
    const uint32_t* src = static_cast<const uint32_t*>(in);
    if (m.host)
    {
        e->tick = (int)src[0];
        return CARLB_OK;
    }
    std::vector<uint32_t> col((size_t)m.rows);
    for (int k = 0; k < m.width; k++)
    {
        for (long long r = 0; r < m.rows; r++) col[r] = src[r * m.width + k];
        uint32_t* dst = static_cast<uint32_t*>(m.base) + (long long)(m.word + k) * m.stride;
        ECHECK(e, cudaMemcpy(dst, col.data(), (size_t)m.rows * 4, cudaMemcpyHostToDevice));
    }
    return CARLB_OK;
}

carlb_status carlb_set_stage_timing(carlb_env* e, int32_t enabled)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    ECHECK(e, cudaSetDevice(e->cfg.device));
    for (int k = 0; k < 2 * STAGE_KERNELS && enabled; k++)
        if (!e->stageEv[k]) ECHECK(e, cudaEventCreate(&e->stageEv[k]));
    e->stageTiming = enabled != 0;
    e->stageTimed = false;
    return CARLB_OK;
}

carlb_status carlb_stage_times(carlb_env* e, float* ms, int32_t capacity, int32_t* count)
{
    if (!e || !count) return fail(e, CARLB_ERR_VALUE, "env or count is null");
    *count = 0;
    if (!e->stageTimed) return fail(e, CARLB_ERR_STATE, "no timed launch since stage timing was enabled");
    for (int k = 0; k < STAGE_KERNELS && k < capacity; k++)
    {
        ECHECK(e, cudaEventSynchronize(e->stageEv[2 * k + 1]));
        ECHECK(e, cudaEventElapsedTime(&ms[k], e->stageEv[2 * k], e->stageEv[2 * k + 1]));
        *count = k + 1;
    }
    return CARLB_OK;
}

carlb_status carlb_stage_work(carlb_env* e, int32_t counts[4])
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (!counts) return fail(e, CARLB_ERR_VALUE, "counts is null");
    ECHECK(e, cudaSetDevice(e->cfg.device));
    ECHECK(e, cudaStreamSynchronize(e->stream));
    int host[8 * STAGE_WORK] = {};
    ECHECK(e, cudaMemcpy(host, e->scratch.stats, sizeof(host), cudaMemcpyDeviceToHost));
    for (int k = 0; k < STAGE_WORK; k++)
    {
        counts[k] = 0;
        for (int g = 0; g < 8; g++) counts[k] += host[g * STAGE_WORK + k];
    }
    return CARLB_OK;
}

carlb_status carlb_last_tick_ms(const carlb_env* e, float* ms)
{
    if (!e || !ms) return CARLB_ERR_VALUE;
    const cudaError_t err = cudaEventElapsedTime(ms, e->ev0, e->ev1);
    return err == cudaSuccess ? CARLB_OK : CARLB_ERR_CUDA;
}

carlb_status carlb_action_mask(const float* obs, int64_t rows, int32_t obsDim, int32_t previousControls,
                               uint8_t* mask, void* stream)
{
    if (rows < 0) return fail(nullptr, CARLB_ERR_VALUE, "rows must be non-negative");
    if (rows == 0) return CARLB_OK;
    if (!obs || !mask) return fail(nullptr, CARLB_ERR_VALUE, "obs and mask must not be null");
    if (reinterpret_cast<uintptr_t>(mask) % 4 != 0) return fail(nullptr, CARLB_ERR_VALUE, "mask must be 4-byte aligned");
    const int controls = previousControls ? OBS_PREVIOUS_CONTROLS : 0;
    if (obsDim < OBS_BALL + OBS_PER_CAR - OBS_EGO_FLIP_INDEX + controls)
        return fail(nullptr, CARLB_ERR_VALUE, "obs_dim is too small for an observation row");
    launchActionMask(obs, rows, obsDim, previousControls != 0, mask, (cudaStream_t)stream);
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(nullptr, CARLB_ERR_CUDA, std::string("action mask: ") + cudaGetErrorString(err));
    return CARLB_OK;
}

carlb_status carlb_set_diagnostics(carlb_env* e, int32_t enabled)
{
    if (!e) return fail(nullptr, CARLB_ERR_VALUE, "env is null");
    if (enabled && !e->diagCar)
    {
        ECHECK(e, allocZero(e, &e->diagCar, (size_t)DIAG_CAR_WORDS * e->carStride));
        ECHECK(e, allocZero(e, &e->diagSim, (size_t)DIAG_SIM_WORDS * e->simStride));
    }
    e->diagnostics = enabled != 0;
    return CARLB_OK;
}

}  // extern "C"
