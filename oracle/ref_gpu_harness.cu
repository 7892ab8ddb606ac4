/*
 * GPU reference harness: a C ABI over the reference's own CUDA build
 * (jwmccarthy/CARL src/{Kernels,EnvIO,RLEnvironment,ArenaMesh,RLConstants}.cu,
 * compiled unchanged for sm_100a with --fmad=false, see Makefile).
 *
 * It mirrors the reference's pybind11 wrapper (python/carl.cu:82-666,
 * EnvWrapper) without Python: construction and initial packing, the env step,
 * reset, apply_reset_state and the setters, plus snapshot access to every
 * persistent state array for parity tests and event timing of raw ticks for
 * the baseline measurement.  Inputs are host arrays; the harness stages them in
 * device memory on the reference env's stream.
 * TEST INFRASTRUCTURE: only tests and bench.py's reference arm use it.
 */
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <cub/device/device_scan.cuh>

#include "RLEnvironment.cuh"
#include "EnvIO.cuh"
#include "Kernels.cuh"

#include "ref_fields.h"

namespace {

thread_local std::string g_error;

#define HCHECK(call)                                                           \
    do {                                                                       \
        cudaError_t err_ = (call);                                             \
        if (err_ != cudaSuccess) {                                             \
            g_error = std::string(#call) + ": " + cudaGetErrorString(err_);    \
            return 1;                                                          \
        }                                                                      \
    } while (0)

struct DeviceBuffer
{
    void* ptr = nullptr;
    size_t bytes = 0;

    ~DeviceBuffer() { if (ptr) cudaFree(ptr); }

    cudaError_t assign(const void* host, size_t n, cudaStream_t stream)
    {
        if (n > bytes)
        {
            if (ptr) cudaFree(ptr);
            ptr = nullptr;
            const cudaError_t e = cudaMalloc(&ptr, n);
            if (e != cudaSuccess) return e;
            bytes = n;
        }
        if (!host || n == 0) return cudaSuccess;
        return cudaMemcpyAsync(ptr, host, n, cudaMemcpyHostToDevice, stream);
    }
};

struct RefGpu
{
    RLEnvironment env;
    EnvIO io;
    int frameskip;
    int obsDim, stateDim;
    DeviceBuffer actions;
    DeviceBuffer staging[16];
    cudaEvent_t start = nullptr, stop = nullptr;

    RefGpu(int nSim, int nBlue, int nOrange, int seed, int fs, bool inv, bool norm, bool prev)
        : env(nSim, nBlue, nOrange, seed)
        , io(nSim, env.getNCars(), env.getStream(), inv, norm, prev)
        , frameskip(fs)
        , obsDim(observationDim(nBlue + nOrange, prev))
        , stateDim(packedStateDim(nBlue + nOrange))
    {
        cudaEventCreate(&start);
        cudaEventCreate(&stop);
        initialPack();
    }

    ~RefGpu()
    {
        cudaStreamSynchronize(env.getStream());
        cudaEventDestroy(start);
        cudaEventDestroy(stop);
    }

    // EnvWrapper ctor / reset (python/carl.cu:286-310,372-381)
    void initialPack()
    {
        env.reset();
        io.packObs(env.getDeviceState());
        io.packState(env.getDeviceState());
        io.packTransitionState(env.getDeviceState(), 1);
        io.packRewardsDones(env.getDeviceState());
        io.packRawMatchState(env.getDeviceState());
    }

    void tickOnce(int kind, const void* deviceActions)
    {
        if (kind == CARLB_ACTIONS_DISCRETE) env.step(static_cast<const DiscreteControls*>(deviceActions));
        else if (kind == CARLB_ACTIONS_CONTINUOUS) env.step(static_cast<const ContinuousControls*>(deviceActions));
        else env.step(static_cast<const CarControls*>(deviceActions));
    }

    // EnvWrapper::step / stepContinuous (python/carl.cu:312-370)
    void envStep(int kind)
    {
        if (kind == CARLB_ACTIONS_DISCRETE) io.setActions(static_cast<const int32_t*>(actions.ptr));
        else io.setContinuousActions(static_cast<const float*>(actions.ptr));
        const void* a = kind == CARLB_ACTIONS_DISCRETE ? (const void*)io.getActions()
                                                       : (const void*)io.getContinuousActions();
        for (int t = 0; t < frameskip; t++) tickOnce(kind, a);
        io.packRewardsDones(env.getDeviceState());
        io.packTransitionState(env.getDeviceState(), frameskip);
        io.packTransitionObs(env.getDeviceState());
        env.resetDones(io.getMaxTicks(), io.getOvertimeTimeoutTicks(), io.getNoTouchTimeoutTicks());
        io.packRawMatchState(env.getDeviceState());
        io.packObs(env.getDeviceState());
        io.packState(env.getDeviceState());
    }

    // Host copies of the device structs: array pointers are device addresses.
    alignas(GameState) unsigned char stateBytes[sizeof(GameState)];
    alignas(Workspace) unsigned char spaceBytes[sizeof(Workspace)];

    int fetchStructs()
    {
        HCHECK(cudaStreamSynchronize(env.getStream()));
        HCHECK(cudaMemcpy(stateBytes, env.getDeviceState(), sizeof(GameState), cudaMemcpyDeviceToHost));
        HCHECK(cudaMemcpy(spaceBytes, env.getDeviceWorkspace(), sizeof(Workspace), cudaMemcpyDeviceToHost));
        return 0;
    }
    const GameState& hs() const { return *reinterpret_cast<const GameState*>(stateBytes); }
    const Workspace& hw() const { return *reinterpret_cast<const Workspace*>(spaceBytes); }
    const void* tickCountAddr()
    {
        return reinterpret_cast<const char*>(env.getDeviceState())
             + (reinterpret_cast<const char*>(&hs().tickCount) - reinterpret_cast<const char*>(stateBytes));
    }
};

RefCopy deviceFetch()
{
    return [](void* d, const void* s, size_t b) { if (b) cudaMemcpy(d, s, b, cudaMemcpyDeviceToHost); };
}
RefCopy deviceStore()
{
    return [](void* d, const void* s, size_t b) { if (b) cudaMemcpy(d, s, b, cudaMemcpyHostToDevice); };
}

size_t actionBytes(int kind, int nCars)
{
    return (size_t)nCars * (kind == CARLB_ACTIONS_DIRECT ? sizeof(CarControls) : 7 * sizeof(int32_t));
}

}  // namespace

extern "C" {

const char* carlrefgpu_error() { return g_error.c_str(); }

void* carlrefgpu_create(int nSim, int nBlue, int nOrange, int seed, int frameskip,
                        int invertOrange, int normalize, int previousControls)
{
    try
    {
        auto* e = new RefGpu(nSim, nBlue, nOrange, seed, frameskip,
                             invertOrange != 0, normalize != 0, previousControls != 0);
        const cudaError_t err = cudaStreamSynchronize(e->env.getStream());
        if (err != cudaSuccess)
        {
            g_error = cudaGetErrorString(err);
            delete e;
            return nullptr;
        }
        return e;
    }
    catch (const std::exception& ex)
    {
        g_error = ex.what();
        return nullptr;
    }
}

void carlrefgpu_destroy(void* h) { delete static_cast<RefGpu*>(h); }

int carlrefgpu_set_limits(void* h, int maxTicks, int overtimeTicks, int noTouchTicks, int frameskip)
{
    auto* e = static_cast<RefGpu*>(h);
    if (maxTicks > 0) e->io.setMaxTicks(maxTicks);
    if (overtimeTicks > 0) e->io.setOvertimeTimeoutTicks(overtimeTicks);
    if (noTouchTicks >= 0) e->io.setNoTouchTimeoutTicks(noTouchTicks);
    if (frameskip > 0) e->frameskip = frameskip;
    return 0;
}

int carlrefgpu_reset(void* h)
{
    auto* e = static_cast<RefGpu*>(h);
    e->initialPack();
    HCHECK(cudaStreamSynchronize(e->env.getStream()));
    return 0;
}

/* Raw ticks; `actions` is host memory ([n_cars_total, 7] or CarControls). */
int carlrefgpu_ticks(void* h, int kind, const void* actions, int nTicks)
{
    auto* e = static_cast<RefGpu*>(h);
    const size_t bytes = actionBytes(kind, e->env.getNSim() * e->env.getNCars());
    HCHECK(e->actions.assign(actions, bytes, e->env.getStream()));
    for (int t = 0; t < nTicks; t++) e->tickOnce(kind, e->actions.ptr);
    HCHECK(cudaGetLastError());
    HCHECK(cudaStreamSynchronize(e->env.getStream()));
    return 0;
}

/* Uploads actions once, then times `nTicks` raw ticks with events on the env
 * stream (device time, milliseconds). */
int carlrefgpu_time_ticks(void* h, int kind, const void* actions, int nTicks, float* ms)
{
    auto* e = static_cast<RefGpu*>(h);
    const size_t bytes = actionBytes(kind, e->env.getNSim() * e->env.getNCars());
    HCHECK(e->actions.assign(actions, bytes, e->env.getStream()));
    HCHECK(cudaStreamSynchronize(e->env.getStream()));
    HCHECK(cudaEventRecord(e->start, e->env.getStream()));
    for (int t = 0; t < nTicks; t++) e->tickOnce(kind, e->actions.ptr);
    HCHECK(cudaEventRecord(e->stop, e->env.getStream()));
    HCHECK(cudaEventSynchronize(e->stop));
    HCHECK(cudaEventElapsedTime(ms, e->start, e->stop));
    return 0;
}

int carlrefgpu_env_step(void* h, int kind, const void* actions)
{
    auto* e = static_cast<RefGpu*>(h);
    const size_t bytes = actionBytes(kind, e->env.getNSim() * e->env.getNCars());
    HCHECK(e->actions.assign(actions, bytes, e->env.getStream()));
    e->envStep(kind);
    HCHECK(cudaGetLastError());
    HCHECK(cudaStreamSynchronize(e->env.getStream()));
    return 0;
}

int carlrefgpu_reset_dones(void* h)
{
    auto* e = static_cast<RefGpu*>(h);
    e->env.resetDones(e->io.getMaxTicks(), e->io.getOvertimeTimeoutTicks(), e->io.getNoTouchTimeoutTicks());
    HCHECK(cudaStreamSynchronize(e->env.getStream()));
    return 0;
}

int carlrefgpu_get_buffer(void* h, int which, void* out)
{
    auto* e = static_cast<RefGpu*>(h);
    HCHECK(cudaStreamSynchronize(e->env.getStream()));
    DLManagedTensor* t = nullptr;
    switch (which)
    {
    case CARLB_BUF_OBS: t = e->io.getObsTensor(); break;
    case CARLB_BUF_TRANSITION_OBS: t = e->io.getTransitionObsTensor(); break;
    case CARLB_BUF_STATE: t = e->io.getStateTensor(); break;
    case CARLB_BUF_TRANSITION_STATE: t = e->io.getTransitionStateTensor(); break;
    case CARLB_BUF_REWARDS: t = e->io.getRewardsTensor(); break;
    case CARLB_BUF_DONES: t = e->io.getDonesTensor(); break;
    case CARLB_BUF_SCORE_DIFFERENCE: t = e->io.getScoreDifferenceTensor(); break;
    case CARLB_BUF_EPISODE_TICKS: t = e->io.getEpisodeTicksTensor(); break;
    case CARLB_BUF_TRANSITION_SCORE_DIFFERENCE: t = e->io.getTransitionScoreDifferenceTensor(); break;
    case CARLB_BUF_TRANSITION_EPISODE_TICKS: t = e->io.getTransitionEpisodeTicksTensor(); break;
    case CARLB_BUF_OVERTIME: t = e->io.getOvertimeTensor(); break;
    case CARLB_BUF_TRANSITION_OVERTIME: t = e->io.getTransitionOvertimeTensor(); break;
    default: g_error = "unknown buffer"; return 1;
    }
    int64_t count = 1;
    for (int d = 0; d < t->dl_tensor.ndim; d++) count *= t->dl_tensor.shape[d];
    const size_t bytes = (size_t)count * (t->dl_tensor.dtype.bits / 8);
    const cudaError_t err = cudaMemcpy(out, t->dl_tensor.data, bytes, cudaMemcpyDeviceToHost);
    t->deleter(t);
    HCHECK(err);
    return 0;
}

int carlrefgpu_read_field(void* h, int field, void* out)
{
    auto* e = static_cast<RefGpu*>(h);
    if (e->fetchStructs()) return 1;
    const RefField f = refField(e->hs(), e->hw(), field, e->tickCountAddr());
    if (f.rows < 0) { g_error = "unknown field"; return 1; }
    uint32_t* words = static_cast<uint32_t*>(out);
    if (field == CARLB_F_DIAG_SAT_PAIRS)
    {
        const int n = e->hs().nTotalCars;
        std::vector<int> hits(n), tris((size_t)n * MAX_CAR_TRI_PAIRS);
        HCHECK(cudaMemcpy(hits.data(), e->hw().ctHit.carHitCount.ptr, n * sizeof(int), cudaMemcpyDeviceToHost));
        HCHECK(cudaMemcpy(tris.data(), e->hw().ctNrw.triIdx.ptr, tris.size() * sizeof(int), cudaMemcpyDeviceToHost));
        for (int car = 0; car < n; car++)
        {
            const int count = hits[car] < MAX_CAR_TRI_PAIRS ? hits[car] : MAX_CAR_TRI_PAIRS;
            uint32_t* row = words + (size_t)car * f.width;
            std::memset(row, 0xff, sizeof(uint32_t) * f.width);
            row[0] = (uint32_t)count;
            for (int s = 0; s < count; s++) row[1 + s] = (uint32_t)tris[(size_t)car * MAX_CAR_TRI_PAIRS + s];
        }
        return 0;
    }
    refReadField(f, words, deviceFetch());
    HCHECK(cudaGetLastError());
    return 0;
}

int carlrefgpu_write_field(void* h, int field, const void* in)
{
    auto* e = static_cast<RefGpu*>(h);
    if (e->fetchStructs()) return 1;
    const RefField f = refField(e->hs(), e->hw(), field, e->tickCountAddr());
    if (f.rows < 0 || f.readOnly) { g_error = "field is unknown or read-only"; return 1; }
    refWriteField(f, static_cast<const uint32_t*>(in), deviceFetch(), deviceStore());
    HCHECK(cudaGetLastError());
    return 0;
}

/* Runs the kernels of one tick up to and including `lastStage` (stage numbers
 * follow src/RLEnvironment.cu:200-211: 0 begin, 1 broadphase, 2 scan,
 * 3 raycast, 4 controls, 5 SAT, 6 clip, 7 car-arena solve, 8 car-car + ball,
 * 9 integrate, 10 impulse cache, 11 boost pads), with the reference's own
 * kernels and launch shapes.  Used to localise parity differences. */
int carlrefgpu_tick_partial(void* h, int kind, const void* actions, int lastStage)
{
    auto* e = static_cast<RefGpu*>(h);
    cudaStream_t s = e->env.getStream();
    const int nSim = e->env.getNSim();
    const int n = nSim * e->env.getNCars();
    const size_t bytes = actionBytes(kind, n);
    HCHECK(e->actions.assign(actions, bytes, s));
    if (e->fetchStructs()) return 1;
    GameState* ds = e->env.getDeviceState();
    Workspace* dw = e->env.getDeviceWorkspace();
    ArenaMesh* da = e->env.getDeviceArena();
    int sms = 0;
    HCHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
    const int perCar = (n + 255) / 256;
    const int perSim = (nSim + 31) / 32;
    for (int stage = 0; stage <= lastStage; stage++)
    {
        switch (stage)
        {
        case 0: beginStepKernel<<<perCar, 256, 0, s>>>(ds, dw); break;
        case 1: carArenaBroadPhaseKernel<<<perCar, 256, 0, s>>>(ds, dw, da); break;
        case 2:
        {
            size_t tmp = 0;
            int* in = e->hw().bp.numTris.ptr;
            int* out = e->hw().bp.triPrefix.ptr;
            HCHECK(cub::DeviceScan::ExclusiveSum(nullptr, tmp, in, out, n + 1, s));
            DeviceBuffer scratch;
            HCHECK(scratch.assign(nullptr, tmp, s));
            HCHECK(cub::DeviceScan::ExclusiveSum(scratch.ptr, tmp, in, out, n + 1, s));
            HCHECK(cudaStreamSynchronize(s));
            break;
        }
        case 3: carSuspensionRaycastKernel<<<perCar, 256, 0, s>>>(ds, dw, da); break;
        case 4:
            if (kind == CARLB_ACTIONS_DISCRETE) carControlsKernel<<<perCar, 256, 0, s>>>(ds, dw, (const DiscreteControls*)e->actions.ptr);
            else if (kind == CARLB_ACTIONS_CONTINUOUS) carContinuousControlsKernel<<<perCar, 256, 0, s>>>(ds, dw, (const ContinuousControls*)e->actions.ptr);
            else carDirectControlsKernel<<<perCar, 256, 0, s>>>(ds, dw, (const CarControls*)e->actions.ptr);
            break;
        case 5: carArenaSATKernel<<<sms * 8, 128, 0, s>>>(ds, dw, da); break;
        case 6: carArenaClipKernel<<<sms * 8, 128, 0, s>>>(da, dw); break;
        case 7: carArenaSolveKernel<<<sms * 3, 256, 0, s>>>(ds, dw, da); break;
        case 8: carCarBallSolveKernel<<<perSim, 32, 0, s>>>(ds, dw, da); break;
        case 9: integrateCarsKernel<<<perCar, 256, 0, s>>>(ds); break;
        case 10: applyImpulseCacheKernel<<<perCar, 256, 0, s>>>(ds); break;
        case 11: boostPadKernel<<<(nSim * NUM_BOOST_PADS + 127) / 128, 128, 0, s>>>(ds); break;
        default: break;
        }
        HCHECK(cudaGetLastError());
    }
    HCHECK(cudaStreamSynchronize(s));
    return 0;
}

/* Times `nSteps` env steps (python/carl.cu:312-370, frameskip ticks + packing),
 * each followed by the masked apply_reset_state sequence of python/carl.cu:508-666
 * (pads, ball, cars with contact refresh, match state, obs / state / raw match
 * repack of the masked sims) with masks[step * n_sim ...]; with masks NULL the
 * steps run alone.  Actions and reset inputs (one row per sim, kickoff states
 * for instance) are staged once; device time of the steps and of the resets is
 * summed separately (milliseconds). */
int carlrefgpu_time_reset_steps(
    void* h, int kind, const void* actions, int nSteps,
    const float* ballPos, const float* ballVel, const float* ballAng,
    const float* carPos, const float* carRot, const float* carVel, const float* carAng,
    const uint8_t* demoed, const int32_t* blue, const int32_t* orange, const int32_t* ticks,
    const uint8_t* masks, float* stepMs, float* resetMs)
{
    auto* e = static_cast<RefGpu*>(h);
    cudaStream_t s = e->env.getStream();
    const int nCars = e->env.getNCars();
    const int nSim = e->env.getNSim();
    const size_t v3 = (size_t)nSim * 3 * 4, c3 = (size_t)nSim * nCars * 3 * 4;
    HCHECK(e->actions.assign(actions, actionBytes(kind, nSim * nCars), s));
    DeviceBuffer* b = e->staging;
    HCHECK(b[0].assign(ballPos, v3, s));
    HCHECK(b[1].assign(ballVel, v3, s));
    HCHECK(b[2].assign(ballAng, v3, s));
    HCHECK(b[3].assign(carPos, c3, s));
    HCHECK(b[4].assign(carRot, (size_t)nSim * nCars * 4 * 4, s));
    HCHECK(b[5].assign(carVel, c3, s));
    HCHECK(b[6].assign(carAng, c3, s));
    HCHECK(b[7].assign(demoed, (size_t)nSim * nCars, s));
    HCHECK(b[12].assign(blue, (size_t)nSim * 4, s));
    HCHECK(b[13].assign(orange, (size_t)nSim * 4, s));
    HCHECK(b[14].assign(ticks, (size_t)nSim * 4, s));
    if (masks) HCHECK(b[15].assign(masks, (size_t)nSteps * nSim, s));
    HCHECK(cudaStreamSynchronize(s));
    cudaEvent_t mid = nullptr;
    HCHECK(cudaEventCreate(&mid));
    float stepTotal = 0.f, resetTotal = 0.f;
    for (int step = 0; step < nSteps; step++)
    {
        GameState* ds = e->env.getDeviceState();
        cudaEventRecord(e->start, s);
        e->envStep(kind);
        cudaEventRecord(mid, s);
        if (masks)
        {
        const bool* dMask = reinterpret_cast<const bool*>(static_cast<const uint8_t*>(b[15].ptr) + (size_t)step * nSim);
        e->io.resetBoostPads(ds, nullptr, nSim, dMask);
        e->io.setBall(ds, (const float*)b[0].ptr, (const float*)b[1].ptr, (const float*)b[2].ptr, nullptr, nSim, dMask);
        e->io.setCar(ds, e->env.getDeviceWorkspace(), e->env.getDeviceArena(),
                     (const float*)b[3].ptr, (const float*)b[4].ptr, (const float*)b[5].ptr,
                     (const float*)b[6].ptr, b[7].ptr, true, nullptr, nullptr, nullptr, nSim, dMask);
        e->io.setMatchState(ds, (const int32_t*)b[12].ptr, (const int32_t*)b[13].ptr, (const int32_t*)b[14].ptr,
                            nullptr, nSim, dMask);
        e->io.packObs(ds, dMask);
        e->io.packState(ds, dMask);
        e->io.packRawMatchState(ds, dMask);
        }
        cudaEventRecord(e->stop, s);
        const cudaError_t err = cudaEventSynchronize(e->stop);
        if (err != cudaSuccess)
        {
            cudaEventDestroy(mid);
            g_error = cudaGetErrorString(err);
            return 1;
        }
        float a = 0.f, c = 0.f;
        cudaEventElapsedTime(&a, e->start, mid);
        cudaEventElapsedTime(&c, mid, e->stop);
        stepTotal += a;
        resetTotal += c;
    }
    cudaEventDestroy(mid);
    HCHECK(cudaGetLastError());
    *stepMs = stepTotal;
    *resetMs = resetTotal;
    return 0;
}

/* apply_reset_state (python/carl.cu:508-666) with host inputs; NULL for the
 * optional ones.  demoed is u8 when demoedIsByte, else int32. */
int carlrefgpu_apply_reset_state(
    void* h, int nSelected,
    const float* ballPos, const float* ballVel, const float* ballAng,
    const float* carPos, const float* carRot, const float* carVel, const float* carAng,
    const void* demoed, int demoedIsByte, const float* boost, const float* internal,
    const int32_t* blue, const int32_t* orange, const int32_t* ticks,
    const int64_t* indices, const uint8_t* mask)
{
    auto* e = static_cast<RefGpu*>(h);
    cudaStream_t s = e->env.getStream();
    const int nCars = e->env.getNCars();
    const int nSim = e->env.getNSim();
    if (mask) nSelected = nSim;
    const size_t v3 = (size_t)nSelected * 3 * 4, c3 = (size_t)nSelected * nCars * 3 * 4;
    DeviceBuffer* b = e->staging;
    HCHECK(b[0].assign(ballPos, v3, s));
    HCHECK(b[1].assign(ballVel, v3, s));
    HCHECK(b[2].assign(ballAng, v3, s));
    HCHECK(b[3].assign(carPos, c3, s));
    HCHECK(b[4].assign(carRot, (size_t)nSelected * nCars * 4 * 4, s));
    HCHECK(b[5].assign(carVel, c3, s));
    HCHECK(b[6].assign(carAng, c3, s));
    HCHECK(b[7].assign(demoed, (size_t)nSelected * nCars * (demoedIsByte ? 1 : 4), s));
    const float* dBoost = nullptr;
    const float* dInternal = nullptr;
    const int64_t* dIdx = nullptr;
    const bool* dMask = nullptr;
    if (boost) { HCHECK(b[8].assign(boost, (size_t)nSelected * nCars * 4, s)); dBoost = (const float*)b[8].ptr; }
    if (internal) { HCHECK(b[9].assign(internal, (size_t)nSelected * nCars * CAR_INTERNAL_SIZE * 4, s)); dInternal = (const float*)b[9].ptr; }
    if (indices) { HCHECK(b[10].assign(indices, (size_t)nSelected * 8, s)); dIdx = (const int64_t*)b[10].ptr; }
    if (mask) { HCHECK(b[11].assign(mask, (size_t)nSim, s)); dMask = (const bool*)b[11].ptr; }
    if (nSelected == 0) return 0;

    GameState* ds = e->env.getDeviceState();
    e->io.resetBoostPads(ds, dIdx, nSelected, dMask);
    e->io.setBall(ds, (const float*)b[0].ptr, (const float*)b[1].ptr, (const float*)b[2].ptr,
                  dIdx, nSelected, dMask);
    e->io.setCar(ds, e->env.getDeviceWorkspace(), e->env.getDeviceArena(),
                 (const float*)b[3].ptr, (const float*)b[4].ptr, (const float*)b[5].ptr,
                 (const float*)b[6].ptr, b[7].ptr, demoedIsByte != 0, dBoost, dInternal,
                 dIdx, nSelected, dMask);
    if (blue)
    {
        HCHECK(b[12].assign(blue, (size_t)nSelected * 4, s));
        HCHECK(b[13].assign(orange, (size_t)nSelected * 4, s));
        HCHECK(b[14].assign(ticks, (size_t)nSelected * 4, s));
        e->io.setMatchState(ds, (const int32_t*)b[12].ptr, (const int32_t*)b[13].ptr,
                            (const int32_t*)b[14].ptr, dIdx, nSelected, dMask);
    }
    e->io.packObs(ds, dMask);
    e->io.packState(ds, dMask);
    e->io.packRawMatchState(ds, dMask);
    HCHECK(cudaGetLastError());
    HCHECK(cudaStreamSynchronize(s));
    return 0;
}

}  // extern "C"
