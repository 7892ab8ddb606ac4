// Launch wrappers for reset, state injection and output packing (envio.cu).
#pragma once

#include <cuda_runtime.h>

#include "cb_state.cuh"
#include "cb_tables.hpp"
#include "tick.cuh"

namespace cb {

// Global-memory view of one env's state.
struct GView
{
    GlobSoa car;         // NCW words per car
    GlobSoa out;         // NOW words per car
    GlobSoa sim;         // NSW words per sim
    int* simOut;         // [nSim] ball-arena contact tick (written by resets only)
    int nSim, nCars, nBlue, nOrange, seed;
    long long simOffset; // env-global index of sim 0
    bool stagedPack;     // obs / state rows through per-warp staging tiles (coalesced stores)
};

struct Outputs
{
    float* rewards;
    uint8_t* dones;
    int* scoreDiff;
    int* episodeTicks;
    int* transitionScoreDiff;
    int* transitionEpisodeTicks;
    uint8_t* overtime;
    uint8_t* transitionOvertime;
};

struct BallInputs
{
    const float *pos, *vel, *ang;  // [n, 3]
};

struct CarInputs
{
    const float *pos, *rot, *vel, *ang;  // [n, nCars, 3|4]
    const void* demoed;                  // [n, nCars] u8 or i32
    int demoedIsByte;
    const float* boost;                  // [n, nCars] or null
    const float* internal;               // [n, nCars, CAR_INTERNAL_SIZE] or null
};

struct MatchInputs
{
    const int32_t *blue, *orange, *ticks;  // [n] each, or all null
};

// Output buffers a masked reset repacks.
struct PackTargets
{
    float* obs;
    int obsDim, invertOrange, normalize, previousControls;
    float* state;
    int stateDim, tick;
    Outputs outputs;
};

// Output buffers and limits of an env step's epilogue.
struct StepOutputs
{
    float *obs, *tobs, *state, *tstate;
    int obsDim, stateDim, invertOrange, normalize, previousControls;
    int tick, frameskip, maxTicks, overtimeTicks, noTouchTicks;
};

int uploadEnvioTables(const Tables& t);
void launchClear(const GView& g, cudaStream_t s);
void launchKickoff(const GView& g, int tick, cudaStream_t s);
void launchResetDones(const GView& g, int tick, int maxTicks, int overtimeTicks, int noTouchTicks, cudaStream_t s);
void launchPackObs(const GView& g, float* out, const uint8_t* mask, int obsDim, bool invertOrange, bool normalize,
                   bool previousControls, cudaStream_t s);
void launchPackState(const GView& g, float* out, int stateDim, int tick, int touchWindow, const uint8_t* mask,
                     cudaStream_t s);
void launchPackRewardsDones(const GView& g, const Outputs& o, int tick, int maxTicks, int overtimeTicks,
                            int noTouchTicks, cudaStream_t s);
void launchPackRawMatch(const GView& g, const Outputs& o, const uint8_t* mask, cudaStream_t s);
void launchSetBall(const GView& g, const BallInputs& in, int n, const int64_t* idx, const uint8_t* mask, cudaStream_t s);
void launchSetCar(const GView& g, const ArenaDev& a, const CarInputs& in, int n, const int64_t* idx,
                  const uint8_t* mask, cudaStream_t s);
void launchSetMatch(const GView& g, const int32_t* blue, const int32_t* orange, const int32_t* ticks, int n,
                    const int64_t* idx, const uint8_t* mask, cudaStream_t s);
void launchResetPads(const GView& g, int n, const int64_t* idx, const uint8_t* mask, cudaStream_t s);
// Everything an env step does after its ticks, in one launch: rewards / dones,
// transition state and obs (done sims), auto-reset, raw match, obs and state.
void launchStepEpilogue(const GView& g, const Outputs& o, const StepOutputs& a, cudaStream_t s);
// Action mask rows [rows, ACTION_LOGITS] (u8) of observation rows [rows, obsDim].
void launchActionMask(const float* obs, long long rows, int obsDim, bool previousControls, uint8_t* mask,
                      cudaStream_t s);
// Masked apply_reset_state (all sims with mask[sim] != 0, input row = sim) and
// the repacking of their obs, state and raw match outputs, in one launch.
void launchResetMasked(const GView& g, const ArenaDev& a, const BallInputs& ball, const CarInputs& cars,
                       const MatchInputs& match, const uint8_t* mask, const PackTargets& pk, cudaStream_t s);

}  // namespace cb
