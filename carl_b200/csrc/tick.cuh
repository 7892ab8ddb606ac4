// Launch-side description of the stage kernels of the tick and the device arena.
#pragma once

#include <cstdint>

#include "cb_state.cuh"

namespace cb {

// Action encodings (numbering of carlb_action_kind).
enum ActionKind : int { ACT_DISCRETE = 0, ACT_CONTINUOUS = 1, ACT_DIRECT = 2 };

struct ArenaDev
{
    const float4* triV;     // [nTris * 3]: vertices; .w of vertex 0 holds the TRI_* flag bits
    const float4* triAng;   // [nTris]: signed edge angles (edge i = v_i -> v_(i+1)%3)
    const int* cellStart;   // [NUM_CELLS + 1]
    const int* cellTris;    // [cellStart[NUM_CELLS]]
    int hitWords;           // ceil(max triangles per cell / 32)
    const float4* cellSph;  // [cellStart[NUM_CELLS]]: bounding sphere of cellTris[e] (centre xyz, radius w),
                            // radius rounded up
    float carReach;         // radius around a car's box centre that holds its box and wheel rays, plus margin
    const float4* cellV;    // [3 * cellStart[NUM_CELLS]]: vertices of cellTris[e] (flags in vertex 0's w;
                            // vertex 1's w: the plane pre-test margin times |cross(v1 - v0, v2 - v0)|)
    // Ball grid (ArenaHost::ball*): origin xyz and 1 / cell size in w, dimensions,
    // per-cell triangle lists and the bounding sphere of each list entry.
    float4 ballGrid;
    int ballDimX, ballDimY, ballDimZ;
    const int* ballCellStart;
    const int* ballCellTris;
    const float4* ballCellSph;
    // Native mesh metadata (ArenaHost::native*), used by the ball when hasNative:
    // Bullet-unit vertices (w of vertex 0: the native mesh, negative = no ball
    // contact), and the native edge angles with the edge flag bits in w.
    int hasNative;
    const float4* nativeV;    // [nTris * 3]
    const float4* nativeAng;  // [nTris]
};

struct TickParams
{
    float* car;             // [NCW][carStride]
    float* sim;             // [NSW][simStride]
    float* carOut;          // [NOW][carStride]
    int* diagCar;           // optional [DIAG_CAR_WORDS][carStride]
    int* diagSim;           // optional [DIAG_SIM_WORDS][simStride]
    const void* actions;    // [nCars total][7] (8 words for direct controls)
    long long carStride, simStride;
    long long globalCarBase;  // env-global index of this env's car 0
    int actionKind;
    int nSim, nCars, nBlue, seed;
    int tick0;              // tick count before the first tick of this launch
    const int* tickDev;     // staged path: when set, the tick count is read from here instead
                            // (lets a captured graph of the launch be replayed at any tick)
    int nTicks;
    int compatFlags;        // carlb_config::compat_flags
};

// Scratch of the staged path (device arrays, word-major with the env's strides).
struct StageScratch
{
    int* first;             // [carStride] first cell-list entry of the car's candidates
    int* cnt;               // [carStride] candidate count
    float* ray;             // [16][carStride] ray distance (4), ray normal (12)
    unsigned* hits;         // [hitWords][carStride] SAT hit bitmask over candidates
    unsigned* wheelBits;    // [carStride] wheels with a ray contact this tick
    unsigned long long* keys;  // [4][carStride] wheel ray minimum (distance bits, candidate)
    float* heavyBody;       // [18][carStride] velocities after the suspension of listed cars
    int* heavyList;         // [HEAVY_CLASSES][carStride] cars with possible plane contacts only / with
                            // SAT hits, this tick
    int* heavyCount;        // [slices][HEAVY_CLASSES] entries of each list; zero between ticks
    float* ball;            // [15][simStride] ball stage hand-over values
    int* ballList;          // [simStride] sims whose ball is moving (arena work), this tick
    int* ballCount;         // [slices] entries of each slice's ballList; zero between ticks
    int* ccCount;           // [slices] sims whose car-car stage had a pair in reach; zero between ticks
    int* stats;             // [slices][STAGE_WORK] the last tick's work-list sizes (see STAGE_WORK)
};

struct Tables;
// Copies the game tables into this kernel's constant memory.
int uploadTickTables(const Tables& t);

// Contact work lists: cars with plane contacts only, cars with SAT hits.
constexpr int HEAVY_CLASSES = 2;
// Work-list sizes kept per slice for the last tick (carlb_stage_work): cars listed
// for the contact stage with plane contacts only, cars listed with SAT hits,
// moving balls listed for the ball stage, sims with a car-car pair in reach.
constexpr int STAGE_WORK = 4;

// Stage kernels of one tick of the staged path, in launch order:
// ballPrep, flat, ray, ctlSusp (controls + suspension), contact, carCar, ball, finish.
constexpr int STAGE_KERNELS = 8;

// Streams and events of the staged path (cudaStream_t / cudaEvent_t): the sims
// are split into `groups` slices stepped concurrently on streams[0..groups).
struct StageStreams
{
    int groups;
    void* streams[8];
    void* join[8];        // event per slice: its last kernel
    void* fork;           // event: work queued on the env stream before the launch
    void* ballStreams[8]; // optional side stream per slice for the ball's arena stage
    void* tickStart[8];   // event per slice: the previous tick's finish (side stream waits)
    void* ballDone[8];    // event per slice: the ball's arena stage (finish waits)
    void* wideDone[8];    // optional event per slice: its wide stages of the tick (phase offset)
    void* stageEvents[2 * STAGE_KERNELS];  // optional: start / end events of slice 0's stage
                                           // kernels in the last tick of the launch
    void* actionsReady[8];  // optional event per slice: its action rows are in place (recorded on
                            // a copy stream before the launch; the slice's first controls stage waits)
};

// Sims [*s0, *s0 + *ns) of slice g when nSim sims are stepped as `groups` slices
// (clamped to 1..8); *ns <= 0 means slice g is empty.
inline void stageSlice(int nSim, int groups, int g, int* s0, int* ns)
{
    groups = groups < 1 ? 1 : (groups > 8 ? 8 : groups);
    const int per = (nSim + groups - 1) / groups;
    *s0 = g * per;
    *ns = nSim - *s0 < per ? nSim - *s0 : per;
}

// Capacity of the file-scope device scratch used by carlb_ticks_static_scratch.
constexpr size_t STATIC_SCRATCH_BYTES = 64ull << 20;
// Device address of that scratch on the current device, and an event
// (cudaEvent_t) that marks the end of the last work enqueued on it, so that
// calls from different envs and streams are ordered on the device.  The first
// call on a device looks the address up, creates the event and loads every
// stage kernel the static-scratch ticks launch; carlb_create makes that call,
// so the ticks themselves allocate nothing.
int staticScratchAddress(void** ptr, size_t* bytes, void** lastUse);

// One-time per-device setup of the staged kernels (shared-memory opt-in); call
// before capturing a launch into a graph.
int stagedSetup();
// Writes `value` to the device tick counter `dst` on `stream`.
int launchSetTick(int* dst, int value, void* stream);

// The same ticks as a sequence of stage kernels over the state in global memory.
int launchTickStaged(const TickParams& p, const ArenaDev& a, const StageScratch& x, void* stream,
                     const StageStreams& aux);

}  // namespace cb
