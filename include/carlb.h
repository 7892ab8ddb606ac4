/*
 * carlb.h — C ABI of the B200-native batched Rocket League tick.
 *
 * One `carlb_env` owns n_sim independent arenas (n_blue + n_orange cars and one
 * ball each) resident on one CUDA device, plus the observation / state / reward
 * buffers the reinforcement-learning front end reads.  Every entry point returns a
 * `carlb_status`; nothing here calls exit().  Device pointers are plain CUDA
 * device addresses on the env's device; host pointers are ordinary host memory.
 *
 * Reference interface each entry point replaces (paths inside jwmccarthy/CARL):
 *   carlb_create / carlb_destroy      python/carl.cu:286-310 (EnvWrapper ctor),
 *                                     src/RLEnvironment.cu:40-82
 *   carlb_env_step                    python/carl.cu:312-370 (step / step_continuous)
 *   carlb_ticks                       src/RLEnvironment.cu:166-211 (RLEnvironment::step)
 *   carlb_reset                       python/carl.cu:372-381, src/RLEnvironment.cu:192-198
 *   carlb_apply_reset_state           python/carl.cu:508-666
 *   carlb_set_ball / carlb_set_car    python/carl.cu:384-506, src/EnvIO.cu:137-318,603-680
 *   carlb_set_match_state             python/carl.cu:668-688, src/EnvIO.cu:320-336
 *   carlb_reset_boost_pads            python/carl.cu:690-706, src/EnvIO.cu:338-357
 *   carlb_get_buffer                  python/carl.cu:708-770, src/EnvIO.cu:452-545
 *   carlb_set_limit                   python/carl.cu:804-842 (max_ticks, ... frameskip)
 *   carlb_stream                      python/carl.cu:780-783
 *   carlb_read_field / write_field    no single counterpart: full snapshot of the
 *                                     persistent tick state (include/State/GameState.cuh,
 *                                     include/State/Workspace.cuh) for parity checks
 */
#ifndef CARLB_H
#define CARLB_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct carlb_env carlb_env;

typedef enum carlb_status {
    CARLB_OK = 0,
    CARLB_ERR_VALUE = 1,   /* bad argument value / shape  (Python: ValueError)   */
    CARLB_ERR_TYPE = 2,    /* bad dtype                   (Python: TypeError)    */
    CARLB_ERR_CUDA = 3,    /* CUDA runtime failure        (Python: RuntimeError) */
    CARLB_ERR_STATE = 4    /* env unusable / missing data (Python: RuntimeError) */
} carlb_status;

typedef struct carlb_config {
    int32_t n_sim;
    int32_t n_blue;
    int32_t n_orange;
    int32_t seed;
    int32_t frameskip;          /* >= 1 */
    int32_t invert_orange;      /* bool */
    int32_t normalize;          /* bool */
    int32_t previous_controls;  /* bool */
    int32_t device;             /* CUDA device ordinal */
    int32_t compat_flags;       /* CARLB_SOURCE_* bits; 0 = what the reference's CUDA build computes */
    int64_t sim_offset;         /* global index of this env's sim 0 (sharding) */
} carlb_config;

/* compat_flags bits.  With no bit set (the default) the tick reproduces what the
 * reference's sm_100a CUDA build computes, which is what the parity tests hold to
 * bit-exact candidate lists and SAT pair sets and the 1e-4 / 1e-3 state tolerance.
 * CARLB_SOURCE_LAGGED_LATERAL_FRICTION: use the previous tick's lateral wheel
 * friction coefficient, as the reference's source intends
 * (include/Physics/CarSuspension.cuh:206-209).  Its CUDA build reads that value
 * with __ldg in the thread that also stores the new one, and nvcc 12.9 (-O3,
 * sm_100a) orders the load after the store, so the build consumes the current
 * tick's coefficient; the reference compiled for a host CPU follows the source.
 * Any other bit is rejected with CARLB_ERR_VALUE. */
#define CARLB_SOURCE_LAGGED_LATERAL_FRICTION 1

/* Action encodings (one record of 7 values per car, [n_sim, n_cars, 7]). */
typedef enum carlb_action_kind {
    CARLB_ACTIONS_DISCRETE = 0,    /* int32 indices, ACTION_NVECS = (3,3,3,2,2,3,2) */
    CARLB_ACTIONS_CONTINUOUS = 1,  /* float32 in [low, high]                       */
    CARLB_ACTIONS_DIRECT = 2       /* CarControls: 5 float32 + 3 int32 = 8 words    */
} carlb_action_kind;

/* Output buffers owned by the env (non-owning views, overwritten in place). */
typedef enum carlb_buffer {
    CARLB_BUF_OBS = 0,                       /* f32 [n_sim, n_cars, obs_dim] */
    CARLB_BUF_TRANSITION_OBS = 1,            /* f32 [n_sim, n_cars, obs_dim] */
    CARLB_BUF_STATE = 2,                     /* f32 [n_sim, state_dim]       */
    CARLB_BUF_TRANSITION_STATE = 3,          /* f32 [n_sim, state_dim]       */
    CARLB_BUF_REWARDS = 4,                   /* f32 [n_sim]                  */
    CARLB_BUF_DONES = 5,                     /* bool(u8) [n_sim]             */
    CARLB_BUF_SCORE_DIFFERENCE = 6,          /* i32 [n_sim]                  */
    CARLB_BUF_EPISODE_TICKS = 7,             /* i32 [n_sim]                  */
    CARLB_BUF_TRANSITION_SCORE_DIFFERENCE = 8,
    CARLB_BUF_TRANSITION_EPISODE_TICKS = 9,
    CARLB_BUF_OVERTIME = 10,                 /* bool(u8) [n_sim]             */
    CARLB_BUF_TRANSITION_OVERTIME = 11,
    CARLB_BUF_COUNT = 12
} carlb_buffer;

typedef enum carlb_dtype {
    CARLB_F32 = 0,
    CARLB_I32 = 1,
    CARLB_BOOL = 2,
    CARLB_I64 = 3
} carlb_dtype;

typedef enum carlb_limit {
    CARLB_LIMIT_MAX_TICKS = 0,               /* >= 1 */
    CARLB_LIMIT_OVERTIME_TIMEOUT_TICKS = 1,  /* >= 1 */
    CARLB_LIMIT_NO_TOUCH_TIMEOUT_TICKS = 2,  /* >= 0 */
    CARLB_LIMIT_FRAMESKIP = 3                /* >= 1 */
} carlb_limit;

/*
 * Snapshot fields: the complete persistent tick state.  Every field is a dense
 * row-major array of 32-bit words; `width` words per entity.  Entity kinds:
 * car (n_sim * n_cars rows, sim-major), sim (n_sim rows), global (1 row), and
 * per-tick diagnostics written by the last tick (read-only).
 */
typedef enum carlb_field {
    CARLB_F_CAR_POS = 0,            /* f32 x3 */
    CARLB_F_CAR_VEL = 1,            /* f32 x3 */
    CARLB_F_CAR_ANG = 2,            /* f32 x3 */
    CARLB_F_CAR_ROT = 3,            /* f32 x4 quaternion (x, y, z, w) */
    CARLB_F_CAR_CEN = 4,            /* f32 x3 hitbox centre */
    CARLB_F_CAR_IMP = 5,            /* f32 x3 pending bump impulse */
    CARLB_F_CAR_IS_DEMOED = 6,      /* i32 */
    CARLB_F_CAR_DEMO_TIMER = 7,     /* f32 */
    CARLB_F_CAR_CONTACT_IDX = 8,    /* i32 env-global car index of last bump victim */
    CARLB_F_CAR_CONTACT_COOLDOWN = 9,   /* f32 */
    CARLB_F_CAR_BALL_HIT_TICK = 10,     /* i32 */
    CARLB_F_CAR_BALL_CONTACT_TICK = 11, /* i32 */
    CARLB_F_CAR_WHEEL_SOURCE = 12,  /* i32 x4 */
    CARLB_F_CAR_WHEEL_CONTACT = 13, /* i32 x4 */
    CARLB_F_CAR_ARENA_CONTACT_TICK = 14, /* i32 */
    CARLB_F_CAR_CONTROLS = 15,      /* 8 words: throttle steer yaw pitch roll (f32) jump boost slide (i32) */
    CARLB_F_CAR_INTERNAL = 16,      /* 24 words, see CARLB_INT_* */
    CARLB_F_SUSP_SCALARS = 17,      /* 15 f32, see CARLB_SUSP_* */
    CARLB_F_SUSP_RAY_DIST = 18,     /* f32 x4 */
    CARLB_F_SUSP_RAY_NORMAL = 19,   /* f32 x12 (4 wheels x xyz) */
    CARLB_F_SUSP_LAT_FRICTION = 20, /* f32 x4 (one-tick-lagged coefficient) */
    CARLB_F_SUSP_LON_FRICTION = 21, /* f32 x4 */
    CARLB_F_MAN_COUNT = 22,         /* i32 car-arena manifold point count (last tick) */
    CARLB_F_MAN_NORMAL0 = 23,       /* f32 x3 world normal of manifold point 0 */
    CARLB_F_BALL_POS = 24,          /* sim: f32 x3 */
    CARLB_F_BALL_VEL = 25,
    CARLB_F_BALL_ANG = 26,
    CARLB_F_BALL_IMP = 27,
    CARLB_F_BALL_INT_POS = 28,      /* Bullet-unit (x0.02) integration cache */
    CARLB_F_BALL_INT_VEL = 29,
    CARLB_F_BALL_EXP_POS = 30,
    CARLB_F_BALL_EXP_VEL = 31,
    CARLB_F_BALL_INT_VALID = 32,    /* i32 */
    CARLB_F_EPISODE_TICKS = 33,     /* i32 */
    CARLB_F_LAST_TOUCH_TICKS = 34,  /* i32 */
    CARLB_F_BALL_ARENA_CONTACT_TICK = 35, /* i32 */
    CARLB_F_GOALS = 36,             /* i32 x5: blue, orange, last_scorer, tick, overtime */
    CARLB_F_PAD_COOLDOWNS = 37,     /* f32 x34 */
    CARLB_F_TICK_COUNT = 38,        /* global: i32 x1 */
    /* per-tick diagnostics (read-only) */
    CARLB_F_DIAG_CELL_IDX = 39,     /* car: i32 broadphase grid cell */
    CARLB_F_DIAG_NUM_TRIS = 40,     /* car: i32 candidate triangle count */
    CARLB_F_DIAG_SAT_PAIRS = 41,    /* car: i32 x33 = [n_hits, tri ids...] (capacity 32) */
    CARLB_F_DIAG_CC_COUNT = 42,     /* sim: i32 x(n_cars*(n_cars-1)/2) car-car contact counts */
    CARLB_F_COUNT = 43
} carlb_field;

/* Words of CARLB_F_CAR_INTERNAL (i = int32 word, f = float32 word). */
enum {
    CARLB_INT_ON_GROUND = 0,          /* i */
    CARLB_INT_AIR_TIME = 1,           /* f */
    CARLB_INT_AIR_TIME_SINCE_JUMP = 2,/* f */
    CARLB_INT_HANDBRAKE = 3,          /* f */
    CARLB_INT_HAS_JUMPED = 4,         /* i */
    CARLB_INT_IS_JUMPING = 5,         /* i */
    CARLB_INT_JUMP_TIME = 6,          /* f */
    CARLB_INT_LAST_JUMP = 7,          /* i */
    CARLB_INT_HAS_DOUBLE_JUMPED = 8,  /* i */
    CARLB_INT_HAS_FLIPPED = 9,        /* i */
    CARLB_INT_IS_FLIPPING = 10,       /* i */
    CARLB_INT_FLIP_TIME = 11,         /* f */
    CARLB_INT_IS_AUTO_FLIPPING = 12,  /* i */
    CARLB_INT_AUTO_FLIP_TIMER = 13,   /* f */
    CARLB_INT_AUTO_FLIP_SCALE = 14,   /* f */
    CARLB_INT_FLIP_TORQUE_X = 15,     /* f */
    CARLB_INT_FLIP_TORQUE_Y = 16,     /* f */
    CARLB_INT_FLIP_TORQUE_Z = 17,     /* f */
    CARLB_INT_RESPAWN_IDX = 18,       /* i */
    CARLB_INT_LAST_RESPAWN_DIR = 19,  /* i */
    CARLB_INT_IS_BOOSTING = 20,       /* i */
    CARLB_INT_BOOST = 21,             /* f */
    CARLB_INT_BOOSTING_TIME = 22,     /* f */
    CARLB_INT_TIME_SINCE_BOOSTED = 23,/* f */
    CARLB_INT_WORDS = 24
};

/* Words of CARLB_F_SUSP_SCALARS (all float32). */
enum {
    CARLB_SUSP_BRAKE = 0,
    CARLB_SUSP_BRAKE_PREV = 1,
    CARLB_SUSP_THROTTLE = 2,
    CARLB_SUSP_RAW_THROTTLE = 3,
    CARLB_SUSP_HANDBRAKE = 4,
    CARLB_SUSP_STEER = 5,
    CARLB_SUSP_STEER_PREV = 6,
    CARLB_SUSP_ENGINE = 7,
    CARLB_SUSP_ENGINE_PREV = 8,
    CARLB_SUSP_JUMP_IMP_X = 9,
    CARLB_SUSP_JUMP_IMP_Y = 10,
    CARLB_SUSP_JUMP_IMP_Z = 11,
    CARLB_SUSP_ANG_IMP_X = 12,
    CARLB_SUSP_ANG_IMP_Y = 13,
    CARLB_SUSP_ANG_IMP_Z = 14,
    CARLB_SUSP_WORDS = 15
};

/* ---- lifetime ---------------------------------------------------------- */
carlb_status carlb_create(const carlb_config* cfg, carlb_env** out);
carlb_status carlb_destroy(carlb_env* env);
/* Last error message for `env` (or the last failed carlb_create when env is NULL). */
const char* carlb_last_error(const carlb_env* env);

/* ---- stepping ------------------------------------------------------------ */
/* One RL step: frameskip ticks, rewards/dones, transition packing, auto-reset of
 * finished sims, fresh obs/state.  `actions` is a device pointer, [n_sim, n_cars, 7]. */
carlb_status carlb_env_step(carlb_env* env, carlb_action_kind kind, const void* actions);
/* Raw physics ticks only (no packing, no auto-reset); `actions` device pointer,
 * [n_sim*n_cars, 7] (8 words for CARLB_ACTIONS_DIRECT). */
carlb_status carlb_ticks(carlb_env* env, carlb_action_kind kind, const void* actions, int32_t n_ticks);
/* Same as carlb_ticks but `host_actions` is host memory: the copy to the device,
 * the ticks and a copy back of the packed rewards into `host_rewards` (f32 [n_sim],
 * may be NULL) are ordered after the work already on the env stream; returns after
 * the stream drains, so both buffers are free again on return.  On the staged path
 * the actions are copied slice by slice on a side stream and each sim slice starts
 * its controls stage once its own rows are in (the copy overlaps the first tick's
 * broadphase; pinned host memory lets it run asynchronously). */
carlb_status carlb_ticks_host(carlb_env* env, carlb_action_kind kind, const void* host_actions,
                              int32_t n_ticks, float* host_rewards);
/* Same ticks as carlb_ticks, for callers that must not allocate device memory
 * while they step: a control loop with a latency budget, where cudaMalloc and
 * cudaFree can stall on the whole device, or a process whose device memory is
 * owned by another allocator (a framework's caching pool), where a new
 * cudaMalloc can fail.  This call allocates nothing (no cudaMalloc, cudaFree or
 * allocating library routine): the stage scratch comes from a fixed 64 MiB
 * file-scope device array, which every GPU that loads this library holds until
 * the process exits.  carlb_create does the set-up once per device: it looks up
 * the array's device address and loads every stage kernel this call launches,
 * so that even the first call loads no code under lazy module loading.  An env
 * that needs more than 64 MiB of stage scratch (roughly 224 bytes per car and
 * 64 per sim: about 47,000 sims at 3v3) gets CARLB_ERR_VALUE before anything is
 * enqueued.  Every call shares the array, which keeps the last call's contents
 * (the work-list counters are cleared on each call).  Calls that overlapped on
 * the GPU would race on it, so each call's work waits on the device for the
 * previous call's work (any env, any stream) before it touches the array: calls
 * run one after another on the GPU even when their streams are independent.
 * The caller's current device is the same on return.  No per-stage timing is recorded
 * (carlb_stage_times then reports CARLB_ERR_STATE).  No counterpart in the
 * reference. */
carlb_status carlb_ticks_static_scratch(carlb_env* env, carlb_action_kind kind, const void* actions,
                                        int32_t n_ticks);
carlb_status carlb_reset(carlb_env* env);
/* Auto-reset of finished sims (src/State/Reset.cuh:82-171 semantics). */
carlb_status carlb_reset_dones(carlb_env* env);

/* ---- state injection (device pointers; indices int64 [k]; mask u8 [n_sim]) ---- */
carlb_status carlb_apply_reset_state(
    carlb_env* env, int32_t n_selected,
    const float* ball_position, const float* ball_velocity, const float* ball_angular_velocity,
    const float* car_position, const float* car_rotation, const float* car_velocity,
    const float* car_angular_velocity, const void* car_demoed, int32_t demoed_is_byte,
    const float* car_boost, const float* car_internal_state,
    const int32_t* blue_score, const int32_t* orange_score, const int32_t* episode_ticks,
    const int64_t* simulation_indices, const uint8_t* reset_mask);
carlb_status carlb_set_ball(carlb_env* env, int32_t n_selected, const float* position,
                            const float* velocity, const float* angular_velocity,
                            const int64_t* simulation_indices);
carlb_status carlb_set_car(carlb_env* env, int32_t n_selected, const float* position,
                           const float* rotation, const float* velocity,
                           const float* angular_velocity, const void* demoed,
                           int32_t demoed_is_byte, const float* boost,
                           const float* internal_state, const int64_t* simulation_indices);
carlb_status carlb_set_match_state(carlb_env* env, int32_t n_selected, const int32_t* blue_score,
                                   const int32_t* orange_score, const int32_t* episode_ticks,
                                   const int64_t* simulation_indices);
carlb_status carlb_reset_boost_pads(carlb_env* env, int32_t n_selected,
                                    const int64_t* simulation_indices);

/* ---- outputs, properties ---------------------------------------------------- */
carlb_status carlb_get_buffer(carlb_env* env, carlb_buffer which, void** data,
                              int64_t shape[3], int32_t* ndim, carlb_dtype* dtype);
carlb_status carlb_set_limit(carlb_env* env, carlb_limit which, int32_t value);
carlb_status carlb_get_limit(const carlb_env* env, carlb_limit which, int32_t* value);
/* n_sim, n_cars, obs_dim, act_dim, state_dim */
carlb_status carlb_dims(const carlb_env* env, int32_t dims[5]);
/* The env's cudaStream_t (non-blocking stream owned by the env). */
void* carlb_stream(const carlb_env* env);
carlb_status carlb_synchronize(carlb_env* env);

/* ---- snapshot / restore (host memory, synchronous) ------------------------- */
/* Words per entity and entity rows for `field` under the env's dimensions. */
carlb_status carlb_field_shape(const carlb_env* env, carlb_field field, int64_t* rows,
                               int32_t* width);
carlb_status carlb_read_field(carlb_env* env, carlb_field field, void* host_out);
carlb_status carlb_write_field(carlb_env* env, carlb_field field, const void* host_in);

/* Per-tick diagnostics (CARLB_F_DIAG_*): when enabled, the last tick of every
 * launch also writes broadphase cells, candidate counts, SAT pair lists and
 * car-car contact counts.  Off by default. */
carlb_status carlb_set_diagnostics(carlb_env* env, int32_t enabled);

/* ---- kernel timing (device time of the last carlb_ticks / carlb_env_step call) ---- */
/* Milliseconds between the start of the first and the end of the last tick
 * kernel of the last call (all stages and sim slices). */
carlb_status carlb_last_tick_ms(const carlb_env* env, float* ms);
/* Staged path only: when enabled, the last tick of every call records CUDA
 * events around each stage kernel of the first sim slice (on that slice's
 * stream).  No counterpart in the reference (profiling aid). */
carlb_status carlb_set_stage_timing(carlb_env* env, int32_t enabled);
/* Durations (ms) of the stage kernels of the last timed tick, in launch order:
 * ball prelude, candidates (flat), ray finish, controls + suspension, contact
 * solve, car-car, ball arena, finish.  Waits for that tick to complete. */
carlb_status carlb_stage_times(carlb_env* env, float* ms, int32_t capacity, int32_t* count);

/* Work-list sizes of the last tick of the last carlb_ticks / carlb_env_step call,
 * summed over the sim slices: [0] cars listed for the contact stage with plane
 * contacts only, [1] cars listed with SAT hits, [2] moving balls listed for the
 * ball stage, [3] sims with a car-car pair in reach.  Waits for the env stream.
 * A measurement aid (the list-driven stages' byte models); no counterpart in
 * the reference. */
carlb_status carlb_stage_work(carlb_env* env, int32_t counts[4]);

/* Action mask of observation rows, on the device: obs is float32 [rows, obs_dim]
 * (device memory, row-major), mask receives uint8 [rows, 18] (1 = logit allowed),
 * enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream).
 * previous_controls says whether the rows end with the 8 previous-control values.
 * Replaces python/carl/gymnasium/action.py:17-37 (CARLActionCodec.mask, a chain of
 * torch ops): all logits allowed except powerslide (ego on ground), boost (ego
 * boost > 0) and jump (on ground, or a flip available with more than PHYS_DT of
 * dodge window left).  CARLB_ERR_VALUE for a null pointer with rows > 0, negative
 * rows, a mask that is not 4-byte aligned, or obs_dim too small for the ego fields. */
carlb_status carlb_action_mask(const float* obs, int64_t rows, int32_t obs_dim, int32_t previous_controls,
                               uint8_t* mask, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CARLB_H */
