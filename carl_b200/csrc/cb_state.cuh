// State layout shared by the tick kernel (shared-memory tiles) and the
// state-injection / packing kernels (global memory).
//
// All persistent state is struct-of-arrays of 32-bit words, "word-major":
// word k of car i lives at base[k * stride + i].  The same accessor serves a
// shared-memory tile (stride = cars in the tile) and the HBM arrays (stride =
// padded car count), so a tile loads and stores with contiguous, coalesced
// 16-byte copies per word.
#pragma once

#include "cb_controls.cuh"

namespace cb {

// ---- persistent per-car words -------------------------------------------------------
enum CarWord : int {
    C_POS = 0,            // 3
    C_VEL = 3,            // 3
    C_ANG = 6,            // 3
    C_ROT = 9,            // 4 (x y z w)
    C_CEN = 13,           // 3
    C_IMP = 16,           // 3
    C_DEMOED = 19,
    C_DEMO_TIMER = 20,
    C_CONTACT_IDX = 21,   // env-global car index of the last bump victim
    C_CONTACT_CD = 22,
    C_BALL_HIT_TICK = 23,
    C_BALL_CONTACT_TICK = 24,
    C_INT = 25,           // 24 words, carlb.h CARLB_INT_* order
    C_SUSP = 49,          // 15 words, carlb.h CARLB_SUSP_* order
    C_LAT = 64,           // 4
    C_LON = 68,           // 4
    C_MAN_COUNT = 72,
    C_MAN_N0 = 73,        // 3
    NCW = 76
};

// Internal-state word offsets (relative to C_INT).
enum IntWord : int {
    I_ON_GROUND = 0, I_AIR_TIME, I_AIR_TIME_SINCE_JUMP, I_HANDBRAKE, I_HAS_JUMPED, I_IS_JUMPING,
    I_JUMP_TIME, I_LAST_JUMP, I_HAS_DOUBLE_JUMPED, I_HAS_FLIPPED, I_IS_FLIPPING, I_FLIP_TIME,
    I_IS_AUTO_FLIPPING, I_AUTO_FLIP_TIMER, I_AUTO_FLIP_SCALE, I_FLIP_TORQUE, I_RESPAWN_IDX = 18,
    I_LAST_RESPAWN_DIR, I_IS_BOOSTING, I_BOOST, I_BOOSTING_TIME, I_TIME_SINCE_BOOSTED, NIW
};

// Staged suspension word offsets (relative to C_SUSP).
enum SuspWord : int {
    SU_BRAKE = 0, SU_BRAKE_PREV, SU_THROTTLE, SU_RAW_THROTTLE, SU_HANDBRAKE, SU_STEER, SU_STEER_PREV,
    SU_ENGINE, SU_ENGINE_PREV, SU_JUMP_IMP, SU_ANG_IMP = 12, NSUW = 15
};

// ---- per-car outputs (rewritten every tick, never read by the next tick) ----
enum CarOutWord : int {
    O_RAY_DIST = 0,       // 4
    O_RAY_NORMAL = 4,     // 12
    O_WHEEL_SRC = 16,     // 4
    O_WHEEL_CON = 20,     // 4
    O_CONTROLS = 24,      // 8: throttle steer yaw pitch roll (f32) jump boost slide (i32)
    O_ARENA_CONTACT_TICK = 32,
    NOW = 33
};

// ---- persistent per-sim words -----------------------------------------------------------
enum SimWord : int {
    S_BPOS = 0, S_BVEL = 3, S_BANG = 6, S_BIMP = 9,
    S_IPOS = 12, S_IVEL = 15, S_EPOS = 18, S_EVEL = 21,  // Bullet-unit integration cache
    S_IVALID = 24,
    S_EP_TICKS = 25,
    S_LAST_TOUCH = 26,
    S_GOALS = 27,         // blue, orange, lastScorer, tick, overtime
    S_PADS = 32,          // 34 cooldowns
    NSW = 66
};
enum GoalWord : int { G_BLUE = 0, G_ORANGE, G_LAST_SCORER, G_TICK, G_OVERTIME };

// Per-sim outputs.
enum SimOutWord : int { SO_BALL_ARENA_CONTACT_TICK = 0, NSOW = 1 };

// Per-tick diagnostics (written by the last tick when enabled).
constexpr int DIAG_CAR_WORDS = 2 + 1 + MAX_CAR_TRI_PAIRS;  // cell, numTris, [hits, tris...]
constexpr int DIAG_SIM_WORDS = 28;                          // car-car pair contact counts (<= 8 cars)

// ---- accessor -------------------------------------------------------------------------------

template <class Idx>
struct Soa
{
    float* base;
    Idx stride;

    CB_HD float& f(int w, Idx i) const { return base[(Idx)w * stride + i]; }
    CB_HD int& n(int w, Idx i) const { return reinterpret_cast<int*>(base)[(Idx)w * stride + i]; }
    CB_HD V3 v(int w, Idx i) const { return V3{ f(w, i), f(w + 1, i), f(w + 2, i) }; }
    CB_HD void setv(int w, Idx i, V3 a) const
    {
        f(w, i) = a.x;
        f(w + 1, i) = a.y;
        f(w + 2, i) = a.z;
    }
    CB_HD Q4 q(int w, Idx i) const { return Q4{ f(w, i), f(w + 1, i), f(w + 2, i), f(w + 3, i) }; }
    CB_HD void setq(int w, Idx i, Q4 a) const
    {
        f(w, i) = a.x;
        f(w + 1, i) = a.y;
        f(w + 2, i) = a.z;
        f(w + 3, i) = a.w;
    }
};

using SmemSoa = Soa<int>;
using GlobSoa = Soa<long long>;

// ---- register images of per-car groups -------------------------------------------------------

template <class S, class Idx>
CB_HD Internal loadInternal(const S& c, Idx i)
{
    Internal s;
    const int b = C_INT;
    s.isOnGround = c.n(b + I_ON_GROUND, i);
    s.airTime = c.f(b + I_AIR_TIME, i);
    s.airTimeSinceJump = c.f(b + I_AIR_TIME_SINCE_JUMP, i);
    s.handbrakeVal = c.f(b + I_HANDBRAKE, i);
    s.hasJumped = c.n(b + I_HAS_JUMPED, i);
    s.isJumping = c.n(b + I_IS_JUMPING, i);
    s.jumpTime = c.f(b + I_JUMP_TIME, i);
    s.lastJump = c.n(b + I_LAST_JUMP, i);
    s.hasDoubleJumped = c.n(b + I_HAS_DOUBLE_JUMPED, i);
    s.hasFlipped = c.n(b + I_HAS_FLIPPED, i);
    s.isFlipping = c.n(b + I_IS_FLIPPING, i);
    s.flipTime = c.f(b + I_FLIP_TIME, i);
    s.isAutoFlipping = c.n(b + I_IS_AUTO_FLIPPING, i);
    s.autoFlipTimer = c.f(b + I_AUTO_FLIP_TIMER, i);
    s.autoFlipTorqueScale = c.f(b + I_AUTO_FLIP_SCALE, i);
    s.flipRelTorque = c.v(b + I_FLIP_TORQUE, i);
    s.respawnIdx = c.n(b + I_RESPAWN_IDX, i);
    s.lastRespawnDir = c.n(b + I_LAST_RESPAWN_DIR, i);
    s.isBoosting = c.n(b + I_IS_BOOSTING, i);
    s.boost = c.f(b + I_BOOST, i);
    s.boostingTime = c.f(b + I_BOOSTING_TIME, i);
    s.timeSinceBoosted = c.f(b + I_TIME_SINCE_BOOSTED, i);
    return s;
}

template <class S, class Idx>
CB_HD void storeInternal(const S& c, Idx i, const Internal& s)
{
    const int b = C_INT;
    c.n(b + I_ON_GROUND, i) = s.isOnGround;
    c.f(b + I_AIR_TIME, i) = s.airTime;
    c.f(b + I_AIR_TIME_SINCE_JUMP, i) = s.airTimeSinceJump;
    c.f(b + I_HANDBRAKE, i) = s.handbrakeVal;
    c.n(b + I_HAS_JUMPED, i) = s.hasJumped;
    c.n(b + I_IS_JUMPING, i) = s.isJumping;
    c.f(b + I_JUMP_TIME, i) = s.jumpTime;
    c.n(b + I_LAST_JUMP, i) = s.lastJump;
    c.n(b + I_HAS_DOUBLE_JUMPED, i) = s.hasDoubleJumped;
    c.n(b + I_HAS_FLIPPED, i) = s.hasFlipped;
    c.n(b + I_IS_FLIPPING, i) = s.isFlipping;
    c.f(b + I_FLIP_TIME, i) = s.flipTime;
    c.n(b + I_IS_AUTO_FLIPPING, i) = s.isAutoFlipping;
    c.f(b + I_AUTO_FLIP_TIMER, i) = s.autoFlipTimer;
    c.f(b + I_AUTO_FLIP_SCALE, i) = s.autoFlipTorqueScale;
    c.setv(b + I_FLIP_TORQUE, i, s.flipRelTorque);
    c.n(b + I_RESPAWN_IDX, i) = s.respawnIdx;
    c.n(b + I_LAST_RESPAWN_DIR, i) = s.lastRespawnDir;
    c.n(b + I_IS_BOOSTING, i) = s.isBoosting;
    c.f(b + I_BOOST, i) = s.boost;
    c.f(b + I_BOOSTING_TIME, i) = s.boostingTime;
    c.f(b + I_TIME_SINCE_BOOSTED, i) = s.timeSinceBoosted;
}

template <class S, class Idx>
CB_HD Susp loadSusp(const S& c, Idx i)
{
    const int b = C_SUSP;
    Susp s;
    s.brake = c.f(b + SU_BRAKE, i);
    s.brakePrev = c.f(b + SU_BRAKE_PREV, i);
    s.throttle = c.f(b + SU_THROTTLE, i);
    s.rawThrottle = c.f(b + SU_RAW_THROTTLE, i);
    s.handbrake = c.f(b + SU_HANDBRAKE, i);
    s.steer = c.f(b + SU_STEER, i);
    s.steerPrev = c.f(b + SU_STEER_PREV, i);
    s.engine = c.f(b + SU_ENGINE, i);
    s.enginePrev = c.f(b + SU_ENGINE_PREV, i);
    s.jumpImp = c.v(b + SU_JUMP_IMP, i);
    s.angImp = c.v(b + SU_ANG_IMP, i);
    return s;
}

template <class S, class Idx>
CB_HD void storeSusp(const S& c, Idx i, const Susp& s)
{
    const int b = C_SUSP;
    c.f(b + SU_BRAKE, i) = s.brake;
    c.f(b + SU_BRAKE_PREV, i) = s.brakePrev;
    c.f(b + SU_THROTTLE, i) = s.throttle;
    c.f(b + SU_RAW_THROTTLE, i) = s.rawThrottle;
    c.f(b + SU_HANDBRAKE, i) = s.handbrake;
    c.f(b + SU_STEER, i) = s.steer;
    c.f(b + SU_STEER_PREV, i) = s.steerPrev;
    c.f(b + SU_ENGINE, i) = s.engine;
    c.f(b + SU_ENGINE_PREV, i) = s.enginePrev;
    c.setv(b + SU_JUMP_IMP, i, s.jumpImp);
    c.setv(b + SU_ANG_IMP, i, s.angImp);
}

}  // namespace cb
