/*
 * Field map between the reference's state structs and the snapshot layout of
 * include/carlb.h (carlb_field).  Shared by the CPU oracle driver
 * (ref_cpu_driver.cpp) and the GPU reference harness (ref_gpu_harness.cu).
 *
 * The reference keeps every field in its own DeviceArray
 * (include/State/GameState.cuh:9-232, include/State/Workspace.cuh:8-234); Vec3 is a
 * 16-byte padded struct (include/Cuda/Math.cuh:36-38) and CarInternalState a
 * 112-byte record.  A snapshot field is a dense [rows, width] array of 32-bit
 * words; each part below copies some words of each row from one array.
 * TEST INFRASTRUCTURE.
 */
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <functional>
#include <vector>

#include "../include/carlb.h"

struct RefFieldPart
{
    const void* base = nullptr;   // array base (host or device memory)
    int64_t rowBytes = 0;         // bytes of one entity record in that array
    int64_t arrayBytes = 0;       // bytes of the whole array
    std::vector<int> offsets;     // byte offset of each copied word inside a record
    std::vector<int> byteWords;   // 1 where the source word is a 1-byte bool
    int dstWord = 0;              // first destination word in the snapshot row
};

struct RefField
{
    int64_t rows = 0;
    int width = 0;
    bool readOnly = false;
    std::vector<RefFieldPart> parts;
};

template <class T>
static RefFieldPart refPart(const T* base, int64_t count, int64_t entities,
                            std::vector<int> offsets, int dstWord = 0)
{
    RefFieldPart p;
    p.base = base;
    p.rowBytes = (int64_t)sizeof(T) * (count / entities);
    p.arrayBytes = (int64_t)sizeof(T) * count;
    p.offsets = std::move(offsets);
    p.byteWords.assign(p.offsets.size(), 0);
    p.dstWord = dstWord;
    return p;
}

static std::vector<int> vecWords(int records, int recordBytes)
{
    std::vector<int> o;
    for (int r = 0; r < records; r++)
        for (int c = 0; c < 3; c++) o.push_back(r * recordBytes + 4 * c);
    return o;
}

static std::vector<int> scalarWords(int records)
{
    std::vector<int> o;
    for (int r = 0; r < records; r++) o.push_back(4 * r);
    return o;
}

/* Builds the map from a host-side copy of GameState / Workspace whose array
 * pointers address wherever the arrays live.  `tickCountAddr` is the address
 * (host or device) of GameState::tickCount. */
static RefField refField(const GameState& s, const Workspace& w, int field, const void* tickCountAddr)
{
    const int64_t n = s.nTotalCars;
    const int64_t ns = s.nSim;
    RefField f;
    auto car = [&](int width) { f.rows = n; f.width = width; };
    auto sim = [&](int width) { f.rows = ns; f.width = width; };

    switch (field)
    {
    case CARLB_F_CAR_POS: car(3); f.parts.push_back(refPart(s.cars.pos.ptr, n, n, vecWords(1, 16))); break;
    case CARLB_F_CAR_VEL: car(3); f.parts.push_back(refPart(s.cars.vel.ptr, n, n, vecWords(1, 16))); break;
    case CARLB_F_CAR_ANG: car(3); f.parts.push_back(refPart(s.cars.ang.ptr, n, n, vecWords(1, 16))); break;
    case CARLB_F_CAR_ROT: car(4); f.parts.push_back(refPart(s.cars.rot.ptr, n, n, { 0, 4, 8, 12 })); break;
    case CARLB_F_CAR_CEN: car(3); f.parts.push_back(refPart(s.cars.cen.ptr, n, n, vecWords(1, 16))); break;
    case CARLB_F_CAR_IMP: car(3); f.parts.push_back(refPart(s.cars.imp.ptr, n, n, vecWords(1, 16))); break;
    case CARLB_F_CAR_IS_DEMOED: car(1); f.parts.push_back(refPart(s.cars.isDemoed.ptr, n, n, { 0 })); break;
    case CARLB_F_CAR_DEMO_TIMER: car(1); f.parts.push_back(refPart(s.cars.demoRespawnTimer.ptr, n, n, { 0 })); break;
    case CARLB_F_CAR_CONTACT_IDX: car(1); f.parts.push_back(refPart(s.cars.carContactIdx.ptr, n, n, { 0 })); break;
    case CARLB_F_CAR_CONTACT_COOLDOWN: car(1); f.parts.push_back(refPart(s.cars.carContactCooldown.ptr, n, n, { 0 })); break;
    case CARLB_F_CAR_BALL_HIT_TICK: car(1); f.parts.push_back(refPart(s.cars.ballHitTick.ptr, n, n, { 0 })); break;
    case CARLB_F_CAR_BALL_CONTACT_TICK: car(1); f.parts.push_back(refPart(s.cars.ballContactTick.ptr, n, n, { 0 })); break;
    case CARLB_F_CAR_WHEEL_SOURCE: car(4); f.parts.push_back(refPart(s.cars.wheelSource.ptr, n * 4, n, scalarWords(4))); break;
    case CARLB_F_CAR_WHEEL_CONTACT: car(4); f.parts.push_back(refPart(s.cars.wheelContact.ptr, n * 4, n, scalarWords(4))); break;
    case CARLB_F_CAR_ARENA_CONTACT_TICK: car(1); f.parts.push_back(refPart(s.cars.arenaContactTick.ptr, n, n, { 0 })); break;
    case CARLB_F_CAR_CONTROLS:
        car(8);
        f.parts.push_back(refPart(s.cars.controls.ptr, n, n, {
            (int)offsetof(CarControls, throttle), (int)offsetof(CarControls, steer),
            (int)offsetof(CarControls, yaw), (int)offsetof(CarControls, pitch),
            (int)offsetof(CarControls, roll), (int)offsetof(CarControls, jump),
            (int)offsetof(CarControls, boost), (int)offsetof(CarControls, slide) }));
        break;
    case CARLB_F_CAR_INTERNAL:
    {
        car(CARLB_INT_WORDS);
        using I = CarInternalState;
        const int vt = (int)offsetof(I, flipRelTorque);
        f.parts.push_back(refPart(s.cars.internal.ptr, n, n, {
            (int)offsetof(I, isOnGround), (int)offsetof(I, airTime),
            (int)offsetof(I, airTimeSinceJump), (int)offsetof(I, handbrakeVal),
            (int)offsetof(I, hasJumped), (int)offsetof(I, isJumping),
            (int)offsetof(I, jumpTime), (int)offsetof(I, lastJump),
            (int)offsetof(I, hasDoubleJumped), (int)offsetof(I, hasFlipped),
            (int)offsetof(I, isFlipping), (int)offsetof(I, flipTime),
            (int)offsetof(I, isAutoFlipping), (int)offsetof(I, autoFlipTimer),
            (int)offsetof(I, autoFlipTorqueScale), vt, vt + 4, vt + 8,
            (int)offsetof(I, respawnIdx), (int)offsetof(I, lastRespawnDir),
            (int)offsetof(I, isBoosting), (int)offsetof(I, boost),
            (int)offsetof(I, boostingTime), (int)offsetof(I, timeSinceBoosted) }));
        break;
    }
    case CARLB_F_SUSP_SCALARS:
    {
        car(CARLB_SUSP_WORDS);
        const CarSuspension& p = w.susp;
        f.parts.push_back(refPart(p.brakeFactor.ptr, n, n, { 0 }, CARLB_SUSP_BRAKE));
        f.parts.push_back(refPart(p.brakeFactorPrev.ptr, n, n, { 0 }, CARLB_SUSP_BRAKE_PREV));
        f.parts.push_back(refPart(p.throttleVal.ptr, n, n, { 0 }, CARLB_SUSP_THROTTLE));
        f.parts.push_back(refPart(p.rawThrottle.ptr, n, n, { 0 }, CARLB_SUSP_RAW_THROTTLE));
        f.parts.push_back(refPart(p.handbrakeVal.ptr, n, n, { 0 }, CARLB_SUSP_HANDBRAKE));
        f.parts.push_back(refPart(p.steerAngle.ptr, n, n, { 0 }, CARLB_SUSP_STEER));
        f.parts.push_back(refPart(p.steerAnglePrev.ptr, n, n, { 0 }, CARLB_SUSP_STEER_PREV));
        f.parts.push_back(refPart(p.engineDrive.ptr, n, n, { 0 }, CARLB_SUSP_ENGINE));
        f.parts.push_back(refPart(p.engineDrivePrev.ptr, n, n, { 0 }, CARLB_SUSP_ENGINE_PREV));
        f.parts.push_back(refPart(p.jumpImpulse.ptr, n, n, vecWords(1, 16), CARLB_SUSP_JUMP_IMP_X));
        f.parts.push_back(refPart(p.angularImpulse.ptr, n, n, vecWords(1, 16), CARLB_SUSP_ANG_IMP_X));
        break;
    }
    case CARLB_F_SUSP_RAY_DIST: car(4); f.parts.push_back(refPart(w.susp.rayDist.ptr, n * 4, n, scalarWords(4))); break;
    case CARLB_F_SUSP_RAY_NORMAL: car(12); f.parts.push_back(refPart(w.susp.rayNormal.ptr, n * 4, n, vecWords(4, 16))); break;
    case CARLB_F_SUSP_LAT_FRICTION: car(4); f.parts.push_back(refPart(w.susp.latFrictionPrev.ptr, n * 4, n, scalarWords(4))); break;
    case CARLB_F_SUSP_LON_FRICTION: car(4); f.parts.push_back(refPart(w.susp.lonFrictionPrev.ptr, n * 4, n, scalarWords(4))); break;
    case CARLB_F_MAN_COUNT: car(1); f.parts.push_back(refPart(w.ctMan.count.ptr, n, n, { 0 })); break;
    case CARLB_F_MAN_NORMAL0:
        car(3);
        f.parts.push_back(refPart(w.ctMan.worldNormal.ptr, n * MAX_CAR_MANIFOLD_POINTS, n, vecWords(1, 16)));
        break;
    case CARLB_F_BALL_POS: sim(3); f.parts.push_back(refPart(s.ball.pos.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_VEL: sim(3); f.parts.push_back(refPart(s.ball.vel.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_ANG: sim(3); f.parts.push_back(refPart(s.ball.ang.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_IMP: sim(3); f.parts.push_back(refPart(s.ball.imp.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_INT_POS: sim(3); f.parts.push_back(refPart(s.ball.integrationPos.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_INT_VEL: sim(3); f.parts.push_back(refPart(s.ball.integrationVel.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_EXP_POS: sim(3); f.parts.push_back(refPart(s.ball.exportedPos.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_EXP_VEL: sim(3); f.parts.push_back(refPart(s.ball.exportedVel.ptr, ns, ns, vecWords(1, 16))); break;
    case CARLB_F_BALL_INT_VALID: sim(1); f.parts.push_back(refPart(s.ball.integrationValid.ptr, ns, ns, { 0 })); break;
    case CARLB_F_EPISODE_TICKS: sim(1); f.parts.push_back(refPart(s.episodeTicks.ptr, ns, ns, { 0 })); break;
    case CARLB_F_LAST_TOUCH_TICKS: sim(1); f.parts.push_back(refPart(s.lastBallTouchTicks.ptr, ns, ns, { 0 })); break;
    case CARLB_F_BALL_ARENA_CONTACT_TICK: sim(1); f.parts.push_back(refPart(s.ballArenaContactTick.ptr, ns, ns, { 0 })); break;
    case CARLB_F_GOALS:
    {
        sim(5);
        RefFieldPart p = refPart(s.goals.ptr, ns, ns, {
            (int)offsetof(GoalState, blueScore), (int)offsetof(GoalState, orangeScore),
            (int)offsetof(GoalState, lastScorer), (int)offsetof(GoalState, tick),
            (int)offsetof(GoalState, overtime) });
        p.byteWords[4] = 1;
        f.parts.push_back(p);
        break;
    }
    case CARLB_F_PAD_COOLDOWNS:
        sim(NUM_BOOST_PADS);
        f.parts.push_back(refPart(s.boostPadCooldowns.ptr, ns * NUM_BOOST_PADS, ns, scalarWords(NUM_BOOST_PADS)));
        break;
    case CARLB_F_TICK_COUNT:
    {
        f.rows = 1; f.width = 1;
        RefFieldPart p;
        p.base = tickCountAddr; p.rowBytes = 4; p.arrayBytes = 4; p.offsets = { 0 }; p.byteWords = { 0 };
        f.parts.push_back(p);
        break;
    }
    case CARLB_F_DIAG_CELL_IDX: car(1); f.readOnly = true; f.parts.push_back(refPart(w.bp.cellIdx.ptr, n, n, { 0 })); break;
    case CARLB_F_DIAG_NUM_TRIS: car(1); f.readOnly = true; f.parts.push_back(refPart(w.bp.numTris.ptr, n, n, { 0 })); break;
    case CARLB_F_DIAG_SAT_PAIRS:
        /* assembled by the drivers (count from ctHit, ids from ctNrw) */
        car(1 + MAX_CAR_TRI_PAIRS); f.readOnly = true;
        break;
    case CARLB_F_DIAG_CC_COUNT:
    {
        const int pairs = w.ccMan.maxPairsPerSim;
        sim(pairs > 0 ? pairs : 1); f.readOnly = true;
        if (pairs > 0) f.parts.push_back(refPart(w.ccMan.count.ptr, ns * pairs, ns, scalarWords(pairs)));
        break;
    }
    default:
        f.rows = -1;
        break;
    }
    return f;
}

/* Copies a field out of (read) or into (write) the arrays.  `fetch(dst, src,
 * bytes)` copies from the array memory to host, `store(dst, src, bytes)` from
 * host to the array memory. */
using RefCopy = std::function<void(void*, const void*, size_t)>;

static void refReadField(const RefField& f, uint32_t* out, const RefCopy& fetch)
{
    std::vector<unsigned char> tmp;
    for (const RefFieldPart& p : f.parts)
    {
        tmp.resize((size_t)p.arrayBytes);
        fetch(tmp.data(), p.base, (size_t)p.arrayBytes);
        for (int64_t r = 0; r < f.rows; r++)
        {
            const unsigned char* rec = tmp.data() + r * p.rowBytes;
            for (size_t k = 0; k < p.offsets.size(); k++)
            {
                uint32_t word = 0;
                if (p.byteWords[k]) word = rec[p.offsets[k]] ? 1u : 0u;
                else std::memcpy(&word, rec + p.offsets[k], 4);
                out[r * f.width + p.dstWord + (int64_t)k] = word;
            }
        }
    }
}

static void refWriteField(const RefField& f, const uint32_t* in, const RefCopy& fetch, const RefCopy& store)
{
    std::vector<unsigned char> tmp;
    for (const RefFieldPart& p : f.parts)
    {
        tmp.resize((size_t)p.arrayBytes);
        fetch(tmp.data(), p.base, (size_t)p.arrayBytes);
        for (int64_t r = 0; r < f.rows; r++)
        {
            unsigned char* rec = tmp.data() + r * p.rowBytes;
            for (size_t k = 0; k < p.offsets.size(); k++)
            {
                const uint32_t word = in[r * f.width + p.dstWord + (int64_t)k];
                if (p.byteWords[k]) rec[p.offsets[k]] = word ? 1 : 0;
                else std::memcpy(rec + p.offsets[k], &word, 4);
            }
        }
        store(const_cast<void*>(p.base), tmp.data(), (size_t)p.arrayBytes);
    }
}
