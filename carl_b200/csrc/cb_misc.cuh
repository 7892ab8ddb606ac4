// End-of-tick bookkeeping, boost pads, kickoff / auto-reset and the
// observation, canonical-state and reward packing.
//
// Follows jwmccarthy/CARL include/Physics/FinishTick.cuh:5-141,
// include/Physics/BoostPads.cuh:58-106, include/State/Reset.cuh:8-171,
// include/Physics/Observations.cuh:7-397 and src/EnvIO.cu:116-357, with the same
// fp32 operation order.  Game tables (pads, spawns) are the reference's values;
// the kickoff permutation table and the mirrored pad order are derived at load
// time (see tables.cpp).
#pragma once

#include "cb_ball.cuh"
#include "cb_tables.hpp"

namespace cb {

#if defined(__CUDACC__)
// One copy per translation unit (no relocatable device code); every .cu file
// that uses it uploads the same host-built tables at env creation.
static __constant__ Tables c_tables;
#endif

// ---- finish tick ------------------------------------------------------------------------

template <class T>
CB_D void finishBall(const T& sims, int s)
{
    const V3 impulse = sims.v(S_BIMP, s);
    V3 vel = sims.v(S_BVEL, s) + impulse;
    V3 ang = sims.v(S_BANG, s);
    float sq = lensq(vel);
    if (sq > BALL_MAX_SPEED * BALL_MAX_SPEED) vel = vel * (BALL_MAX_SPEED * rsqrtf(sq));
    sq = lensq(ang);
    if (sq > BALL_MAX_ANG_SPEED * BALL_MAX_ANG_SPEED) ang = ang * (BALL_MAX_ANG_SPEED * rsqrtf(sq));
    sims.setv(S_BVEL, s, vel);
    sims.setv(S_BANG, s, ang);
    sims.setv(S_BIMP, s, v3zero());
}

// Respawn of a demolished car at its selected spot; `orange` mirrors y and yaw.
template <class S>
CB_D void respawnCar(const S& c, int i, bool orange, const Tables& T)
{
    const int spawn = c.n(C_INT + I_RESPAWN_IDX, i);
    const float y = orange ? -T.respY[spawn] : T.respY[spawn];
    const float yaw = orange ? T.respYaw[spawn] + PI : T.respYaw[spawn];
    const Q4 rot = qyaw(yaw);
    const V3 pos = { T.respX[spawn], y, CAR_RESPAWN_Z };
    c.setv(C_POS, i, pos);
    c.setv(C_CEN, i, pos + carOffsetWorld(rot));
    c.setq(C_ROT, i, rot);
    c.setv(C_VEL, i, v3zero());
    c.setv(C_ANG, i, v3zero());
    c.setv(C_IMP, i, v3zero());
    c.n(C_DEMOED, i) = 0;
    c.f(C_DEMO_TIMER, i) = 0.f;
    c.n(C_CONTACT_IDX, i) = -1;
    c.f(C_CONTACT_CD, i) = 0.f;
    c.n(C_BALL_HIT_TICK, i) = -1;
    c.n(C_BALL_CONTACT_TICK, i) = -1;
    for (int k = 0; k < NIW; k++) c.n(C_INT + k, i) = 0;
    c.n(C_INT + I_ON_GROUND, i) = 1;
    c.f(C_INT + I_BOOST, i) = BOOST_SPAWN_AMOUNT;
}

// Impulse cache, demo timer / respawn and bump cooldown of one car.  Returns
// true when the car respawned (its wheel contacts read as cleared).
template <class S>
CB_D bool finishCar(const S& c, int i, float steer, bool orange, const Tables& T)
{
    if (c.n(C_DEMOED, i))
    {
        float timer = c.f(C_DEMO_TIMER, i);
        if (timer <= DEMO_RESPAWN_TIME)
        {
            const int dir = steer < -DEMO_RESPAWN_INPUT_DEADZONE ? -1 : (steer > DEMO_RESPAWN_INPUT_DEADZONE ? 1 : 0);
            int& idx = c.n(C_INT + I_RESPAWN_IDX, i);
            int& last = c.n(C_INT + I_LAST_RESPAWN_DIR, i);
            if (dir != 0 && dir != last)
            {
                if (dir < 0 && idx > 0) idx--;
                else if (dir > 0 && idx < 3) idx++;
            }
            last = dir;
        }
        timer = fmaxf(timer - PHYS_DT, 0.f);
        c.f(C_DEMO_TIMER, i) = timer;
        if (timer <= 0.f)
        {
            respawnCar(c, i, orange, T);
            return true;
        }
        return false;
    }
    const V3 impulse = c.v(C_IMP, i);
    if (lensq(impulse) > 1e-12f)
    {
        V3 vel = c.v(C_VEL, i) + impulse;
        const float sq = lensq(vel);
        if (sq > CAR_MAX_SPEED * CAR_MAX_SPEED) vel = vel * (CAR_MAX_SPEED * rsqrtf(sq));
        c.setv(C_VEL, i, vel);
        c.setv(C_IMP, i, v3zero());
    }
    float cd = c.f(C_CONTACT_CD, i);
    if (cd <= 0.f) return false;
    cd = fmaxf(cd - PHYS_DT, 0.f);
    c.f(C_CONTACT_CD, i) = cd;
    return false;
}

// ---- boost pads -------------------------------------------------------------------------------

// Pad `pad` of the sim whose cars start at `carBase`; the last overlapping
// non-demolished car (in car order) takes it.
template <class S, class U>
CB_D void boostPad(const S& c, int carBase, int nCars, const U& sims, int s, int pad, const Tables& T)
{
    float cd = sims.f(S_PADS + pad, s);
    if (cd > 0.f)
    {
        cd = fmaxf(cd - PHYS_DT, 0.f);
        sims.f(S_PADS + pad, s) = cd;
    }
    if (cd > 0.f) return;
    const bool big = T.padBig[pad] != 0;
    const float radius = big ? BIG_PAD_RADIUS : SMALL_PAD_RADIUS;
    int locked = -1;
    for (int k = 0; k < nCars; k++)
    {
        const int i = carBase + k;
        if (c.n(C_DEMOED, i)) continue;
        const V3 p = c.v(C_POS, i);
        const float dx = p.x - T.padX[pad];
        const float dy = p.y - T.padY[pad];
        const float distSq = dx * dx + dy * dy;
        if (distSq < radius * radius && fabsf(p.z - T.padZ[pad]) < BOOST_PAD_HEIGHT) locked = i;
    }
    if (locked < 0) return;
    const float boost = c.f(C_INT + I_BOOST, locked);
    if (boost >= BOOST_MAX) return;
    c.f(C_INT + I_BOOST, locked) = fminf(boost + (big ? BIG_PAD_AMOUNT : SMALL_PAD_AMOUNT), BOOST_MAX);
    sims.f(S_PADS + pad, s) = big ? BIG_PAD_COOLDOWN : SMALL_PAD_COOLDOWN;
}

}  // namespace cb
