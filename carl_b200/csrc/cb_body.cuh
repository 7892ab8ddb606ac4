// Car body kinematics: integration, the solver body, broadphase bounds and the
// suspension hardpoint geometry.
//
// Follows jwmccarthy/CARL include/Physics/Integration.cuh:6-69 (integrateQuat,
// integrateCarState, predictCarPose), include/AABB.cuh:11-34 (car bounds),
// include/Arena/BroadPhaseGrid.cuh:12-27 (grid cell), include/Physics/
// SuspensionUtils.cuh:5-31 and include/Physics/CarArena/SolverBody.cuh:6-78, with
// the same fp32 operation order.
#pragma once

#include "cb_consts.cuh"

namespace cb {

// ---- integration ---------------------------------------------------------------

CB_HD Q4 integrateQuat(Q4 rot, V3 ang)
{
    constexpr float dt = PHYS_DT;
    constexpr float maxMotion = CAR_ANGULAR_MOTION_THRESH;

    const float angSpeedSq = lensq(ang);
    float angSpeed = angSpeedSq > 1e-8f ? sqrtf(angSpeedSq) : 0.f;
    if (angSpeed * dt > maxMotion) angSpeed = maxMotion / dt;

    V3 axis;
    if (angSpeed < 0.001f)
    {
        // Taylor expansion of sin(x/2)/x near zero.
        const float dtSq = dt * dt;
        const float scale = 0.5f * dt - dtSq * dt * 0.020833333333f * angSpeed * angSpeed;
        axis = ang * scale;
    }
    else
    {
        axis = ang * (sinf(0.5f * angSpeed * dt) / angSpeed);
    }

    const Q4 delta = { axis.x, axis.y, axis.z, cosf(0.5f * angSpeed * dt) };
    const Q4 basis = qfromAxes(rotate(rot, axisVec(0)), rotate(rot, axisVec(1)), rotate(rot, axisVec(2)));
    return qnormalized(qmul(delta, basis));
}

CB_HD V3 carOffsetWorld(Q4 rot) { return rotate(rot, V3{ CAR_OFF_X, CAR_OFF_Y, CAR_OFF_Z }); }

// pos += vel dt, rot advanced by ang, hitbox centre rebuilt.
CB_HD void integratePose(V3& pos, V3& cen, Q4& rot, V3 vel, V3 ang)
{
    pos = pos + vel * PHYS_DT;
    rot = integrateQuat(rot, ang);
    cen = pos + carOffsetWorld(rot);
}

// ---- broadphase ------------------------------------------------------------------

CB_HD V3 carHalfExtents() { return V3{ CAR_HALF_X, CAR_HALF_Y, CAR_HALF_Z }; }

CB_HD V3 carAabbMin(V3 cen, Q4 rot)
{
    const V3 rx = rotate(rot, axisVec(0));
    const V3 ry = rotate(rot, axisVec(1));
    const V3 rz = rotate(rot, axisVec(2));
    const V3 half = vabs(rx) * CAR_HALF_X + vabs(ry) * CAR_HALF_Y + vabs(rz) * CAR_HALF_Z;
    return cen - half;
}

CB_HD I3 gridCell(V3 p)
{
    const float gx = fminf(fmaxf((p.x - ARENA_MIN_X) / CELL_X, 0.f), GRID_X - 1.f);
    const float gy = fminf(fmaxf((p.y - ARENA_MIN_Y) / CELL_Y, 0.f), GRID_Y - 1.f);
    const float gz = fminf(fmaxf((p.z - ARENA_MIN_Z) / CELL_Z, 0.f), GRID_Z - 1.f);
    return I3{ (int)gx, (int)gy, (int)gz };
}

CB_HD int flatCell(I3 c) { return c.x + c.y * GRID_W + c.z * (GRID_W * GRID_H); }

// Cell holding the minimum corner of the car's box swept over one tick.
CB_HD int broadphaseCell(V3 pos, V3 vel, V3 ang, V3 cen, Q4 rot)
{
    V3 predPos = pos, predCen;
    Q4 predRot = rot;
    integratePose(predPos, predCen, predRot, vel, ang);
    const V3 swept = vmin(carAabbMin(cen, rot), carAabbMin(predCen, predRot));
    return flatCell(gridCell(swept));
}

// ---- suspension geometry -----------------------------------------------------------

CB_HD V3 suspConnection(int wheel)
{
    const float x = wheel < 2 ? FRONT_SUSP_X : BACK_SUSP_X;
    const float absY = wheel < 2 ? FRONT_SUSP_Y : BACK_SUSP_Y;
    const float y = (wheel & 1) ? -absY : absY;
    return V3{ x, y, 0.f };
}
CB_HD float suspRayLength(int wheel) { return wheel < 2 ? FRONT_SUSP_RAY_LEN : BACK_SUSP_RAY_LEN; }
CB_HD float suspRadius(int wheel) { return wheel < 2 ? FRONT_WHEEL_RADIUS : BACK_WHEEL_RADIUS; }
CB_HD float suspRestLength(int wheel) { return wheel < 2 ? FRONT_SUSPENSION_REST : BACK_SUSPENSION_REST; }
CB_HD float suspForceScale(int wheel) { return wheel < 2 ? SUSP_FORCE_SCALE_FRONT : SUSP_FORCE_SCALE_BACK; }

// ---- solver body ---------------------------------------------------------------------

struct Body
{
    V3 pos, vel, ang, cen;
    Q4 rot;
    V3 extVel, extAng, deltaVel, deltaAng, pushVel, turnVel;
};

CB_HD Body makeBody(V3 pos, V3 vel, V3 ang, V3 cen, Q4 rot)
{
    Body b;
    b.pos = pos;
    b.vel = vel;
    b.ang = ang;
    b.cen = cen;
    b.rot = rot;
    b.extVel = V3{ 0.f, 0.f, GRAVITY_Z } * PHYS_DT;
    b.extAng = v3zero();
    b.deltaVel = v3zero();
    b.deltaAng = v3zero();
    b.pushVel = v3zero();
    b.turnVel = v3zero();
    return b;
}

CB_HD V3 carInvInertia() { return V3{ CAR_INV_INERTIA_X, CAR_INV_INERTIA_Y, CAR_INV_INERTIA_Z }; }

// World-space inverse inertia applied to a world vector.
CB_HD V3 invInertiaWorld(Q4 rot, V3 value)
{
    const V3 local = unrotate(rot, value);
    return rotate(rot, local * carInvInertia());
}

CB_D void clampCarVelocity(V3& vel, V3& ang)
{
    const float v2 = lensq(vel);
    if (v2 > CAR_MAX_SPEED * CAR_MAX_SPEED) vel = vel * (CAR_MAX_SPEED * rsqrtf(v2));
    const float a2 = lensq(ang);
    if (a2 > CAR_MAX_ANG_SPEED * CAR_MAX_ANG_SPEED) ang = ang * (CAR_MAX_ANG_SPEED * rsqrtf(a2));
}

// ---- integer hash used for kickoff permutations and demo respawns ----------------------

CB_HD uint32_t hash32(uint32_t v)
{
    v = ((v >> 16) ^ v) * 0x45d9f3bu;
    v = ((v >> 16) ^ v) * 0x45d9f3bu;
    return (v >> 16) ^ v;
}
CB_HD int randomIndex(uint32_t seed, int count) { return (int)(hash32(seed) % (uint32_t)count); }

}  // namespace cb
