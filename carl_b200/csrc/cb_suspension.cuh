// Raycast-vehicle suspension: spring/damper impulse with Bullet-style wheel
// pushback, lateral slip and rolling friction with one-tick-lagged friction
// coefficients, sticky force and autoroll.
//
// Follows jwmccarthy/CARL include/Physics/CarSuspension.cuh:8-339 with the same
// fp32 operation order.
#pragma once

#include "cb_controls.cuh"

namespace cb {

CB_D float nonStickyFriction(float normZ)
{
    if (normZ <= 0.f) return 0.1f;
    if (normZ >= 1.f) return 1.f;
    if (normZ < 0.7075f) return 0.1f + (normZ / 0.7075f) * 0.4f;
    return 0.5f + ((normZ - 0.7075f) / (1.f - 0.7075f)) * 0.5f;
}

struct SuspFrame
{
    V3 cenOffset, forward, right, up, vel, ang, angCrossUp;
    float brakeTorque, pushbackDt;
};

// One wheel's contribution; returns whether the wheel touches.
CB_D bool suspWheel(const Body& body, const SuspFrame& f, int wheel, float dist, V3 normal,
                    float steerPrev, float handbrake, float throttle, float enginePrev,
                    float& latPrev, float& lonPrev, V3& directVel, V3& directAng, V3& deltaVel,
                    bool unlaggedLateral)
{
    directVel = v3zero();
    directAng = v3zero();
    deltaVel = v3zero();
    if (dist > suspRayLength(wheel)) return false;

    const float radius = suspRadius(wheel);
    const float restLen = suspRestLength(wheel);
    const float suspLen = fminf(fmaxf(dist - radius, restLen - MAX_SUSPENSION_TRAVEL),
                                restLen + MAX_SUSPENSION_TRAVEL);

    const V3 hardPointRel = f.cenOffset + rotate(body.rot, suspConnection(wheel));
    const V3 fullRelPos = hardPointRel - f.up * dist;
    const V3 pointVel = f.vel + cross(f.ang, fullRelPos);
    const float projVel = dot(normal, pointVel);
    const float denom = dot(normal, f.up);
    const float clipped = denom > 0.1f ? 1.f / denom : 10.f;
    const float relVel = projVel * clipped;
    const float damping = relVel < 0.f ? SUSP_DAMPING_COMPRESSION : SUSP_DAMPING_RELAXATION;

    float suspForce = ((restLen - suspLen) * SUSP_STIFFNESS - damping * projVel) * clipped * suspForceScale(wheel);
    if (suspForce <= 0.f) suspForce = 0.f;

    float suspImpulse = 0.f;
    if (suspForce != 0.f)
    {
        suspImpulse = suspForce * PHYS_DT;
        const float pushbackThreshold = restLen + radius - SUSPENSION_SUBTRACTION;
        if (dist < pushbackThreshold)
        {
            const float penetration = pushbackThreshold - dist;
            const V3 torqueAxis = cross(fullRelPos, normal);
            const V3 invTorque = invInertiaWorld(body.rot, torqueAxis);
            const float jacobian = CAR_INV_MASS + dot(invTorque, torqueAxis);
            const float jacInv = 1.f / fmaxf(jacobian, 1e-8f);
            const float posError = SUSP_PUSHBACK_ERP * penetration / f.pushbackDt;
            const float velError = -projVel;
            float pushback = (posError + velError) * jacInv;
            if (pushback < 0.f) pushback = 0.f;
            suspImpulse += pushback * 0.25f;
        }
    }

    deltaVel = normal * (suspImpulse * CAR_INV_MASS);
    directAng = invInertiaWorld(body.rot, cross(fullRelPos, normal)) * suspImpulse;

    V3 lateralAxle = f.right;
    if (wheel < 2 && fabsf(steerPrev) > 1e-6f)
    {
        float s, c;
        fast_sincos(steerPrev, &s, &c);
        lateralAxle = f.right * c + cross(f.up, f.right) * s;
    }

    V3 axleDir = lateralAxle - normal * dot(lateralAxle, normal);
    const float axleLenSq = lensq(axleDir);
    if (axleLenSq <= 1e-10f) return true;
    axleDir = axleDir * rsqrtf(axleLenSq);

    const V3 lateralRelPos = fullRelPos - f.up * dot(f.up, fullRelPos);
    const V3 hardPointVel = pointVel + f.angCrossUp * dist;
    const V3 curveLongDir = cross(lateralAxle, normal);
    const V3 forwardDir = cross(normal, axleDir);

    float curveInput = 0.f;
    const float baseFriction = fabsf(dot(hardPointVel, lateralAxle));
    if (baseFriction > 5.f) curveInput = baseFriction / (fabsf(dot(hardPointVel, curveLongDir)) + baseFriction);

    float lateralBase = 1.f - 0.8f * clampf(curveInput, 0.f, 1.f);
    float longitudinalBase = 1.f;
    if (handbrake > 0.f)
    {
        lateralBase *= (0.1f - 1.f) * handbrake + 1.f;
        longitudinalBase *= ((0.5f + 0.4f * clampf(curveInput, 0.f, 1.f)) - 1.f) * handbrake + 1.f;
    }
    const float frictionScale = throttle != 0.f ? 1.f : nonStickyFriction(normal.z);
    const float lateralFriction = lateralBase * frictionScale;
    const float longitudinalFriction = longitudinalBase * frictionScale;

    // The reference's source uses each coefficient one tick after it is computed;
    // its CUDA build uses the current tick's lateral one (unlaggedLateral, the
    // default; CARLB_SOURCE_LAGGED_LATERAL_FRICTION selects the source's form).
    const float latUsed = unlaggedLateral ? lateralFriction : latPrev;
    const float lonUsed = lonPrev;
    latPrev = lateralFriction;
    lonPrev = longitudinalFriction;

    const V3 torqueAxis = cross(fullRelPos, axleDir);
    const V3 angularLateral = invInertiaWorld(body.rot, torqueAxis);
    const float jacobian = CAR_INV_MASS + dot(axleDir, cross(angularLateral, fullRelPos));
    const float latJacInv = 1.f / fmaxf(jacobian, 1e-8f);
    const float lateralVel = dot(axleDir, pointVel);
    constexpr float CONTACT_DAMPING = 0.2f;
    const float sideImpulse = -CONTACT_DAMPING * lateralVel * latJacInv;

    const float longitudinalVel = dot(forwardDir, pointVel);
    constexpr float ROLLING_FRICTION_SCALE = 113.73963f;
    const float rolling = enginePrev != 0.f
        ? -0.75f * enginePrev
        : clampf(-longitudinalVel * ROLLING_FRICTION_SCALE, -f.brakeTorque, f.brakeTorque);

    V3 wheelImpulse = axleDir * (sideImpulse * latUsed) + forwardDir * (rolling * lonUsed);
    wheelImpulse = wheelImpulse * ((CAR_MASS / 3.f) * PHYS_DT);

    directVel = wheelImpulse * CAR_INV_MASS;
    directAng = directAng + invInertiaWorld(body.rot, cross(lateralRelPos, wheelImpulse));
    return true;
}

// Whole suspension stage for one car.  `manCount` / `manNormal0` are the
// car-arena manifold from the previous tick.
CB_D void applySuspension(Body& body, Susp& susp, float* lat, float* lon, const float* rayDist,
                          const V3* rayNormal, int manCount, V3 manNormal0, int tick,
                          bool unlaggedLateral = false)
{
    const float brakeTorque = susp.brakePrev * (CAR_MASS * (14.25f + 1.f / 3.f));
    const V3 up = rotate(body.rot, axisVec(2));
    SuspFrame f;
    f.cenOffset = body.cen - body.pos;
    f.forward = rotate(body.rot, axisVec(0));
    f.right = rotate(body.rot, axisVec(1));
    f.up = up;
    f.vel = body.vel;
    f.ang = body.ang;
    f.angCrossUp = cross(body.ang, up);
    f.brakeTorque = brakeTorque;
    f.pushbackDt = tick <= 1 ? SUSP_PUSHBACK_DT_FIRST_TICK : PHYS_DT;

    V3 normalSum = v3zero();
    int contactCount = 0;
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        V3 dv, da, dd;
        const bool contact = suspWheel(body, f, w, rayDist[w], rayNormal[w], susp.steerPrev, susp.handbrake,
                                       susp.throttle, susp.enginePrev, lat[w], lon[w], dv, da, dd, unlaggedLateral);
        body.vel = body.vel + dv;
        body.ang = body.ang + da;
        body.deltaVel = body.deltaVel + dd;
        // Non-touching wheels add a zero normal.
        normalSum = normalSum + (contact ? rayNormal[w] : v3zero());
        contactCount += contact;
    }

    // Sticky force and autoroll.
    const bool hasRawThrottle = susp.rawThrottle != 0.f;
    const bool hasWorldContact = manCount != 0;
    V3 upwards;
    bool autoroll = false;
    bool apply = true;
    if (contactCount > 0)
    {
        upwards = normalSum * rsqrtf(lensq(normalSum) + 1e-16f);
        const float forwardSpeed = fabsf(dot(f.vel, f.forward));
        const bool fullStick = susp.throttle != 0.f || forwardSpeed > CAR_STOPPING_VEL;
        float stickyScale = 0.5f;
        if (fullStick) stickyScale += 1.f - fabsf(upwards.z);
        body.extVel = body.extVel + upwards * (stickyScale * GRAVITY_Z * PHYS_DT);
        autoroll = hasRawThrottle && (contactCount < NUM_WHEELS || hasWorldContact);
    }
    else if (hasWorldContact)
    {
        upwards = manNormal0;
        autoroll = hasRawThrottle;
    }
    else
    {
        apply = false;
    }

    if (apply && autoroll)
    {
        const V3 groundDown = neg(upwards);
        const V3 crossRight = cross(upwards, f.forward);
        const V3 crossForward = cross(groundDown, crossRight);
        const float rightFactor = 1.f - clampf(dot(f.right, crossRight), 0.f, 1.f);
        const float forwardFactor = 1.f - clampf(dot(f.forward, crossForward), 0.f, 1.f);
        const V3 rightDir = f.forward * (dot(f.right, upwards) >= 0.f ? -1.f : 1.f);
        const V3 forwardDir = f.right * (dot(f.forward, upwards) >= 0.f ? 1.f : -1.f);
        body.deltaVel = body.deltaVel + groundDown * (CAR_AUTOROLL_FORCE * PHYS_DT);
        body.deltaAng = body.deltaAng + (forwardDir * forwardFactor + rightDir * rightFactor) * (CAR_AUTOROLL_TORQUE * PHYS_DT);
    }

    body.extVel = body.extVel + susp.jumpImp;
    susp.jumpImp = v3zero();
    body.extAng = body.extAng + susp.angImp;
    susp.angImp = v3zero();
}

}  // namespace cb
