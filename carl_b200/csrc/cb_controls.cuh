// Car control state machine: drive/brake staging, boost, steering, jump,
// dodge / double jump, air control, flip torque and turtle auto-flip.
//
// Follows jwmccarthy/CARL include/Physics/Controls.cuh:7-35 (stage order),
// include/Physics/Controls/Context.cuh:55-111, Drive.cuh:6-178, Aerial.cuh:14-342
// and action decoding include/State/Controls.cuh:47-112, with the same fp32
// operation order.  Works on register copies of one car's state.
#pragma once

#include "cb_body.cuh"

namespace cb {

struct Controls
{
    float throttle, steer, yaw, pitch, roll;
    int jump, boost, slide;
};

struct Internal
{
    int isOnGround;
    float airTime, airTimeSinceJump, handbrakeVal;
    int hasJumped, isJumping;
    float jumpTime;
    int lastJump;
    int hasDoubleJumped, hasFlipped, isFlipping;
    float flipTime;
    int isAutoFlipping;
    float autoFlipTimer, autoFlipTorqueScale;
    V3 flipRelTorque;
    int respawnIdx, lastRespawnDir, isBoosting;
    float boost, boostingTime, timeSinceBoosted;
};

// Suspension / drive values staged by controls and consumed by the solve.
struct Susp
{
    float brake, brakePrev, throttle, rawThrottle, handbrake, steer, steerPrev, engine, enginePrev;
    V3 jumpImp, angImp;
};

// ---- action decoding ------------------------------------------------------------

CB_HD float discreteAxis(int32_t a) { return a == 1 ? -1.f : (a == 2 ? 1.f : 0.f); }
CB_HD float continuousAxis(float a) { return a < -1.f ? -1.f : (a > 1.f ? 1.f : a); }

// Discrete [horizontal, vertical, throttle, powerslide, boost, air_roll, jump].
CB_HD Controls decodeDiscrete(const int32_t* a)
{
    const float h = discreteAxis(a[0]);
    return Controls{ discreteAxis(a[2]), h, h, discreteAxis(a[1]), discreteAxis(a[5]),
                     a[6] == 1, a[4] == 1, a[3] == 1 };
}

CB_HD Controls decodeContinuous(const float* a)
{
    const float h = continuousAxis(a[0]);
    return Controls{ continuousAxis(a[2]), h, h, continuousAxis(a[1]), continuousAxis(a[5]),
                     a[6] >= .5f, a[4] >= .5f, a[3] >= .5f };
}

// ---- per-car control context ---------------------------------------------------------

struct ControlCtx
{
    Internal& s;
    Susp& susp;
    V3& vel;
    V3& ang;
    const Controls& c;
    Q4 rot;
    V3 fwd, up;
    float fwdSpeed, absFwdSpeed;
    int wheelConCount;
    bool onGround, jumpPressed;
    int manCount;    // car-arena manifold count from the previous tick
    V3 manNormal0;   // its first world normal
};

CB_D void addDeferredVel(ControlCtx& x, V3 v) { x.susp.jumpImp = x.susp.jumpImp + v; }

CB_D bool opposingThrottle(float throttle, float fwdSpeed, float absFwdSpeed)
{
    return absFwdSpeed > CAR_STOPPING_VEL && ((throttle > 0.f) != (fwdSpeed > 0.f));
}

CB_D void updateGroundDrive(ControlCtx& x)
{
    const float throttle = x.c.boost && x.s.boost > 0.f ? 1.f : x.c.throttle;
    const bool opposing = opposingThrottle(throttle, x.fwdSpeed, x.absFwdSpeed);

    float brake;
    if (x.wheelConCount == 0 || x.c.slide) brake = 0.f;
    else if (fabsf(throttle) >= THROTTLE_DEADZONE) brake = opposing ? 1.f : 0.f;
    else brake = x.absFwdSpeed < CAR_STOPPING_VEL ? 1.f : COASTING_BRAKE_FACTOR;

    float drive;
    if (x.wheelConCount == 0 || fabsf(throttle) < THROTTLE_DEADZONE || (!x.c.slide && opposing))
    {
        drive = 0.f;
    }
    else
    {
        float scale = driveSpeedTorqueFactor(x.absFwdSpeed);
        if (x.wheelConCount < 3) scale *= 0.25f;
        drive = throttle * THROTTLE_GROUND_ACCEL * scale;
    }

    x.susp.brakePrev = x.susp.brake;
    x.susp.brake = brake;
    x.susp.throttle = throttle;
    x.susp.rawThrottle = x.c.throttle;
    x.susp.enginePrev = x.susp.engine;
    x.susp.engine = drive;
}

CB_D void updateBoost(ControlCtx& x)
{
    Internal& s = x.s;
    bool boosting;
    if (s.boost <= 0.f) boosting = false;
    else if (!s.isBoosting) boosting = x.c.boost;
    else boosting = x.c.boost || s.boostingTime < BOOST_MIN_TIME;
    s.isBoosting = boosting;

    if (s.isBoosting)
    {
        s.boostingTime += PHYS_DT;
        s.boost = fmaxf(s.boost - BOOST_USED_PER_SECOND * PHYS_DT, 0.f);
        const float accel = x.onGround ? BOOST_ACCEL_GROUND : BOOST_ACCEL_AIR;
        addDeferredVel(x, x.fwd * (accel * PHYS_DT));
        s.timeSinceBoosted = 0.f;
    }
    else
    {
        s.boostingTime = 0.f;
        s.timeSinceBoosted += PHYS_DT;
    }
    s.boost = fminf(s.boost, BOOST_MAX);
}

CB_D void updateSteer(ControlCtx& x)
{
    Internal& s = x.s;
    if (x.c.slide) s.handbrakeVal += POWERSLIDE_RISE_RATE * PHYS_DT;
    else s.handbrakeVal -= POWERSLIDE_FALL_RATE * PHYS_DT;
    s.handbrakeVal = clampf(s.handbrakeVal, 0.f, 1.f);
    x.susp.handbrake = s.handbrakeVal;

    float angle = steerAngleFromSpeed(x.absFwdSpeed);
    if (s.handbrakeVal > 0.f)
    {
        const float slideAngle = powerslideSteerAngleFromSpeed(x.absFwdSpeed);
        angle += (slideAngle - angle) * s.handbrakeVal;
    }
    x.susp.steerPrev = x.susp.steer;
    x.susp.steer = angle * x.c.steer;
}

// ---- aerial --------------------------------------------------------------------------

CB_D bool applyFlipTorque(ControlCtx& x)
{
    Internal& s = x.s;
    if (s.isFlipping) s.isFlipping = s.hasFlipped && s.flipTime < FLIP_TORQUE_TIME;
    if (!s.isFlipping) return true;

    const V3 rel = s.flipRelTorque;
    if (lensq(rel) <= 1e-12f) return true;

    float pitchScale = 1.f;
    bool useAir = false;
    const bool hasPitchInput = rel.y != 0.f && x.c.pitch != 0.f;
    const bool pitchMatchesFlip = (rel.y > 0.f) == (x.c.pitch > 0.f);
    if (hasPitchInput && pitchMatchesFlip)
    {
        pitchScale = 1.f - fminf(fabsf(x.c.pitch), 1.f);
        useAir = true;
    }

    const V3 relTorque = { rel.x * FLIP_TORQUE_X, rel.y * FLIP_TORQUE_Y * pitchScale, 0.f };
    const V3 worldTorque = rotate(x.rot, relTorque);
    x.susp.angImp = x.susp.angImp + worldTorque * PHYS_DT;
    return useAir;
}

CB_D void applyAirTorque(ControlCtx& x)
{
    const Internal& s = x.s;
    const bool pitchLocked = s.isFlipping
        || (s.hasFlipped && s.flipTime < FLIP_TORQUE_TIME + FLIP_PITCHLOCK_EXTRA_TIME);
    const float pitchScale = pitchLocked ? 0.f : 1.f;

    const V3 input = { x.c.pitch, x.c.yaw, x.c.roll };
    const V3 controlScale = { pitchScale, 1.f, 1.f };
    const V3 dampInput = { x.c.pitch * pitchScale, x.c.yaw, 0.f };
    const V3 ang = x.ang;
    const V3 torqueCoef = { AIR_TORQUE_PITCH, AIR_TORQUE_YAW, AIR_TORQUE_ROLL };
    const V3 dampCoef = { AIR_DAMP_PITCH, AIR_DAMP_YAW, AIR_DAMP_ROLL };

    V3 torque = v3zero();
    V3 damping = v3zero();
    const bool hasInput = lensq(input) > 0.f;

    #pragma unroll
    for (int i = 0; i < 3; i++)
    {
        const V3 dir = i == 0 ? neg(rotate(x.rot, axisVec(1))) : (i == 1 ? x.up : neg(x.fwd));
        const float control = vget(input, i) * vget(controlScale, i);
        const float proj = dot(dir, ang);
        const float damp = proj * vget(dampCoef, i) * (1.f - fabsf(vget(dampInput, i)));
        if (hasInput) torque = torque + dir * (control * vget(torqueCoef, i));
        damping = damping + dir * damp;
    }
    x.susp.angImp = x.susp.angImp + (torque - damping) * (CAR_TORQUE_SCALE * PHYS_DT);
}

CB_D void updateAirControl(ControlCtx& x, bool allowAir)
{
    const bool useAir = applyFlipTorque(x);
    if (useAir && allowAir && !x.s.isAutoFlipping) applyAirTorque(x);
    if (x.c.throttle != 0.f) addDeferredVel(x, x.fwd * (x.c.throttle * THROTTLE_AIR_ACCEL * PHYS_DT));
}

// ---- jump ------------------------------------------------------------------------------

CB_D void updateJump(ControlCtx& x)
{
    Internal& s = x.s;
    const bool grace = s.hasJumped && s.jumpTime < JUMP_MIN_TIME + JUMP_RESET_TIME_PAD;
    if (x.onGround && !s.isJumping && !grace)
    {
        s.hasJumped = false;
        s.jumpTime = 0.f;
    }

    if (s.isJumping)
    {
        s.isJumping = s.jumpTime < JUMP_MIN_TIME || (x.c.jump && s.jumpTime < JUMP_MAX_TIME);
    }
    else if (x.onGround && x.jumpPressed)
    {
        s.isJumping = true;
        s.jumpTime = 0.f;
        addDeferredVel(x, x.up * JUMP_IMMEDIATE_FORCE);
    }

    if (s.isJumping)
    {
        s.hasJumped = true;
        float accel = JUMP_ACCEL;
        if (s.jumpTime < JUMP_MIN_TIME) accel *= 0.62f;
        addDeferredVel(x, x.up * (accel * PHYS_DT));
    }

    if (s.isJumping || s.hasJumped) s.jumpTime += PHYS_DT;
}

// ---- auto-flip (turtle recovery) ------------------------------------------------------------

CB_D void updateAutoFlip(ControlCtx& x)
{
    Internal& s = x.s;
    if (x.jumpPressed && x.manCount != 0 && x.manNormal0.z > CAR_AUTOFLIP_NORMZ_THRESH)
    {
        const V3 right = rotate(x.rot, axisVec(1));
        const float roll = -atan2f(right.z, x.up.z);
        const float absRoll = fabsf(roll);
        if (absRoll > CAR_AUTOFLIP_ROLL_THRESH)
        {
            s.autoFlipTimer = CAR_AUTOFLIP_TIME * (absRoll / PI);
            s.autoFlipTorqueScale = roll > 0.f ? 1.f : -1.f;
            s.isAutoFlipping = true;
            x.vel = x.vel + x.up * -CAR_AUTOFLIP_IMPULSE;
        }
    }
    if (!s.isAutoFlipping) return;

    if (s.autoFlipTimer <= 0.f)
    {
        s.isAutoFlipping = false;
        s.autoFlipTimer = 0.f;
        return;
    }
    const float torque = CAR_AUTOFLIP_TORQUE * s.autoFlipTorqueScale * PHYS_DT;
    x.ang = x.ang + x.fwd * torque;
    s.autoFlipTimer -= PHYS_DT;
}

// ---- dodge ---------------------------------------------------------------------------------

CB_D bool hasFlipOrJump(const Internal& s)
{
    return !s.hasFlipped && !s.hasDoubleJumped && s.airTimeSinceJump < DOUBLEJUMP_MAX_DELAY;
}

CB_D void startFlip(ControlCtx& x, V3 dodge)
{
    Internal& s = x.s;
    s.flipTime = 0.f;
    s.hasFlipped = true;
    s.isFlipping = true;

    if (fabsf(dodge.x) < 0.1f && fabsf(dodge.y) < 0.1f) dodge = v3zero();
    else dodge = dodge * rsqrtf(lensq(dodge));
    s.flipRelTorque = V3{ -dodge.y, dodge.x, 0.f };

    // Local dodge velocity, scaled by forward speed and direction.
    V3 d = dodge;
    if (fabsf(d.x) < 0.1f) d.x = 0.f;
    if (fabsf(d.y) < 0.1f) d.y = 0.f;
    const float speedScale = clampf(x.absFwdSpeed / CAR_MAX_SPEED, 0.f, 1.f);
    const bool isBackward = x.absFwdSpeed < 100.f ? d.x < 0.f : ((d.x >= 0.f) != (x.fwdSpeed >= 0.f));
    const float maxFwdScale = isBackward ? FLIP_BACKWARD_IMPULSE_MAX_SPEED_SCALE : FLIP_FORWARD_IMPULSE_MAX_SPEED_SCALE;
    V3 local = d * FLIP_INITIAL_VEL_SCALE;
    local.x *= (maxFwdScale - 1.f) * speedScale + 1.f;
    local.y *= (FLIP_SIDE_IMPULSE_MAX_SPEED_SCALE - 1.f) * speedScale + 1.f;
    if (isBackward) local.x *= FLIP_BACKWARD_IMPULSE_SCALE_X;

    // Into the car's horizontal world basis.
    const V3 flatFwd = { x.fwd.x, x.fwd.y, 0.f };
    const float denom = lensq(flatFwd);
    const V3 flatFwdN = denom > 1e-12f ? flatFwd * rsqrtf(denom) : axisVec(0);
    const V3 right = { -flatFwdN.y, flatFwdN.x, 0.f };
    x.vel = x.vel + (flatFwdN * local.x + right * local.y);
}

CB_D void updateDodge(ControlCtx& x)
{
    Internal& s = x.s;
    if (x.onGround)
    {
        s.hasDoubleJumped = false;
        s.hasFlipped = false;
        s.isFlipping = false;
        s.airTime = 0.f;
        s.airTimeSinceJump = 0.f;
        s.flipTime = 0.f;
    }
    else
    {
        s.airTime += PHYS_DT;
        if (s.hasJumped && !s.isJumping) s.airTimeSinceJump += PHYS_DT;
        else s.airTimeSinceJump = 0.f;

        if (x.jumpPressed && hasFlipOrJump(s))
        {
            const V3 dodge = { -x.c.pitch, x.c.yaw + x.c.roll, 0.f };
            const float magnitude = fabsf(x.c.yaw) + fabsf(x.c.pitch) + fabsf(x.c.roll);
            if (magnitude >= DODGE_DEADZONE)
            {
                startFlip(x, dodge);
            }
            else
            {
                x.vel = x.vel + x.up * JUMP_IMMEDIATE_FORCE;
                s.hasDoubleJumped = true;
            }
        }
    }

    // Flip motion: flip timer and vertical damping during the landing window.
    if (!s.isFlipping)
    {
        if (s.hasFlipped) s.flipTime += PHYS_DT;
        return;
    }
    s.flipTime += PHYS_DT;
    if (s.flipTime > FLIP_TORQUE_TIME) return;
    const bool dampZ = s.flipTime >= FLIP_Z_DAMP_START && (x.vel.z < 0.f || s.flipTime < FLIP_Z_DAMP_END);
    if (dampZ) x.vel.z *= 1.f - FLIP_Z_DAMP_120;
}

// ---- whole control stage for one car ---------------------------------------------------------

// rayDist: this tick's suspension ray distances.  Updates vel, ang, internal and
// staged suspension values in place.  Demoed cars only clear the staged impulses.
CB_D void processControls(const Controls& c, bool demoed, Q4 rot, V3& vel, V3& ang, Internal& s,
                          Susp& susp, const float* rayDist, int manCount, V3 manNormal0)
{
    if (demoed)
    {
        susp.jumpImp = v3zero();
        susp.angImp = v3zero();
        return;
    }
    ControlCtx x{ s, susp, vel, ang, c };
    x.rot = rot;
    x.fwd = rotate(rot, axisVec(0));
    x.up = rotate(rot, axisVec(2));
    x.fwdSpeed = dot(vel, x.fwd);
    x.absFwdSpeed = fabsf(x.fwdSpeed);
    int con = 0;
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
        if (rayDist[w] <= suspRayLength(w)) con++;
    x.wheelConCount = con;
    x.onGround = con >= 3;
    x.manCount = manCount;
    x.manNormal0 = manNormal0;
    x.jumpPressed = c.jump && !s.lastJump;
    s.lastJump = c.jump;
    s.isOnGround = x.onGround;

    updateGroundDrive(x);
    updateBoost(x);
    updateSteer(x);
    if (x.wheelConCount < 3) updateAirControl(x, x.wheelConCount == 0);
    updateJump(x);
    updateAutoFlip(x);
    updateDodge(x);
}

}  // namespace cb
