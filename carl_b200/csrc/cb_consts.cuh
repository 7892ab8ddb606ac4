// Physical constants, tables and curves of the tick.
//
// Values and the constant expressions that produce them are those of the
// reference (jwmccarthy/CARL include/RLConstants.cuh:1-278,
// include/Physics/BoostPads.cuh:9-56, include/Arena/BroadPhaseGrid.cuh:9-10,
// include/Physics/BallArena/Contact.cuh:28-35, include/Physics/CarArena/Clip.cuh:12-13,
// include/Arena/TriMesh.cuh:11): they define the simulated game, and keeping the
// same constant expressions keeps every folded constant bit-identical.
#pragma once

#include "cb_math.cuh"

namespace cb {

// ---- math ----
constexpr float PI = 3.1415926535897932384626433832795029;
constexpr float PI_2 = PI / 2;
constexpr float PI_4 = PI / 4;
constexpr float SQRT_1_2 = 0.7071067811865475244f;
constexpr float FLOAT_EPSILON = 1.192092896e-07f;

// ---- arena and broadphase grid ----
constexpr float ARENA_MIN_X = -4108.f, ARENA_MIN_Y = -6000.f, ARENA_MIN_Z = -14.f;
constexpr float ARENA_MAX_X = 4108.f, ARENA_MAX_Y = 6000.f, ARENA_MAX_Z = 2076.f;
constexpr float GRID_X = 48.f, GRID_Y = 48.f, GRID_Z = 10.f;
constexpr float CELL_X = (ARENA_MAX_X - ARENA_MIN_X) / GRID_X;
constexpr float CELL_Y = (ARENA_MAX_Y - ARENA_MIN_Y) / GRID_Y;
constexpr float CELL_Z = (ARENA_MAX_Z - ARENA_MIN_Z) / GRID_Z;
constexpr int GRID_W = 48, GRID_H = 48, GRID_D = 10;
constexpr int NUM_CELLS = GRID_W * GRID_H * GRID_D;

// ---- car ----
constexpr float CAR_HALF_X = 60.186455f, CAR_HALF_Y = 43.282655f, CAR_HALF_Z = 19.262505f;
constexpr float CAR_OFF_X = 13.87566f, CAR_OFF_Y = 0.f, CAR_OFF_Z = 20.755f;
constexpr float CAR_SHAPE_MARGIN = 1.932955f;
constexpr float CAR_REST_Z = 17.f;
constexpr float CAR_RESPAWN_Z = 36.f;

// ---- ball ----
constexpr float BALL_REST_Z = 93.15f;
constexpr float BALL_COLLISION_RADIUS = 91.25f;

// ---- boost ----
constexpr int NUM_BOOST_PADS = 34;
constexpr float BOOST_MAX = 100.f;
constexpr float BOOST_SPAWN_AMOUNT = BOOST_MAX / 3.f;

// ---- wheels / suspension geometry ----
constexpr int NUM_WHEELS = 4;
constexpr float FRONT_WHEEL_RADIUS = 12.5f;
constexpr float BACK_WHEEL_RADIUS = 15.f;
constexpr float FRONT_SUSPENSION_REST = 26.755f;
constexpr float BACK_SUSPENSION_REST = 25.055f;
constexpr float MAX_SUSPENSION_TRAVEL = 12.f;
constexpr float SUSPENSION_SUBTRACTION = 2.5f;
constexpr float FRONT_SUSP_X = 37.3743f;
constexpr float FRONT_SUSP_Y = 25.9f;
constexpr float BACK_SUSP_X = -47.6257f;
constexpr float BACK_SUSP_Y = 29.5f;
constexpr float FRONT_SUSP_RAY_LEN =
    FRONT_SUSPENSION_REST + MAX_SUSPENSION_TRAVEL + FRONT_WHEEL_RADIUS - SUSPENSION_SUBTRACTION;
constexpr float BACK_SUSP_RAY_LEN =
    BACK_SUSPENSION_REST + MAX_SUSPENSION_TRAVEL + BACK_WHEEL_RADIUS - SUSPENSION_SUBTRACTION;

enum WheelSource { WHEEL_NONE = 0, WHEEL_ARENA = 1, WHEEL_CAR = 2, WHEEL_BALL = 3 };

// ---- collision capacity ----
constexpr int MAX_CAR_TRI_PAIRS = 32;
constexpr int MAX_PAIR_CONTACTS = 8;
constexpr int MAX_CAR_MANIFOLD_POINTS = 4;
constexpr float CAR_ANGULAR_MOTION_THRESH = PI_4;
constexpr float CAR_WORLD_RESTITUTION = 0.3f;
constexpr float CAR_WORLD_FRICTION = 0.3f;
constexpr float CAR_CONTACT_BREAK = 2.03122735f;
constexpr float CAR_MANIFOLD_BREAK_SQ = CAR_CONTACT_BREAK * CAR_CONTACT_BREAK;
constexpr float TRI_EDGE_DIST_MAX = 5.f;
constexpr float TRI_EDGE_DIST_MAX_SQ = TRI_EDGE_DIST_MAX * TRI_EDGE_DIST_MAX;
constexpr float BOUNDARY_EDGE_ANGLE = 2.f * PI;
constexpr float RAY_PARALLEL_EPS = 1e-8f;

// ---- rigid body ----
constexpr int PHYS_TICKS_PER_SECOND = 120;
constexpr float PHYS_DT = 1.f / PHYS_TICKS_PER_SECOND;
constexpr int REGULATION_TICKS = 5 * 60 * PHYS_TICKS_PER_SECOND;
constexpr float CAR_MASS = 180.f;
constexpr float CAR_INV_MASS = 1.f / CAR_MASS;
constexpr float CAR_MAX_SPEED = 2300.f;
constexpr float CAR_MAX_ANG_SPEED = 5.5f;
constexpr float CAR_INV_INERTIA_X = 1.f / 134665.94f;
constexpr float CAR_INV_INERTIA_Y = 1.f / 239607.22f;
constexpr float CAR_INV_INERTIA_Z = 1.f / 329747.90f;
constexpr float GRAVITY_Z = -650.f;

// ---- solver ----
constexpr int CAR_SOLVER_ITERS = 10;
constexpr float CAR_CONTACT_ERP = 0.8f;
constexpr float CAR_SOLVER_WARMSTART = 0.85f;
constexpr float CAR_SOLVER_LINEAR_SLOP = 0.f;
constexpr float CAR_SPLIT_IMPULSE_TURN_ERP = 0.1f;
constexpr float CAR_SPLIT_PENETRATION_THRESH = 1.0e30f;
constexpr float CAR_RESTITUTION_VEL_THRESH = 10.f;

// ---- suspension forces ----
constexpr float SUSP_STIFFNESS = 500.f;
constexpr float SUSP_DAMPING_COMPRESSION = 25.f;
constexpr float SUSP_DAMPING_RELAXATION = 40.f;
constexpr float SUSP_FORCE_SCALE_FRONT = 35.75f;
constexpr float SUSP_FORCE_SCALE_BACK = 54.265f;
constexpr float SUSP_PUSHBACK_ERP = 0.2f;
constexpr float SUSP_PUSHBACK_DT_FIRST_TICK = 1.f / 60.f;
constexpr float CAR_STOPPING_VEL = 25.f;
constexpr float CAR_AUTOROLL_FORCE = 100.f;
constexpr float CAR_AUTOROLL_TORQUE = 80.f;

// ---- jump and dodge ----
constexpr float JUMP_ACCEL = 4375.f / 3.f;
constexpr float JUMP_IMMEDIATE_FORCE = 875.f / 3.f;
constexpr float JUMP_MIN_TIME = 0.025f;
constexpr float JUMP_RESET_TIME_PAD = 1.f / 40.f;
constexpr float JUMP_MAX_TIME = 0.2f;
constexpr float DOUBLEJUMP_MAX_DELAY = 1.25f;
constexpr float FLIP_Z_DAMP_120 = 0.35f;
constexpr float FLIP_Z_DAMP_START = 0.15f;
constexpr float FLIP_Z_DAMP_END = 0.21f;
constexpr float FLIP_TORQUE_TIME = 0.65f;
constexpr float FLIP_PITCHLOCK_EXTRA_TIME = 0.3f;
constexpr float FLIP_INITIAL_VEL_SCALE = 500.f;
constexpr float FLIP_TORQUE_X = 260.f;
constexpr float FLIP_TORQUE_Y = 224.f;
constexpr float FLIP_FORWARD_IMPULSE_MAX_SPEED_SCALE = 1.f;
constexpr float FLIP_SIDE_IMPULSE_MAX_SPEED_SCALE = 1.9f;
constexpr float FLIP_BACKWARD_IMPULSE_MAX_SPEED_SCALE = 2.5f;
constexpr float FLIP_BACKWARD_IMPULSE_SCALE_X = 16.f / 15.f;
constexpr float DODGE_DEADZONE = 0.5f;

// ---- drive and boost ----
constexpr float THROTTLE_AIR_ACCEL = 200.f / 3.f;
constexpr float THROTTLE_GROUND_ACCEL = 1600.f;
constexpr float THROTTLE_DEADZONE = 0.001f;
constexpr float COASTING_BRAKE_FACTOR = 0.15f;
constexpr float BOOST_USED_PER_SECOND = BOOST_MAX / 3.f;
constexpr float BOOST_MIN_TIME = 0.1f;
constexpr float BOOST_ACCEL_GROUND = 2975.f / 3.f;
constexpr float BOOST_ACCEL_AIR = 3175.f / 3.f;
constexpr float POWERSLIDE_RISE_RATE = 5.f;
constexpr float POWERSLIDE_FALL_RATE = 2.f;

// ---- air control and autoflip ----
constexpr float CAR_TORQUE_SCALE = 2.f * PI / 65536.f * 1000.f;
constexpr float AIR_TORQUE_PITCH = 130.f, AIR_TORQUE_YAW = 95.f, AIR_TORQUE_ROLL = 400.f;
constexpr float AIR_DAMP_PITCH = 30.f, AIR_DAMP_YAW = 20.f, AIR_DAMP_ROLL = 50.f;
constexpr float CAR_AUTOFLIP_IMPULSE = 200.f;
constexpr float CAR_AUTOFLIP_TORQUE = 50.f;
constexpr float CAR_AUTOFLIP_TIME = 0.4f;
constexpr float CAR_AUTOFLIP_NORMZ_THRESH = 0.70710678f;
constexpr float CAR_AUTOFLIP_ROLL_THRESH = 2.8f;

// ---- car-car ----
constexpr float CARCAR_COLLISION_FRICTION = 0.09f;
constexpr float CARCAR_COLLISION_RESTITUTION = 0.1f;
constexpr float BUMP_COOLDOWN_TIME = 0.25f;
constexpr float BUMP_MIN_FORWARD_DIST = 64.5f;
constexpr float DEMO_RESPAWN_TIME = 3.f;
constexpr float DEMO_RESPAWN_INPUT_DEADZONE = 0.5f;
constexpr float SUPERSONIC_START_SPEED = 2200.f;

// ---- ball ----
constexpr float BALL_MASS = CAR_MASS / 6.f;
constexpr float BALL_INV_MASS = 1.f / BALL_MASS;
constexpr float BALL_RADIUS = BALL_COLLISION_RADIUS;
constexpr float BALL_DRAG = 0.03f;
constexpr float BALL_MAX_SPEED = 6000.f;
constexpr float BALL_MAX_ANG_SPEED = 6.f;
constexpr float BALL_WORLD_RESTITUTION = 0.6f;
constexpr float BALL_WORLD_FRICTION = 0.35f;
constexpr float BALL_INERTIA = 0.4f * BALL_MASS * BALL_RADIUS * BALL_RADIUS;
constexpr float BALL_INV_INERTIA = 1.f / BALL_INERTIA;
constexpr float BALL_ARENA_CONTACT_BREAK = 1.905f;

// ---- car-ball ----
constexpr float CAR_BALL_RESTITUTION = 0.f;
constexpr float CAR_BALL_FRICTION = 2.f;
constexpr float CAR_BALL_CONTACT_BREAK = 1.825f;
constexpr float CAR_BALL_SHAPE_MARGIN = CAR_SHAPE_MARGIN;
constexpr float CB_SOLVER_HALF_X = CAR_HALF_X + CAR_BALL_SHAPE_MARGIN;
constexpr float CB_SOLVER_HALF_Y = CAR_HALF_Y + CAR_BALL_SHAPE_MARGIN;
constexpr float CB_SOLVER_HALF_Z = CAR_HALF_Z + CAR_BALL_SHAPE_MARGIN;
constexpr float CB_CORE_HALF_X = CAR_HALF_X - CAR_BALL_SHAPE_MARGIN;
constexpr float CB_CORE_HALF_Y = CAR_HALF_Y - CAR_BALL_SHAPE_MARGIN;
constexpr float CB_CORE_HALF_Z = CAR_HALF_Z - CAR_BALL_SHAPE_MARGIN;
constexpr float BALL_CAR_EXTRA_IMPULSE_Z_SCALE = 0.35f;
constexpr float BALL_CAR_EXTRA_IMPULSE_FORWARD_SCALE = 0.65f;
constexpr float BALL_CAR_EXTRA_IMPULSE_MAXDELTAVEL_UU = 4600.f;

// ---- goals ----
constexpr float SOCCAR_GOAL_CENTER_Y = 5120.f;
constexpr float SOCCAR_GOAL_CENTER_Z = 321.3875f;
constexpr float SOCCAR_GOAL_SCORE_BASE_THRESHOLD_Y = 5124.25f;

// ---- boost pads ----
constexpr float SMALL_PAD_RADIUS = 144.f;
constexpr float BIG_PAD_RADIUS = 208.f;
constexpr float BOOST_PAD_HEIGHT = 95.f;
constexpr float SMALL_PAD_AMOUNT = 12.f;
constexpr float BIG_PAD_AMOUNT = 100.f;
constexpr float SMALL_PAD_COOLDOWN = 4.f;
constexpr float BIG_PAD_COOLDOWN = 10.f;

// ---- observation layout (include/Cuda/DLPack.h:76-107 of the reference) ----
constexpr int OBS_VECTOR_SIZE = 3;
constexpr int OBS_POS = 0, OBS_VEL = 3, OBS_ANG = 6, OBS_FORWARD = 9, OBS_UP = 12;
constexpr int OBS_BOOST = 15, OBS_ON_GROUND = 16, OBS_DEMOED = 17, OBS_HAS_FLIPPED = 18;
constexpr int OBS_HAS_DOUBLE_JUMPED = 19, OBS_IS_BOOSTING = 20, STATE_BALL_TOUCH = 21;
constexpr int OBS_BALL = OBS_FORWARD;
constexpr int OBS_PER_CAR = STATE_BALL_TOUCH;
constexpr int STATE_PER_CAR = STATE_BALL_TOUCH + 1;
constexpr int OBS_BOOST_PADS = 2 * NUM_BOOST_PADS;
constexpr int OBS_RELATIVE_EGO_BALL = 2 * OBS_VECTOR_SIZE;
constexpr int OBS_RELATIVE_PER_OTHER_CAR = OBS_RELATIVE_EGO_BALL;
constexpr int OBS_RELATIVE_GOALS = 2 * OBS_VECTOR_SIZE;
constexpr int OBS_EGO_DODGE = 2;
constexpr int OBS_EGO_CONTROLLER = 5;
constexpr int OBS_PREVIOUS_CONTROLS = 8;
constexpr int OBS_CONTROLLER_VERSION = 3;
constexpr int OBS_EGO_FLIP_INDEX = -OBS_EGO_DODGE - OBS_EGO_CONTROLLER;
constexpr int OBS_EGO_DODGE_TIME_INDEX = OBS_EGO_FLIP_INDEX + 1;
constexpr int CAR_INTERNAL_SIZE = 19;  // fields of the set_car internal-state record

CB_HD constexpr int observationDim(int nCars, bool previousControls)
{
    return OBS_BALL + nCars * OBS_PER_CAR + OBS_BOOST_PADS + OBS_RELATIVE_EGO_BALL
         + (nCars - 1) * OBS_RELATIVE_PER_OTHER_CAR + OBS_RELATIVE_GOALS + OBS_EGO_DODGE
         + OBS_EGO_CONTROLLER + (previousControls ? OBS_PREVIOUS_CONTROLS : 0);
}

CB_HD constexpr int packedStateDim(int nCars)
{
    return OBS_BALL + nCars * STATE_PER_CAR + NUM_BOOST_PADS;
}

// ---- actions (include/State/Controls.cuh:17-46 of the reference) ----
constexpr int ACT_PER_CAR = 7;
constexpr int ACTION_NVECS[ACT_PER_CAR] = { 3, 3, 3, 2, 2, 3, 2 };
constexpr int ACTION_LOGITS = 18;
constexpr int ACT_NON_NEUTRAL = 1;
// Logit columns the action mask gates (python/carl.cu:825-909 ACTION_*_LOGIT:
// the non-neutral logit of powerslide, boost and jump).
constexpr int ACTION_POWERSLIDE_LOGIT = 3 + 3 + 3 + 1;
constexpr int ACTION_BOOST_LOGIT = 3 + 3 + 3 + 2 + 1;
constexpr int ACTION_JUMP_LOGIT = 3 + 3 + 3 + 2 + 2 + 3 + 1;

// ---- curves ----
CB_HD float steerAngleFromSpeed(float x)
{
    if (x <= 0.f) return 0.53356f;
    if (x <= 500.f) return 0.53356f + (0.31930f - 0.53356f) * (x / 500.f);
    if (x <= 1000.f) return 0.31930f + (0.18203f - 0.31930f) * ((x - 500.f) / 500.f);
    if (x <= 1500.f) return 0.18203f + (0.10570f - 0.18203f) * ((x - 1000.f) / 500.f);
    if (x <= 1750.f) return 0.10570f + (0.08507f - 0.10570f) * ((x - 1500.f) / 250.f);
    if (x <= 3000.f) return 0.08507f + (0.03454f - 0.08507f) * ((x - 1750.f) / 1250.f);
    return 0.03454f;
}

CB_HD float powerslideSteerAngleFromSpeed(float x)
{
    if (x <= 0.f) return 0.39235f;
    if (x <= 2500.f) return 0.39235f + (0.12610f - 0.39235f) * (x / 2500.f);
    return 0.12610f;
}

CB_HD float driveSpeedTorqueFactor(float x)
{
    if (x <= 0.f) return 1.f;
    if (x >= 1410.f) return 0.f;
    if (x <= 1400.f) return 1.f - (x / 1400.f) * 0.9f;
    return 0.1f * (1.f - (x - 1400.f) / 10.f);
}

}  // namespace cb
