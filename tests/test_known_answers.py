"""Known-answer cases from the reference's own device tests
(tests/physics_regressions.cu:19-150, tests/turtle_recovery.cu:31-78), with
their expectation tables restated here.  Each case runs on the reference's
physics compiled for the host (the oracle) and on the product's physics
compiled for the host; the per-sim reset case also runs through the C ABI on
the device."""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from carl_b200 import capi
import host_tick_lib

# tests/physics_regressions.cu:32-41: (pitch, yaw, roll) and whether a flip starts.
DODGE_CASES = [((0.0, 1.0, -1.0), True), ((0.0, -1.0, 1.0), True), ((0.3, 0.3, 0.0), True),
               ((-0.3, -0.3, 0.0), True), ((0.0, 0.25, -0.25), True), ((0.0, 0.24, -0.24), False),
               ((0.0, 0.0, 0.0), False), ((1.0, 0.0, 0.0), True)]
# tests/turtle_recovery.cu:66-76: (yaw, roll, expected, jump, contacts, normal).
TURTLE_CASES = [(yaw, roll, exp, True, 1, (0.0, 0.0, 1.0))
                for yaw in (0.0, 0.7, math.pi / 2, math.pi, -math.pi / 2, -0.7)
                for roll, exp in ((-3.0, True), (3.0, True), (-2.7, False), (2.7, False))]
TURTLE_CASES += [(0.0, 3.0, False, False, 1, (0.0, 0.0, 1.0)), (0.0, 3.0, False, True, 0, (0.0, 0.0, 1.0)),
                 (0.0, 3.0, False, True, 1, (1.0, 0.0, 0.0))]


class _Impl:
    def __init__(self, lib, prefix):
        self.lib, self.p = lib, prefix
        f = ctypes.c_float
        vp, i = ctypes.c_void_p, ctypes.c_int
        getattr(lib, prefix + "ball_hit_previous_tick").argtypes = [i, i]
        getattr(lib, prefix + "floor_push_z").argtypes = [i]
        getattr(lib, prefix + "floor_push_z").restype = f
        getattr(lib, prefix + "dodge").argtypes = [f, f, f, vp, vp]
        getattr(lib, prefix + "goal_twice").argtypes = [i, vp, vp]
        getattr(lib, prefix + "steer_lag").argtypes = [vp]
        getattr(lib, prefix + "autoflip").argtypes = [f, f, i, i, f, f, f, vp]

    def call(self, name, *args):
        return getattr(self.lib, self.p + name)(*args)


@pytest.fixture(scope="module", params=["oracle", "product"])
def impl(request, oracle_built):
    if request.param == "oracle":
        return _Impl(ctypes.CDLL(str(oracle_built / "libcarlref_ka.so")), "refka_")
    return _Impl(host_tick_lib.lib(), "ka_")


def test_hit_age(impl):
    assert not impl.call("ball_hit_previous_tick", -1, 0)
    assert impl.call("ball_hit_previous_tick", 99, 100)
    assert not impl.call("ball_hit_previous_tick", 98, 100)
    assert not impl.call("ball_hit_previous_tick", 100, 100)


def test_floor_split_suppressed_right_after_a_hit(impl):
    assert impl.call("floor_push_z", 1) == 0.0
    assert impl.call("floor_push_z", 2) > 0.0


@pytest.mark.parametrize("inputs, flips", DODGE_CASES)
def test_dodge_or_double_jump(impl, inputs, flips):
    flags = np.zeros(2, np.int32)
    vel = np.zeros(3, np.float32)
    impl.call("dodge", *inputs, flags.ctypes.data, vel.ctypes.data)
    assert bool(flags[0]) == flips and bool(flags[1]) == (not flips)
    assert np.isfinite(vel).all()
    if DODGE_CASES.index((inputs, flips)) < 2:
        assert float((vel.astype(np.float64) ** 2).sum()) == 0.0


@pytest.mark.parametrize("sign", [-1, 1])
def test_goal_recorded_once_and_ball_kept(impl, sign):
    goals = np.zeros(5, np.int32)
    ball = np.zeros(2, np.float32)
    impl.call("goal_twice", sign, goals.ctypes.data, ball.ctypes.data)
    blue, orange, scorer, tick, first_tick = goals.tolist()
    assert blue + orange == 1 and scorer == sign and tick == first_tick
    assert ball[0] == 0.0 and ball[1] == 0.0


def test_steer_lag(impl):
    out = np.zeros(2, np.float32)
    impl.call("steer_lag", out.ctypes.data)
    assert out[0] == np.float32(0.25) and out[1] == 0.0


@pytest.mark.parametrize("yaw, roll, expected, jump, contacts, normal", TURTLE_CASES)
def test_turtle_recovery(impl, yaw, roll, expected, jump, contacts, normal):
    out = np.zeros(4, np.float32)
    impl.call("autoflip", yaw, roll, int(jump), contacts, *normal, out.ctypes.data)
    flipping, timer, torque, ang_sq = out.tolist()
    if expected:
        assert flipping and torque * roll < 0 and timer > 0
    else:
        assert not flipping and ang_sq == 0.0


def test_oracle_reset_ball_and_per_sim_reset(oracle_built):
    lib = ctypes.CDLL(str(oracle_built / "libcarlref_ka.so"))
    assert lib.refka_reset_ball_clears_valid() == 0
    out = np.zeros(2 * 3 + 4 * 5, np.int32)
    lib.refka_reset_after_done.argtypes = [ctypes.c_void_p]
    lib.refka_reset_after_done(out.ctypes.data)
    sims, cars = out[:6].reshape(2, 3), out[6:].reshape(4, 5)
    assert sims[0].tolist() == [0, 0, -1] and sims[1].tolist() == [0, 10, 77]
    assert (cars[:2, 0] == -1).all() and (cars[2:, 0] == 77).all()
    assert (cars[:2, 1:] == 0).all() and (cars[2:, 1:] == 3).all()  # WHEEL_NONE / WHEEL_BALL


@pytest.mark.gpu
def test_device_reset_clears_only_the_finished_sim():
    """tests/physics_regressions.cu:112-150 through the C ABI: sim 0 scored, sim 1 did not."""
    env = capi.Env(2, 1, 1, 42)
    env.set_limit(capi.LIMIT_MAX_TICKS, 1200)
    env.set_limit(capi.LIMIT_OVERTIME_TIMEOUT_TICKS, 1200)
    env.set_limit(capi.LIMIT_NO_TOUCH_TIMEOUT_TICKS, 0)
    env.write_field("TICK_COUNT", np.array([[77]], np.int32))
    goals = np.zeros(env.field_shape("GOALS"), np.int32)
    goals[0, 2] = 1  # lastScorer of sim 0
    env.write_field("GOALS", goals)
    env.write_field("EPISODE_TICKS", np.full((2, 1), 10, np.int32))
    env.write_field("LAST_TOUCH_TICKS", np.full((2, 1), 77, np.int32))
    env.write_field("BALL_ARENA_CONTACT_TICK", np.full((2, 1), 77, np.int32))
    env.write_field("CAR_ARENA_CONTACT_TICK", np.full((4, 1), 77, np.int32))
    env.write_field("CAR_WHEEL_SOURCE", np.full((4, 4), 3, np.int32))
    env.reset_dones()
    env.synchronize()
    g = env.read_field("GOALS").view(np.int32)
    ep = env.read_field("EPISODE_TICKS").view(np.int32)[:, 0]
    bact = env.read_field("BALL_ARENA_CONTACT_TICK").view(np.int32)[:, 0]
    cact = env.read_field("CAR_ARENA_CONTACT_TICK").view(np.int32)[:, 0]
    ws = env.read_field("CAR_WHEEL_SOURCE").view(np.int32)
    assert g[0, 2] == 0 and ep[0] == 0 and ep[1] == 10
    assert bact[0] == -1 and bact[1] == 77
    assert (cact[:2] == -1).all() and (cact[2:] == 77).all()
    assert (ws[:2] == 0).all() and (ws[2:] == 3).all()
    # Resetting the ball clears its integration cache flag (physics_regressions.cu:100-102).
    env.write_field("BALL_INT_VALID", np.ones((2, 1), np.int32))
    env.reset()
    assert (env.read_field("BALL_INT_VALID").view(np.int32) == 0).all()
    env.close()
