"""The reference's own Python layer on this project's drop-in module.

The reference's package (python/carl/__init__.py:11-20) imports its native
module as `carl._carl`.  Here carl_b200.carl is installed under that name, the
reference's package is imported from its source tree unchanged, and its
pure-Python layer runs on top:

* its own test file tests/test_state_views.py (view layout and storage);
* its state views (python/carl/gymnasium/state.py: CarlState, CARLObservation,
  the car and ball views) over output buffers of this project's front end,
  checked against the snapshot words those buffers were packed from;
* its action codec (python/carl/gymnasium/action.py:17-37) over this project's
  observations, checked against the device mask kernel's output;
* its reward context (state.py:503-515) built from this project's transition
  state, previous state, observations, events and counters as the wrapper builds
  it for `reward_funcs` (gymnasium/torch.py:371-418), with reward functions over
  those views checked against the snapshot words.

The buffers come from tests/golden/make_front_end_fixture.py, run on a GPU
machine (the reference's CUDA module cannot run here and its Python sources
cannot run there).  The gymnasium wrapper itself (gymnasium/torch.py) needs
the `gymnasium` package, which this image does not have; its import is not
attempted.  Skipped when the reference tree is absent.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import pytest

from oracle.paths import reference_dir

REF = reference_dir()
GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = sorted(GOLDEN.glob("front_end_*.npz"))

pytestmark = pytest.mark.skipif(not (REF / "python" / "carl" / "__init__.py").exists(),
                                reason="reference tree absent")


@pytest.fixture(scope="module")
def ref_carl():
    """The reference's `carl` package with carl_b200.carl as its `_carl`, and
    its gymnasium state / action modules (loaded without the gymnasium wrapper)."""
    from carl_b200 import carl as front

    saved = {k: v for k, v in sys.modules.items() if k == "carl" or k.startswith("carl.")}
    for k in saved:
        del sys.modules[k]
    pkg_dir = REF / "python" / "carl"
    sys.modules["carl._carl"] = front
    spec = importlib.util.spec_from_file_location("carl", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    carl = importlib.util.module_from_spec(spec)
    sys.modules["carl"] = carl
    spec.loader.exec_module(carl)
    gym = types.ModuleType("carl.gymnasium")
    gym.__path__ = [str(pkg_dir / "gymnasium")]
    sys.modules["carl.gymnasium"] = gym
    mods = {}
    for name in ("state", "action"):
        s = importlib.util.spec_from_file_location(f"carl.gymnasium.{name}", pkg_dir / "gymnasium" / f"{name}.py")
        m = importlib.util.module_from_spec(s)
        sys.modules[f"carl.gymnasium.{name}"] = m
        s.loader.exec_module(m)
        mods[name] = m
    yield carl, mods["state"], mods["action"]
    for k in [k for k in sys.modules if k == "carl" or k.startswith("carl.")]:
        del sys.modules[k]
    sys.modules.update(saved)


def test_reference_package_imports_the_drop_in(ref_carl):
    from carl_b200 import carl as front

    carl, _, _ = ref_carl
    assert carl.Env is front.Env
    for name in carl.__all__:
        assert getattr(carl, name) is getattr(front, name), name
    assert "Env" in carl.__all__ and "OBS_BALL" in carl.__all__


def test_reference_state_view_tests(ref_carl):
    """The reference's tests/test_state_views.py, run as written."""
    path = REF / "tests" / "test_state_views.py"
    spec = importlib.util.spec_from_file_location("ref_test_state_views", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    tests = [getattr(mod, n) for n in dir(mod) if n.startswith("test_")]
    assert tests
    for t in tests:
        t()


def _f32(words: np.ndarray) -> np.ndarray:
    return words.view(np.float32)


@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_reference_views_read_the_drop_in_buffers(ref_carl, path):
    import torch

    carl, state_mod, _ = ref_carl
    z = np.load(path)
    n_sim, nb, no, _, _, invert, normalize, prev = (int(x) for x in z["dims"])
    n_cars = nb + no
    team_sign = torch.tensor([1.0] * nb + [-1.0] * no)
    pads = torch.tensor(carl.BOOST_PAD_POSITIONS, dtype=torch.float32)
    state = state_mod.CarlState.from_raw(torch.from_numpy(z["state"]), n_cars, pads, team_sign)
    # The packed state is never normalised and never mirrored.
    ball_pos = _f32(z["snap/BALL_POS"]).reshape(n_sim, 3)
    car_pos = _f32(z["snap/CAR_POS"]).reshape(n_sim, n_cars, 3)
    car_vel = _f32(z["snap/CAR_VEL"]).reshape(n_sim, n_cars, 3)
    boost = _f32(z["snap/CAR_INTERNAL"])[:, 21].reshape(n_sim, n_cars)
    demoed = z["snap/CAR_IS_DEMOED"].view(np.int32).reshape(n_sim, n_cars)
    assert (state.ball_position.numpy() == ball_pos).all()
    assert (state.car_position.numpy() == car_pos).all()
    assert (state.car_velocity.numpy() == car_vel).all()
    assert (state.car_boost.numpy() == boost).all()
    assert (state.car_demoed.numpy() == (demoed != 0)).all()
    pad_cd = _f32(z["snap/PAD_COOLDOWNS"]).reshape(n_sim, 34)
    assert (state.boost_pad_active.numpy() == (pad_cd <= 0)).all()
    scale = (np.array(carl.OBS_POSITION_SCALE, np.float32) if normalize else np.ones(3, np.float32))
    pos_scale = lambda v: (v / scale).astype(np.float32)  # noqa: E731

    # Observations: the ego block is the agent's own car; for orange agents with
    # invert_orange the x and y axes are mirrored.
    obs = state_mod.CARLObservation.from_tensor(torch.from_numpy(z["obs"]), n_cars)
    ego = obs.cars.ego.position.numpy()
    sign = np.ones((n_sim, n_cars, 3), np.float32)
    if invert:
        sign[:, nb:, :2] = -1
    np.testing.assert_allclose(ego, pos_scale(car_pos) * sign, rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(obs.ball_position.numpy(), pos_scale(ball_pos)[:, None, :] * sign, rtol=1e-5,
                               atol=1e-4)
    assert obs.shape[-1] == carl.OBS_BALL + n_cars * carl.OBS_PER_CAR + carl.OBS_BOOST_PADS + \
        carl.OBS_RELATIVE_EGO_BALL + (n_cars - 1) * carl.OBS_RELATIVE_PER_OTHER_CAR + carl.OBS_RELATIVE_GOALS + \
        carl.OBS_EGO_DODGE + carl.OBS_EGO_CONTROLLER + (carl.OBS_PREVIOUS_CONTROLS if prev else 0)
    if prev:
        assert obs.ego_previous_controls.shape[-1] == carl.OBS_PREVIOUS_CONTROLS


@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_reference_action_codec_equals_the_device_mask(ref_carl, path):
    import torch

    _, _, action_mod = ref_carl
    z = np.load(path)
    prev = bool(int(z["dims"][7]))
    codec = action_mod.CARLActionCodec(previous_controls=prev)
    ref_mask = codec.mask(torch.from_numpy(z["obs"])).numpy()
    assert ref_mask.shape == z["mask"].shape
    assert (ref_mask == z["mask"].astype(bool)).all()


@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_reference_reward_context_over_the_drop_in(ref_carl, path):
    """The reference's RewardContext (state.py:503-515) built from this build's
    buffers the way its wrapper builds it for `reward_funcs`
    (gymnasium/torch.py:371-418, whose module needs gymnasium): the transition
    state and the previous state as CarlState, both observations, the events, the
    actions and the transition counters.  Reward functions written against those
    views give the values computed from the snapshot words directly."""
    import torch

    carl, state_mod, _ = ref_carl
    z = np.load(path)
    n_sim, nb, no, _, _, _, normalize, _ = (int(x) for x in z["dims"])
    n_cars = nb + no
    team_sign = torch.tensor([1.0] * nb + [-1.0] * no)
    pads = torch.tensor(state_mod.BOOST_PAD_POSITIONS, dtype=torch.float32)

    def carl_state(raw):
        return state_mod.CarlState.from_raw(torch.from_numpy(raw), n_cars, pads, team_sign)

    score_delta = torch.from_numpy(z["rewards"])
    done = torch.from_numpy(z["dones"]).bool()
    terminated = done & score_delta.ne(0)
    truncated = done & ~terminated
    ctx = state_mod.RewardContext(
        current=carl_state(z["transition_state"]),
        previous=carl_state(z["prev_state"]),
        current_observation=state_mod.CARLObservation.from_tensor(torch.from_numpy(z["obs"]), n_cars),
        previous_observation=state_mod.CARLObservation.from_tensor(torch.from_numpy(z["prev_obs"]), n_cars),
        events=state_mod.CarlEvents(score_delta=score_delta, done=done, terminated=terminated, truncated=truncated),
        actions=torch.from_numpy(z["actions/2"]),
        score_difference=torch.from_numpy(z["transition_score_difference"]),
        episode_ticks=torch.from_numpy(z["transition_episode_ticks"]),
        overtime=torch.from_numpy(z["transition_overtime"]),
    )

    def velocity_to_ball(c):
        to_ball = c.current.ball_position[:, None, :] - c.current.car_position
        return (c.current.car_velocity * to_ball / to_ball.norm(dim=-1, keepdim=True)).sum(-1)

    def boost_gained(c):
        return c.current.car_boost - c.previous.car_boost

    def goal(c):
        return c.events.score_delta[:, None] * team_sign[None, :]

    # The wrapper's accumulation: each function's result must be [n_sim, n_cars].
    reward = torch.zeros((n_sim, n_cars))
    for func in (velocity_to_ball, boost_gained, goal):
        r = func(ctx)
        assert r.shape == reward.shape
        reward += r

    # The same terms from the snapshot words (sims not reset by the step: there the
    # transition state is the state after the step).
    keep = ~z["dones"].astype(bool)
    car_pos = _f32(z["snap/CAR_POS"]).reshape(n_sim, n_cars, 3).astype(np.float64)
    car_vel = _f32(z["snap/CAR_VEL"]).reshape(n_sim, n_cars, 3).astype(np.float64)
    ball_pos = _f32(z["snap/BALL_POS"]).reshape(n_sim, 1, 3).astype(np.float64)
    to_ball = ball_pos - car_pos
    want = (car_vel * to_ball / np.linalg.norm(to_ball, axis=-1, keepdims=True)).sum(-1)
    want += _f32(z["snap/CAR_INTERNAL"])[:, 21].reshape(n_sim, n_cars) - \
        _f32(z["prev_snap/CAR_INTERNAL"])[:, 21].reshape(n_sim, n_cars)
    want += z["rewards"].astype(np.float64)[:, None] * np.array([1.0] * nb + [-1.0] * no)[None, :]
    np.testing.assert_allclose(reward.numpy()[keep], want[keep], rtol=1e-4, atol=1e-2)
    # The previous side is the state one step earlier, not the current one.
    assert (ctx.previous.car_position.numpy() == _f32(z["prev_snap/CAR_POS"]).reshape(n_sim, n_cars, 3)).all()
    assert not torch.equal(ctx.previous.car_position, ctx.current.car_position)
    # Transition counters: the sims' episode ticks (snapshot words) and no overtime.
    assert ctx.episode_ticks.shape == (n_sim,) and ctx.overtime.shape == (n_sim,)
    ticks = z["snap/EPISODE_TICKS"].reshape(n_sim).astype(np.int64)
    assert (ctx.episode_ticks.numpy()[keep] == ticks[keep]).all()
    assert not ctx.overtime.numpy().any()
