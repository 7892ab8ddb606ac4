"""The drop-in front end (carl_b200.Env, mirroring the reference's carl._carl.Env):
constants, argument validation and error types, output views, stream handoff."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest

import carl_b200
from carl_b200 import carl as front

from oracle.paths import reference_dir

REFERENCE = reference_dir()


def test_constants_match_the_reference_module():
    assert carl_b200.ACTION_NVECS == (3, 3, 3, 2, 2, 3, 2)
    assert carl_b200.ACTION_LOGITS == 18
    assert carl_b200.OBS_PER_CAR == 21 and carl_b200.STATE_PER_CAR == 22
    assert carl_b200.OBS_EGO_FLIP_INDEX == -7 and carl_b200.OBS_EGO_DODGE_TIME_INDEX == -6
    assert carl_b200.CAR_INTERNAL_SIZE == 19
    assert carl_b200.REGULATION_TICKS == 36000
    assert len(carl_b200.BOOST_PAD_POSITIONS) == carl_b200.NUM_BOOST_PADS == 34
    assert "Env" in carl_b200.__all__
    # Observation width formula (include/Cuda/DLPack.h:95-102) for 3v3: 252.
    n = 6
    dim = (front.OBS_BALL + n * front.OBS_PER_CAR + front.OBS_BOOST_PADS + front.OBS_RELATIVE_EGO_BALL
           + (n - 1) * front.OBS_RELATIVE_PER_OTHER_CAR + front.OBS_RELATIVE_GOALS + front.OBS_EGO_DODGE
           + front.OBS_EGO_CONTROLLER)
    assert dim == 252


@pytest.mark.skipif(not (REFERENCE / "python" / "carl.cu").exists(), reason="reference tree absent")
def test_constant_names_cover_the_reference_module():
    text = (REFERENCE / "python" / "carl.cu").read_text()
    names = set(re.findall(r'm\.attr\("([A-Z_]+)"\)', text))
    missing = sorted(n for n in names if not hasattr(carl_b200, n))
    assert not missing, missing


@pytest.mark.skipif(not (REFERENCE / "python" / "carl.cu").exists(), reason="reference tree absent")
def test_env_methods_cover_the_reference_class():
    text = (REFERENCE / "python" / "carl.cu").read_text()
    names = set(re.findall(r'\.def\("([a-z_]+)"', text)) | set(re.findall(r'\.def_property(?:_readonly)?\("([a-z_]+)"', text))
    missing = sorted(n for n in names if not hasattr(front.Env, n))
    assert not missing, missing


@pytest.fixture
def env():
    import torch

    e = front.Env(8, 1, 1, 7)
    yield e
    e.close()


@pytest.mark.gpu
def test_step_returns_obs_view(env):
    import torch

    actions = torch.zeros((8, 2, 7), dtype=torch.int32, device="cuda")
    obs = env.step(actions)
    assert obs.shape == (8, 2, env.obs_dim) and obs.dtype == torch.float32 and obs.is_cuda
    assert obs.data_ptr() == env.get_obs().data_ptr()  # the same in-place buffer
    # DLPack export as the reference's capsules: a CUDA device tuple, zero copy.
    assert obs.__dlpack_device__() == (2, torch.cuda.current_device())
    assert torch.from_dlpack(obs).data_ptr() == obs.data_ptr()
    assert env.get_dones().dtype == torch.bool and env.get_rewards().shape == (8,)
    assert env.get_state().shape == (8, 9 + 2 * 22 + 34)
    assert torch.isfinite(obs).all()


@pytest.mark.gpu
@pytest.mark.parametrize("bad, exc, msg", [
    (lambda t: t.zeros((8, 2, 7), dtype=t.float32, device="cuda"), TypeError, "int32"),
    (lambda t: t.zeros((8, 2, 7), dtype=t.int32), ValueError, "cuda"),
    (lambda t: t.zeros((8, 2, 6), dtype=t.int32, device="cuda"), ValueError, "shape"),
    (lambda t: t.zeros((8, 7, 2), dtype=t.int32, device="cuda").transpose(1, 2), ValueError, "contiguous"),
])
def test_step_validation(env, bad, exc, msg):
    import torch

    before = env.get_obs().clone()
    with pytest.raises(exc, match=msg):
        env.step(bad(torch))
    assert torch.equal(before, env.get_obs())


@pytest.mark.gpu
def test_step_continuous_and_frameskip(env):
    import torch

    env.frameskip = 4
    assert env.frameskip == 4
    with pytest.raises(ValueError):
        env.frameskip = 0
    obs = env.step_continuous(torch.zeros((8, 2, 7), dtype=torch.float32, device="cuda"))
    assert torch.isfinite(obs).all()
    assert int(env.get_episode_ticks()[0]) == 4


@pytest.mark.gpu
def test_reset_state_validation_and_effect(env):
    import torch

    k, nc = 3, 2
    idx = torch.tensor([0, 3, 5], dtype=torch.int64, device="cuda")
    z3 = torch.zeros((k, 3), device="cuda")
    pos = torch.tensor([[0.0, 0.0, 500.0]] * k, device="cuda")
    cars = torch.zeros((k, nc, 3), device="cuda")
    cars[..., 2] = 17.0
    cars[:, 1, 1] = 1000.0
    rot = torch.zeros((k, nc, 4), device="cuda")
    rot[..., 3] = 1.0
    demo = torch.zeros((k, nc), dtype=torch.bool, device="cuda")
    with pytest.raises(TypeError, match="int64"):
        env.apply_reset_state(pos, z3, z3, cars, rot, cars * 0, cars * 0, demo, simulation_indices=idx.int())
    with pytest.raises(ValueError, match="shape"):
        env.apply_reset_state(pos[:2], z3, z3, cars, rot, cars * 0, cars * 0, demo, simulation_indices=idx)
    with pytest.raises(ValueError, match="together"):
        env.apply_reset_state(pos, z3, z3, cars, rot, cars * 0, cars * 0, demo, blue_score=idx.int(),
                              simulation_indices=idx)
    env.apply_reset_state(pos, z3, z3, cars, rot, cars * 0, cars * 0, demo, simulation_indices=idx)
    state = env.get_state().clone()
    # Packed state starts with the ball position (unnormalised).
    assert torch.allclose(state[idx, 0:3], pos)


@pytest.mark.gpu
def test_stream_handoff_async_equals_sync():
    """Work queued by torch on another stream is seen by the env, and env
    outputs read on torch's stream after a wait match a fully synchronised run
    (reference tests/test_stream_handoff.py)."""
    import torch

    def run(sync: bool):
        e = front.Env(4, 1, 1, 7)
        frames = [e.get_obs().clone()]
        ext = torch.cuda.ExternalStream(e.stream)
        actions = torch.zeros((4, 2, 7), dtype=torch.int32, device="cuda")
        for step in range(8):
            if step == 4:
                zeros = torch.zeros((4, 3), device="cuda")
                position = zeros.clone()
                position[:, 2] = 800.0
                torch.cuda._sleep(50_000_000)  # the producer is still running when set_ball is queued
                e.set_ball(position, zeros, zeros)
            else:
                actions = actions + 1
                actions.remainder_(2)
                e.step(actions)
            if sync:
                torch.cuda.synchronize()
            torch.cuda.current_stream().wait_stream(ext)
            frames.append(e.get_obs().clone())
        e.close()
        return frames

    expected = run(True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        actual = run(False)
    torch.cuda.synchronize()
    for a, b in zip(actual, expected):
        assert torch.equal(a, b)
