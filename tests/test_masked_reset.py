"""Masked apply_reset_state: the fused one-launch kernel (the default) leaves
the same state and outputs as the separate part kernels (CARLB_FUSED_RESET=0),
for every input option, obs option and mask density, and the ticks after it
agree too.  Parity of the reset itself with the reference's CUDA build is
checked in test_gpu_env.py."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads
from test_gpu_env import ALL_BUFFERS, read_buffer

pytestmark = pytest.mark.gpu


def _inputs(rng, n_sim, n_cars, demoed_byte, boost, internal, match):
    import torch

    f = np.float32
    d = {
        "ball_position": np.stack([rng.uniform(-3000, 3000, n_sim), rng.uniform(-4000, 4000, n_sim),
                                   rng.uniform(100, 1500, n_sim)], 1).astype(f),
        "ball_velocity": rng.normal(0, 500, (n_sim, 3)).astype(f),
        "ball_angular_velocity": rng.normal(0, 1, (n_sim, 3)).astype(f),
        "car_position": np.stack([rng.uniform(-3500, 3500, (n_sim, n_cars)),
                                  rng.uniform(-4500, 4500, (n_sim, n_cars)),
                                  rng.uniform(17, 600, (n_sim, n_cars))], 2).astype(f),
        "car_rotation": workloads.random_quat(rng, n_sim * n_cars).reshape(n_sim, n_cars, 4).astype(f),
        "car_velocity": rng.normal(0, 600, (n_sim, n_cars, 3)).astype(f),
        "car_angular_velocity": rng.normal(0, 2, (n_sim, n_cars, 3)).astype(f),
    }
    dem = rng.uniform(size=(n_sim, n_cars)) < 0.1
    d["car_demoed"] = dem.astype(np.uint8) if demoed_byte else dem.astype(np.int32)
    opt = {}
    if boost:
        opt["car_boost"] = rng.uniform(-10, 120, (n_sim, n_cars)).astype(f)
    if internal:
        st = rng.uniform(0, 1, (n_sim, n_cars, 19)).astype(f)
        st[..., [0, 3, 4, 5, 7, 8, 9, 11, 17]] = (st[..., [0, 3, 4, 5, 7, 8, 9, 11, 17]] < 0.5)
        opt["car_internal_state"] = st
    if match:
        opt["blue_score"] = rng.integers(0, 5, n_sim).astype(np.int32)
        opt["orange_score"] = rng.integers(0, 5, n_sim).astype(np.int32)
        opt["episode_ticks"] = rng.integers(0, 1000, n_sim).astype(np.int32)
    dev = {k: torch.from_numpy(v).cuda() for k, v in {**d, **opt}.items()}
    return dev


def _apply(env, inp, mask, demoed_byte):
    order = ["ball_position", "ball_velocity", "ball_angular_velocity", "car_position", "car_rotation",
             "car_velocity", "car_angular_velocity", "car_demoed"]
    env.apply_reset_state(env.n_sim, *[inp[o] for o in order], demoed_byte, inp.get("car_boost"),
                          inp.get("car_internal_state"), inp.get("blue_score"), inp.get("orange_score"),
                          inp.get("episode_ticks"), reset_mask=mask)


def _same(a, b, where):
    sa, sb = a.snapshot(), b.snapshot()
    for name in sa:
        assert (sa[name] == sb[name]).all(), (where, name)
    for buf in ALL_BUFFERS:
        assert (read_buffer(a, buf) == read_buffer(b, buf)).all(), (where, buf)


CASES = [
    # (n_sim, nb, no, density, demoed_byte, boost, internal, match, env flags)
    (4096, 3, 3, 0.01, True, False, False, False, {}),
    (4096, 3, 3, 0.3, False, True, True, True, {}),
    (2048, 4, 4, 1.0, True, True, False, True, {"normalize": True, "previous_controls": True}),
    (3000, 1, 2, 0.05, True, False, True, False, {"invert_orange": False}),
    (1024, 2, 2, 0.0, True, True, True, True, {}),
]


@pytest.mark.parametrize("n_sim,nb,no,density,demoed_byte,boost,internal,match,flags", CASES)
def test_fused_masked_reset_equals_part_kernels(monkeypatch, n_sim, nb, no, density, demoed_byte, boost, internal,
                                                match, flags):
    import torch

    n_cars = nb + no
    envs = []
    for fused in (True, False):
        monkeypatch.setenv("CARLB_FUSED_RESET", "1" if fused else "0")
        envs.append(capi.Env(n_sim, nb, no, 41, frameskip=2, **flags))
    a, b = envs
    workloads.mixed_state(a, 42)
    b.restore(a.snapshot())
    rng = np.random.default_rng(43)
    for rnd in range(3):
        mask = torch.from_numpy(rng.uniform(size=n_sim) < density).cuda()
        inp = _inputs(rng, n_sim, n_cars, demoed_byte, boost, internal, match)
        _apply(a, inp, mask, demoed_byte)
        _apply(b, inp, mask, demoed_byte)
        _same(a, b, ("reset", rnd))
        act = torch.from_numpy(workloads.discrete_actions(rng, n_sim * n_cars)).cuda()
        a.env_step(capi.ACTIONS_DISCRETE, act)
        b.env_step(capi.ACTIONS_DISCRETE, act)
        _same(a, b, ("step", rnd))
    a.close()
    b.close()
