"""Reset paths of the front end agree bit for bit (the reference's
tests/test_resets.py equivalences): a masked apply_reset_state (one fused
kernel) equals the indexed one given the compacted rows, and the combined
apply_reset_state equals set_ball + set_car + set_match_state +
reset_boost_pads; the env steps after each pair agree too."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import carl as front, workloads

pytestmark = pytest.mark.gpu

N_SIM, NB, NO = 96, 2, 2
N_CARS = NB + NO


def _rows(rng, k):
    import torch

    f = np.float32
    d = {
        "ball_position": np.stack([rng.uniform(-3000, 3000, k), rng.uniform(-4000, 4000, k),
                                   rng.uniform(100, 1500, k)], 1).astype(f),
        "ball_velocity": rng.normal(0, 500, (k, 3)).astype(f),
        "ball_angular_velocity": rng.normal(0, 1, (k, 3)).astype(f),
        "car_position": np.stack([rng.uniform(-3500, 3500, (k, N_CARS)), rng.uniform(-4500, 4500, (k, N_CARS)),
                                  rng.uniform(17, 600, (k, N_CARS))], 2).astype(f),
        "car_rotation": workloads.random_quat(rng, k * N_CARS).reshape(k, N_CARS, 4).astype(f),
        "car_velocity": rng.normal(0, 600, (k, N_CARS, 3)).astype(f),
        "car_angular_velocity": rng.normal(0, 2, (k, N_CARS, 3)).astype(f),
        "car_demoed": rng.uniform(size=(k, N_CARS)) < 0.1,
        "car_boost": rng.uniform(0, 100, (k, N_CARS)).astype(f),
        "blue_score": rng.integers(0, 5, k).astype(np.int32),
        "orange_score": rng.integers(0, 5, k).astype(np.int32),
        "episode_ticks": rng.integers(0, 1000, k).astype(np.int32),
    }
    return {name: torch.from_numpy(v).cuda() for name, v in d.items()}


def _envs():
    a, b = front.Env(N_SIM, NB, NO, 9), front.Env(N_SIM, NB, NO, 9)
    workloads.mixed_state(a._env, 10)
    b._env.restore(a._env.snapshot())
    return a, b


def _same(a, b, where):
    import torch

    sa, sb = a._env.snapshot(), b._env.snapshot()
    for name in sa:
        assert (sa[name] == sb[name]).all(), (where, name)
    for getter in ("get_obs", "get_state", "get_score_difference", "get_episode_ticks", "get_overtime"):
        assert torch.equal(getattr(a, getter)(), getattr(b, getter)()), (where, getter)


def _steps(a, b, rng, n=8):
    import torch

    for step in range(n):
        act = torch.from_numpy(workloads.discrete_actions(rng, N_SIM * N_CARS).reshape(N_SIM, N_CARS, 7)).cuda()
        a.step(act)
        b.step(act)
        torch.cuda.synchronize()
        _same(a, b, ("step", step))


def test_masked_reset_matches_indexed_reset():
    import torch

    rng = np.random.default_rng(11)
    a, b = _envs()
    act = torch.zeros((N_SIM, N_CARS, 7), dtype=torch.int32, device="cuda")
    a.step(act)
    b.step(act)  # obs buffers reflect the state before the resets
    mask = torch.from_numpy(rng.uniform(size=N_SIM) < 0.3).cuda()
    idx = torch.nonzero(mask).flatten().to(torch.int64)
    full = _rows(rng, N_SIM)
    a.apply_reset_state(**full, reset_mask=mask)
    b.apply_reset_state(**{k: v[idx] for k, v in full.items()}, simulation_indices=idx)
    torch.cuda.synchronize()
    _same(a, b, "reset")
    _steps(a, b, rng)
    a.close()
    b.close()


def test_combined_reset_matches_setters():
    import torch

    rng = np.random.default_rng(12)
    a, b = _envs()
    idx = torch.from_numpy(np.sort(rng.choice(N_SIM, 40, replace=False)).astype(np.int64)).cuda()
    r = _rows(rng, idx.numel())
    a.apply_reset_state(**r, simulation_indices=idx)
    b.reset_boost_pads(simulation_indices=idx)
    b.set_ball(r["ball_position"], r["ball_velocity"], r["ball_angular_velocity"], simulation_indices=idx)
    b.set_car(r["car_position"], r["car_rotation"], r["car_velocity"], r["car_angular_velocity"], r["car_demoed"],
              boost=r["car_boost"], simulation_indices=idx)
    b.set_match_state(r["blue_score"], r["orange_score"], r["episode_ticks"], simulation_indices=idx)
    torch.cuda.synchronize()
    sa, sb = a._env.snapshot(), b._env.snapshot()
    for name in sa:
        assert (sa[name] == sb[name]).all(), name
    _steps(a, b, rng)
    a.close()
    b.close()
