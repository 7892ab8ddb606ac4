"""Staged ticks replayed from a captured CUDA graph (the default; CARLB_GRAPH=0
launches kernel by kernel) give the same state as the same ticks launched
kernel by kernel: across launches of different tick counts and action kinds,
after a reset, and after the tick counter is written directly."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads

pytestmark = pytest.mark.gpu


def _env(monkeypatch, graph: bool, n_sim: int, nb: int, no: int) -> capi.Env:
    monkeypatch.setenv("CARLB_GRAPH", "1" if graph else "0")
    return capi.Env(n_sim, nb, no, 31)


def _same(a: capi.Env, b: capi.Env, where) -> None:
    sa, sb = a.snapshot(), b.snapshot()
    for name in sa:
        assert (sa[name] == sb[name]).all(), (where, name)


@pytest.mark.parametrize("n_sim,nb,no", [(8192, 3, 3), (4096, 1, 2)])
def test_graph_replay_equals_launches(monkeypatch, n_sim, nb, no):
    import torch

    a = _env(monkeypatch, False, n_sim, nb, no)
    b = _env(monkeypatch, True, n_sim, nb, no)
    workloads.mixed_state(a, 32)
    b.restore(a.snapshot())
    rng = np.random.default_rng(33)
    n_cars = n_sim * (nb + no)
    # Repeated tick counts replay a cached graph; new ones capture another.
    for call, n_ticks in enumerate([8, 8, 3, 8, 3, 1]):
        ctl = torch.from_numpy(workloads.controls(rng, n_cars).view(np.int32)).cuda()
        a.ticks(capi.ACTIONS_DIRECT, ctl, n_ticks)
        b.ticks(capi.ACTIONS_DIRECT, ctl, n_ticks)
        _same(a, b, ("ticks", call))
    for call in range(3):
        act = torch.from_numpy(workloads.discrete_actions(rng, n_cars)).cuda()
        a.env_step(capi.ACTIONS_DISCRETE, act)
        b.env_step(capi.ACTIONS_DISCRETE, act)
        _same(a, b, ("env_step", call))
    a.reset()
    b.reset()
    for call in range(2):
        ctl = torch.from_numpy(workloads.controls(rng, n_cars).view(np.int32)).cuda()
        a.ticks(capi.ACTIONS_DIRECT, ctl, 8)
        b.ticks(capi.ACTIONS_DIRECT, ctl, 8)
        _same(a, b, ("after reset", call))
    tick = np.array([12345], dtype=np.int32)
    a.write_field("TICK_COUNT", tick)
    b.write_field("TICK_COUNT", tick)
    ctl = torch.from_numpy(workloads.controls(rng, n_cars).view(np.int32)).cuda()
    a.ticks(capi.ACTIONS_DIRECT, ctl, 8)
    b.ticks(capi.ACTIONS_DIRECT, ctl, 8)
    _same(a, b, "after tick write")
    a.close()
    b.close()


@pytest.mark.parametrize("graph", [False, True])
def test_stage_times(monkeypatch, graph):
    import torch

    n_sim = 8192
    env = _env(monkeypatch, graph, n_sim, 3, 3)
    workloads.mixed_state(env, 34)
    rng = np.random.default_rng(35)
    env.set_stage_timing(True)
    for _ in range(3):
        ctl = torch.from_numpy(workloads.controls(rng, n_sim * 6).view(np.int32)).cuda()
        env.ticks(capi.ACTIONS_DIRECT, ctl, 8)
        times = env.stage_times()
        assert list(times) == capi.Env.STAGES
        assert all(0.0 < ms < 100.0 for ms in times.values()), times
    env.set_stage_timing(False)
    env.close()
