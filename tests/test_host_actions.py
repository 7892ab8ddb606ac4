"""carlb_ticks_host with the actions copied in slice by slice beside the launch
(the default for the staged path; CARLB_OVERLAP_COPY=0 copies them on the env
stream first): the state and rewards equal those of the device-actions path,
with 2 sim slices, graph replay on and off, every action kind, tick counts 0, 1
and 8, and the host buffer rewritten right after each call returns."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads

pytestmark = pytest.mark.gpu


def _env(monkeypatch, graph: bool, overlap: bool, n_sim: int, nb: int, no: int) -> capi.Env:
    monkeypatch.setenv("CARLB_GRAPH", "1" if graph else "0")
    monkeypatch.setenv("CARLB_OVERLAP_COPY", "1" if overlap else "0")
    return capi.Env(n_sim, nb, no, 41)


def _actions(rng, kind: int, n_cars: int) -> np.ndarray:
    if kind == capi.ACTIONS_DIRECT:
        return workloads.controls(rng, n_cars)
    if kind == capi.ACTIONS_DISCRETE:
        return workloads.discrete_actions(rng, n_cars)
    return rng.uniform(-1.2, 1.2, (n_cars, 7)).astype(np.float32)


@pytest.mark.parametrize("graph", [True, False])
def test_sliced_host_copy_equals_device_actions(monkeypatch, graph):
    import torch

    n_sim, nb, no = 8192, 2, 2  # two slices of 4096 sims
    n_cars = n_sim * (nb + no)
    a = _env(monkeypatch, graph, True, n_sim, nb, no)
    b = _env(monkeypatch, graph, True, n_sim, nb, no)
    c = _env(monkeypatch, graph, False, n_sim, nb, no)
    workloads.mixed_state(a, 42)
    snap = a.snapshot()
    b.restore(snap)
    c.restore(snap)
    rng = np.random.default_rng(43)
    rb = np.zeros(n_sim, np.float32)
    rc = np.zeros(n_sim, np.float32)
    host = torch.empty(n_cars * 8, dtype=torch.int32).pin_memory().numpy()
    kinds = [capi.ACTIONS_DIRECT, capi.ACTIONS_DISCRETE, capi.ACTIONS_CONTINUOUS]
    for call, (kind, n_ticks) in enumerate([(k, n) for k in kinds for n in (8, 1, 0, 8)]):
        act = _actions(rng, kind, n_cars)
        words = act.view(np.int32).reshape(-1)
        a.ticks(kind, torch.from_numpy(words.copy()).cuda(), n_ticks)
        host[: words.size] = words  # pinned source for b
        b.ticks_host(kind, host, n_ticks, rb)
        host[:] = -1  # the call has returned: its buffer may be reused at once
        c.ticks_host(kind, act, n_ticks, rc)
        a.synchronize()
        sa, sb, sc = a.snapshot(), b.snapshot(), c.snapshot()
        for name in sa:
            assert (sa[name] == sb[name]).all(), (call, kind, n_ticks, name)
            assert (sa[name] == sc[name]).all(), (call, kind, n_ticks, name)
        assert np.array_equal(rb.view(np.int32), rc.view(np.int32)), call
    for e in (a, b, c):
        e.close()
