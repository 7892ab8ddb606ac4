"""An env step's packing and auto-reset in one kernel (CARLB_FUSED_EPILOGUE=1)
leave the same state and outputs as the seven separate kernels (the default),
bit for bit, over episodes that end by goals, timeouts, no-touch timeouts and
overtime, for every obs option and team size (CTAs that split the last sims
unevenly included).  Parity of the step with the reference is checked in
test_gpu_env.py."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads
from test_gpu_env import ALL_BUFFERS, read_buffer

pytestmark = pytest.mark.gpu

CASES = [
    (2048, 3, 3, 8, {}),
    (1001, 1, 1, 1, {"normalize": True}),
    (777, 4, 4, 2, {"previous_controls": True}),
    (515, 2, 1, 4, {"invert_orange": False, "normalize": True, "previous_controls": True}),
]


@pytest.mark.parametrize("n_sim,nb,no,frameskip,flags", CASES)
def test_fused_epilogue_equals_separate_kernels(monkeypatch, n_sim, nb, no, frameskip, flags):
    import torch

    n_cars = nb + no
    envs = []
    for fused in (True, False):
        monkeypatch.setenv("CARLB_FUSED_EPILOGUE", "1" if fused else "0")
        envs.append(capi.Env(n_sim, nb, no, 61, frameskip=frameskip, **flags))
    a, b = envs
    for e in envs:
        e.set_limit(capi.LIMIT_MAX_TICKS, 48)
        e.set_limit(capi.LIMIT_OVERTIME_TIMEOUT_TICKS, 24)
        e.set_limit(capi.LIMIT_NO_TOUCH_TIMEOUT_TICKS, 40)
    workloads.mixed_state(a, 62)
    b.restore(a.snapshot())
    rng = np.random.default_rng(63)
    dones = 0
    for step in range(96 // frameskip):
        act = torch.from_numpy(workloads.discrete_actions(rng, n_sim * n_cars)).cuda()
        a.env_step(capi.ACTIONS_DISCRETE, act)
        b.env_step(capi.ACTIONS_DISCRETE, act)
        dones += int(read_buffer(a, capi.BUF_DONES).sum())
        for buf in ALL_BUFFERS:
            assert (read_buffer(a, buf) == read_buffer(b, buf)).all(), (step, buf)
        sa, sb = a.snapshot(), b.snapshot()
        for name in sa:
            assert (sa[name] == sb[name]).all(), (step, name)
    assert dones > 0
    a.close()
    b.close()
