"""Obs and state rows written through per-warp staging tiles (the default)
equal the rows a thread per row writes (CARLB_STAGED_PACK=0), bit for bit, for
every obs option, team sizes with a ragged last warp, and the masked packs
(transition obs of done sims).  The masked-reset tests cover the masked
packs the other way round: the fused reset writes its rows a thread per row,
the separate kernels through the staging tiles."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads
from test_gpu_env import ALL_BUFFERS, read_buffer

pytestmark = pytest.mark.gpu

CASES = [
    (2048, 3, 3, {}),
    (1001, 1, 2, {"normalize": True}),
    (777, 4, 4, {"normalize": True, "previous_controls": True}),
    (513, 2, 1, {"invert_orange": False, "previous_controls": True}),
]


@pytest.mark.parametrize("n_sim,nb,no,flags", CASES)
def test_staged_rows_equal_direct_rows(monkeypatch, n_sim, nb, no, flags):
    import torch

    n_cars = nb + no
    envs = []
    for staged in (True, False):
        monkeypatch.setenv("CARLB_STAGED_PACK", "1" if staged else "0")
        envs.append(capi.Env(n_sim, nb, no, 51, frameskip=4, **flags))
    a, b = envs
    for e in envs:
        e.set_limit(capi.LIMIT_MAX_TICKS, 40)  # episodes end within the test: transition packs masked by dones
        e.set_limit(capi.LIMIT_NO_TOUCH_TIMEOUT_TICKS, 24)
    workloads.mixed_state(a, 52)
    b.restore(a.snapshot())
    rng = np.random.default_rng(53)
    saw_done = False
    for step in range(16):
        act = torch.from_numpy(workloads.discrete_actions(rng, n_sim * n_cars)).cuda()
        a.env_step(capi.ACTIONS_DISCRETE, act)
        b.env_step(capi.ACTIONS_DISCRETE, act)
        saw_done |= bool(read_buffer(a, capi.BUF_DONES).any())
        for buf in ALL_BUFFERS:
            assert (read_buffer(a, buf) == read_buffer(b, buf)).all(), (step, buf)
    assert saw_done
    a.close()
    b.close()
