"""carlb_ticks_static_scratch, the tick entry point for callers that must not
allocate device memory while they step (a latency-bound control loop, where
cudaMalloc can stall the device, or a process whose device memory belongs to
another allocator, where it can fail).  Its stage scratch is a fixed 64 MiB
file-scope device array.  Two calls in a row give the same state as
carlb_ticks, and an env that needs more scratch than the array holds is
rejected.  This file is collected last, so a run that stops at the first
failure has run every other test before it."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads

pytestmark = pytest.mark.gpu


def test_static_scratch_ticks_equal_ticks():
    import torch

    n_sim, nb, no = 4096, 3, 3
    a = capi.Env(n_sim, nb, no, 21)
    b = capi.Env(n_sim, nb, no, 21)
    workloads.mixed_state(a, 22)
    b.restore(a.snapshot())
    rng = np.random.default_rng(23)
    for call in range(2):
        ctl = torch.from_numpy(workloads.controls(rng, n_sim * (nb + no)).view(np.int32)).cuda()
        a.ticks(capi.ACTIONS_DIRECT, ctl, 8)
        b.ticks_static_scratch(capi.ACTIONS_DIRECT, ctl, 8)
        sa, sb = a.snapshot(), b.snapshot()
        for name in sa:
            assert (sa[name] == sb[name]).all(), (call, name)
    a.close()
    b.close()


def test_static_scratch_rejects_oversized_env():
    import torch

    n_sim, nb, no = 65536, 4, 4  # 524,288 cars: more stage scratch than the 64 MiB array
    env = capi.Env(n_sim, nb, no, 0)
    before = env.read_field("CAR_POS")
    ctl = torch.zeros((n_sim * (nb + no), 8), dtype=torch.int32, device="cuda")
    with pytest.raises(capi.CarlbError, match="static scratch") as exc:
        env.ticks_static_scratch(capi.ACTIONS_DIRECT, ctl, 1)
    assert exc.value.status == capi.ERR_VALUE
    assert (env.read_field("CAR_POS") == before).all()
    env.close()
