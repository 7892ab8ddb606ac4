"""carl_b200's no-allocation tick entry point, carlb_ticks_static_scratch.

Some callers cannot allocate device memory while they step: a control loop
with a latency budget, where cudaMalloc and cudaFree can stall the whole
device, or a process whose device memory belongs to another allocator (a
framework's caching pool), where a new cudaMalloc can fail.  For them the
stage scratch is a fixed 64 MiB file-scope device array, set up when the env is
created.  These tests call that entry point through the C ABI and check that:

* two envs of different sizes, whose calls are enqueued back to back on their
  own streams and so share the one array, each give the same state as
  carlb_ticks, on two calls in a row (the library orders the calls on the
  device, and nothing one call leaves in the array leaks into the next);
* the device's free memory is the same before and after those calls;
* an env that needs more scratch than the array holds is rejected before
  anything runs;
* the caller's current device is unchanged.

This file is collected last, so a run that stops at the first failure has run
every other test before it.
"""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads

pytestmark = pytest.mark.gpu


def _controls(rng, env, torch):
    return torch.from_numpy(workloads.controls(rng, env.n_sim * env.n_cars).view(np.int32)).cuda()


def test_static_scratch_ticks_equal_ticks_across_envs():
    import torch

    # Two envs of different sizes share the one array; each is checked against
    # carlb_ticks on the same state and controls.
    envs = [capi.Env(4096, 3, 3, 21), capi.Env(1024, 2, 2, 31)]
    workloads.mixed_state(envs[0], 22)
    workloads.crowd_state(envs[1], 32)
    rng = np.random.default_rng(23)
    ctls = [[_controls(rng, e, torch) for e in envs] for _ in range(2)]
    torch.cuda.synchronize()
    for call in range(2):
        expected = []
        for e, ctl in zip(envs, ctls[call]):
            s0 = e.snapshot()
            e.ticks(capi.ACTIONS_DIRECT, ctl, 8)
            expected.append(e.snapshot())
            e.restore(s0)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        for e, ctl in zip(envs, ctls[call]):
            e.ticks_static_scratch(capi.ACTIONS_DIRECT, ctl, 8)
        for e in envs:
            e.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        assert free_after == free_before, f"call {call}: free device memory {free_before} -> {free_after}"
        for k, (e, want) in enumerate(zip(envs, expected)):
            got = e.snapshot()
            for name in want:
                assert (got[name] == want[name]).all(), (call, k, name)
    for e in envs:
        e.close()


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


def test_static_scratch_keeps_the_callers_device():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two devices")
    env = capi.Env(64, 1, 1, 3, device=1)
    env.reset()
    ctl = torch.zeros((128, 8), dtype=torch.int32, device="cuda:1")
    torch.cuda.set_device(0)
    env.ticks_static_scratch(capi.ACTIONS_DIRECT, ctl, 1)
    env.synchronize()
    assert torch.cuda.current_device() == 0
    env.close()
