"""The product's tick physics, compiled for the host and stepped in the fused
kernel's stage order, against the reference's tick compiled for the host.

Both run the same fp32 operations in the same order (no contraction, correctly
rounded libm on both sides), so every persistent word must agree bit for bit,
the broadphase candidate lists must be identical and the car-vs-mesh SAT pair
sets must be equal as sets.  This pins the physics restatement independently
of device intrinsics.
"""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import workloads
from host_tick_lib import HostTick
import parity

SCENARIOS = [
    ("1v1-floor", 32, 1, 1, "floor", 1),
    ("3v3-floor", 32, 3, 3, "floor", 2),
    ("2v2-mixed", 48, 2, 2, "mixed", 3),
    ("3v3-crowd", 32, 3, 3, "crowd", 4),
    ("4v4-crowd", 16, 4, 4, "crowd", 5),
]


def warm_snapshot(n_sim, nb, no, scenario, seed, warm=8):
    """Scenario state advanced `warm` ticks by the reference (so internal
    state, lagged suspension values and contacts are populated)."""
    from oracle.refenv import RefCpu

    ref = RefCpu(n_sim, nb, no, seed)
    getattr(workloads, scenario + "_state")(ref, seed)
    rng = np.random.default_rng(seed + 1)
    ctl = workloads.controls(rng, n_sim * (nb + no))
    ref.ticks(2, ctl, warm)
    snap = ref.snapshot()
    ref.close()
    return snap


@pytest.mark.parametrize("name, n_sim, nb, no, scenario, seed", SCENARIOS, ids=[s[0] for s in SCENARIOS])
def test_host_tick_matches_reference_bitwise(oracle_built, arena_path, name, n_sim, nb, no, scenario, seed):
    from oracle.refenv import RefCpu

    s0 = warm_snapshot(n_sim, nb, no, scenario, seed)
    ctl = workloads.controls(np.random.default_rng(seed + 99), n_sim * (nb + no))
    ours = HostTick(arena_path, n_sim, nb, no, seed)
    ref = RefCpu(n_sim, nb, no, seed)
    ours.restore(s0)
    ref.restore(s0)
    done = 0
    for k in (1, 8):
        ours.ticks(ctl, k - done)
        ref.ticks(2, ctl, k - done)
        done = k
        a, b = ours.snapshot(), ref.snapshot()
        for f in ("DIAG_CELL_IDX", "DIAG_NUM_TRIS"):
            a[f], b[f] = ours.read_field(f), ref.read_field(f)
        bad = {n: int((a[n] != b[n]).sum()) for n in a if (a[n] != b[n]).any()}
        assert not bad, f"{name} tick {k}: words differ {bad}"
        sat = parity.compare_sat_pairs(ours.read_field("DIAG_SAT_PAIRS"), ref.read_field("DIAG_SAT_PAIRS"))
        assert sat.size == 0, f"{name} tick {k}: SAT pair sets differ for cars {sat[:8]}"
    ours.close()
    ref.close()


def test_direct_controls_pass_through(oracle_built, arena_path):
    """Direct controls reach the car unchanged (reference tests/direct_controls.cu:37-80):
    after 8 ticks the stored controls equal the inputs and positions are finite."""
    inputs = np.zeros((2, 8), dtype=np.uint32)
    inputs[0, :5] = np.array([1.0, 0.5, -0.75, 0.25, -0.5], np.float32).view(np.uint32)
    inputs[0, 5:] = [0, 1, 0]
    inputs[1, :5] = np.array([-1.0, -0.25, 0.5, -0.5, 0.75], np.float32).view(np.uint32)
    inputs[1, 5:] = [1, 0, 1]
    from oracle.refenv import RefCpu

    ref = RefCpu(1, 1, 1, 42)
    ours = HostTick(arena_path, 1, 1, 1, 42)
    ours.restore(ref.snapshot())
    ours.ticks(inputs, 8)
    ref.ticks(2, inputs, 8)
    for impl in (ours, ref):
        assert (impl.read_field("CAR_CONTROLS") == inputs).all()
        assert np.isfinite(impl.read_field("CAR_POS").view(np.float32)).all()
    assert (ours.read_field("CAR_POS") == ref.read_field("CAR_POS")).all()
