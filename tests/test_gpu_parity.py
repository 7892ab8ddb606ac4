"""Parity of the sm_100a staged tick with the reference.

Two oracles (both built from the reference's own sources):
  * RefGpu: the reference's CUDA build for sm_100a.  The product's default mode
    (compat_flags = 0) reproduces what that build computes, including its
    compiled read of the current tick's lateral friction coefficient (the
    source intends the previous tick's value).  This is the mode the benchmark
    runs, and it is held to the strict gates below at small sizes and at the
    benchmark's full size.
  * RefCpu: the reference's tick compiled for the host, which follows the
    source semantics.  The product's SOURCE_LAGGED_LATERAL_FRICTION mode follows
    the same semantics; the remaining differences come from device intrinsics
    (rsqrtf, __sincosf) that the reference's own CUDA build has too.

Gates of the default mode against RefGpu: broadphase cells, candidate counts
and SAT pair sets bit-exact; single-tick fp32 state within 1e-4 relative or
1e-3 absolute and integer words exact, for every sim row and every car row
except cars whose SAT pairs the reference's CUDA build offers to its manifold
in run-dependent order (it fills the pair slots with atomicAdd,
include/Physics/CarArena/SAT.cuh:149-150, so of two equally deep mesh contacts
either may be kept).  8-tick rollouts: a stated drift bound on the car rows
that leave that tolerance (contacts are chaotic: one ulp in a contact normal
can flip a discrete event such as a wheel touching down).
"""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads
import parity

pytestmark = pytest.mark.gpu

SCENARIOS = [
    ("1v1-floor", 64, 1, 1, "floor", 1),
    ("3v3-floor", 256, 3, 3, "floor", 2),
    ("2v2-mixed", 256, 2, 2, "mixed", 3),
    ("3v3-crowd", 256, 3, 3, "crowd", 4),
    ("4v4-crowd", 128, 4, 4, "crowd", 5),
]
IDS = [s[0] for s in SCENARIOS]

# Share of car rows allowed outside the single-tick tolerance after 8 ticks
# (the stated drift bound).  Default mode against the reference CUDA build:
# 2 % (measured 0 % on every scenario but 3v3 floor).  Source mode against the
# host build: dense car-car play (crowd) amplifies last-ulp differences through
# discrete contact events; measured 4v4 crowd 15.6 %, 3v3 crowd about 10 %.
DRIFT_ROWS_8 = 0.02
DRIFT_ROWS_8_CROWD = 0.25
# SOURCE_LAGGED_LATERAL_FRICTION mode against the host build only (not the
# benchmarked mode): share of car rows allowed outside the single-tick
# tolerance (device rsqrtf/__sincosf versus host libm; measured 0 % floor and
# mixed, 1.0-1.5 % crowd) and share of cars in another broadphase cell.
SINGLE_TICK_ROWS_HOST = 0.02
CELLS_HOST = 0.005


def _torch():
    import torch

    return torch


def warm_snapshot(n_sim, nb, no, scenario, seed, warm=16):
    from oracle.refenv import RefCpu

    ref = RefCpu(n_sim, nb, no, seed)
    getattr(workloads, scenario + "_state")(ref, seed)
    rng = np.random.default_rng(seed + 1)
    for t in range(warm):
        if t % 8 == 0:
            ctl = workloads.controls(rng, n_sim * (nb + no))
        ref.ticks(2, ctl, 1)
    snap = ref.snapshot()
    ref.close()
    return snap


def run_pair(n_sim, nb, no, seed, s0, ctl, compat, ref_cls, ticks):
    torch = _torch()
    env = capi.Env(n_sim, nb, no, seed, compat_flags=compat)
    env.set_diagnostics(True)
    env.restore(s0)
    ref = ref_cls(n_sim, nb, no, seed)
    ref.restore(s0)
    d = torch.from_numpy(ctl.view(np.int32)).cuda()
    out = []
    done = 0
    for k in ticks:
        env.ticks(capi.ACTIONS_DIRECT, d, k - done)
        env.synchronize()
        ref.ticks(capi.ACTIONS_DIRECT, ctl, k - done)
        done = k
        a, b = env.snapshot(), ref.snapshot()
        diag = {f: (env.read_field(f), ref.read_field(f)) for f in ("DIAG_CELL_IDX", "DIAG_NUM_TRIS", "DIAG_SAT_PAIRS")}
        out.append((k, a, b, diag))
    env.close()
    ref.close()
    return out


def car_rows_bad(rep: dict, n_cars_total: int) -> float:
    return parity.bad_row_fraction(rep, n_cars_total)


def check_tick1_against_cuda_build(name, n_sim, n_cars, a, b, diag):
    """The single-tick gates of the default mode (see the module docstring)."""
    rows = n_sim * n_cars
    rep = parity.compare_snapshots(a, b)
    assert (diag["DIAG_CELL_IDX"][0] == diag["DIAG_CELL_IDX"][1]).all(), f"{name}: broadphase cells differ"
    assert (diag["DIAG_NUM_TRIS"][0] == diag["DIAG_NUM_TRIS"][1]).all(), f"{name}: candidate counts differ"
    sat_bad = parity.compare_sat_pairs(*diag["DIAG_SAT_PAIRS"])
    assert sat_bad.size == 0, f"{name}: SAT pair sets differ on car rows {sat_bad[:10].tolist()}"
    bad = set()
    for r in rep.values():
        if r["rows"] == rows:
            bad.update(r["bad_rows"].tolist())
    pairs = diag["DIAG_SAT_PAIRS"][1].view(np.int32)[:, 0]
    unexplained = sorted(row for row in bad if pairs[row] < 2)
    assert not unexplained, f"{name} tick 1 car rows {unexplained[:10]}\n" + parity.summarize(rep)
    # Rows with two or more SAT pairs may keep another, equally deep contact in
    # the reference; they stay rare (measured 0 or 1 per scenario).
    assert len(bad) <= max(1, rows // 1000), parity.summarize(rep)
    sims_ok = {k: r for k, r in rep.items() if r["rows"] == n_sim and n_sim != rows}
    assert parity.all_ok(sims_ok), parity.summarize(sims_ok)
    return len(bad)


@pytest.mark.parametrize("name, n_sim, nb, no, scenario, seed", SCENARIOS, ids=IDS)
def test_default_matches_reference_cuda_build(oracle_built, name, n_sim, nb, no, scenario, seed):
    from oracle.refenv import RefGpu

    s0 = warm_snapshot(n_sim, nb, no, scenario, seed)
    ctl = workloads.controls(np.random.default_rng(seed + 99), n_sim * (nb + no))
    results = run_pair(n_sim, nb, no, seed, s0, ctl, 0, RefGpu, (1, 8))
    for k, a, b, diag in results:
        if k == 1:
            check_tick1_against_cuda_build(name, n_sim, nb + no, a, b, diag)
        else:
            frac = car_rows_bad(parity.compare_snapshots(a, b), n_sim * (nb + no))
            print(f"{name}: default mode vs reference CUDA build, 8 ticks: {100 * frac:.2f}% car rows outside tolerance")
            assert frac <= DRIFT_ROWS_8, parity.summarize(parity.compare_snapshots(a, b))


BENCH_WORKLOADS = [
    # name, n_sim, blue, orange, initial state (bench.py initial_state, rank 0)
    ("C3", 32768, 3, 3, "floor"),
    ("C4", 32768, 2, 2, "mixed"),
    ("C1", 1024, 1, 1, "kickoff"),
]


@pytest.mark.parametrize("name, n_sim, nb, no, state", BENCH_WORKLOADS, ids=[w[0] for w in BENCH_WORKLOADS])
def test_bench_size_matches_reference_cuda_build(oracle_built, name, n_sim, nb, no, state):
    """A benchmark workload at its full per-GPU size: bench.py's seeded initial
    states (rank 0) after its 5 warm-up steps of 8 ticks, then 1 and 8 ticks of
    the next control set, default mode against the reference's CUDA build on the
    same states and controls."""
    from oracle.refenv import RefGpu

    seed = 0
    n = n_sim * (nb + no)
    ref = RefGpu(n_sim, nb, no, seed)
    if state == "kickoff":
        ref.reset()
    else:
        (workloads.floor_state if state == "floor" else workloads.mixed_state)(ref, seed)
    rng = np.random.default_rng(seed + 1)
    pool = [workloads.controls(rng, n) for _ in range(6)]
    for i in range(5):
        ref.ticks(capi.ACTIONS_DIRECT, pool[i], 8)
    s0 = ref.snapshot()
    ref.close()
    results = run_pair(n_sim, nb, no, seed, s0, pool[5], 0, RefGpu, (1, 8))
    for k, a, b, diag in results:
        if k == 1:
            nbad = check_tick1_against_cuda_build(f"{name} {n_sim}", n_sim, nb + no, a, b, diag)
            print(f"{name} n_sim={n_sim} tick 1: {nbad} car rows outside tolerance (all with >= 2 SAT pairs)")
        else:
            frac = car_rows_bad(parity.compare_snapshots(a, b), n)
            print(f"{name} n_sim={n_sim}, 8 ticks: {100 * frac:.3f}% car rows outside tolerance")
            assert frac <= DRIFT_ROWS_8, parity.summarize(parity.compare_snapshots(a, b))


@pytest.mark.parametrize("name, n_sim, nb, no, scenario, seed", SCENARIOS, ids=IDS)
def test_source_mode_matches_reference_semantics(oracle_built, name, n_sim, nb, no, scenario, seed):
    """SOURCE_LAGGED_LATERAL_FRICTION mode (the source's one-tick-lagged lateral
    friction; not the default) against the reference's host build.  Device intrinsics separate any CUDA build from a
    host build by a few ulps; in dense car-car play these can flip a discrete
    contact event within a tick."""
    from oracle.refenv import RefCpu

    s0 = warm_snapshot(n_sim, nb, no, scenario, seed)
    ctl = workloads.controls(np.random.default_rng(seed + 77), n_sim * (nb + no))
    results = run_pair(n_sim, nb, no, seed, s0, ctl, capi.SOURCE_LAGGED_LATERAL_FRICTION, RefCpu, (1, 8))
    n = n_sim * (nb + no)
    for k, a, b, diag in results:
        rep = parity.compare_snapshots(a, b)
        frac = car_rows_bad(rep, n)
        print(f"{name}: tick {k}: {100 * frac:.2f}% car rows outside tolerance of the host build")
        if k == 1:
            cells_diff = (diag["DIAG_CELL_IDX"][0] != diag["DIAG_CELL_IDX"][1]).mean()
            assert cells_diff <= CELLS_HOST
            assert frac <= SINGLE_TICK_ROWS_HOST, parity.summarize(rep)
        else:
            bound = DRIFT_ROWS_8_CROWD if scenario == "crowd" else DRIFT_ROWS_8
            assert frac <= bound, parity.summarize(rep)


@pytest.mark.parametrize("case", ["2v2_mixed", "3v3_crowd", "1v1_floor"])
def test_golden_ticks_on_device(case):
    """The committed golden vectors (reference host build, source semantics)
    reproduced by the kernel in SOURCE_LAGGED_LATERAL_FRICTION mode within the
    single-tick tolerance."""
    from test_golden import load_tick

    torch = _torch()
    (n_sim, nb, no, seed), ctl, g = load_tick(case)
    env = capi.Env(n_sim, nb, no, seed, compat_flags=capi.SOURCE_LAGGED_LATERAL_FRICTION)
    env.set_diagnostics(True)
    env.restore(g["s0"])
    env.ticks(capi.ACTIONS_DIRECT, torch.from_numpy(ctl.view(np.int32)).cuda(), 1)
    env.synchronize()
    rep = parity.compare_snapshots(env.snapshot(), g["s1"])
    assert parity.all_ok(rep), parity.summarize(rep)
    assert (env.read_field("DIAG_NUM_TRIS") == g["d1"]["DIAG_NUM_TRIS"]).all()
    assert parity.compare_sat_pairs(env.read_field("DIAG_SAT_PAIRS"), g["d1"]["DIAG_SAT_PAIRS"]).size == 0
    env.close()


def test_kickoff_reset_matches_golden():
    z = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "kickoff_4v4.npz")
    env = capi.Env(96, 4, 4, int(z["seed"]))
    env.reset()
    assert (env.read_field("CAR_POS") == z["car_pos"]).all()
    # Kickoff yaw quaternions use device sinf/cosf (the golden vectors: host libm).
    rep = parity.compare_field("CAR_ROT", env.read_field("CAR_ROT"), z["car_rot"])
    assert rep["ok"] == rep["words"] and rep["max_abs"] <= 1.2e-7
    env.close()


def test_direct_controls_pass_through_on_device():
    torch = _torch()
    inputs = np.zeros((2, 8), dtype=np.uint32)
    inputs[0, :5] = np.array([1.0, 0.5, -0.75, 0.25, -0.5], np.float32).view(np.uint32)
    inputs[0, 5:] = [0, 1, 0]
    inputs[1, :5] = np.array([-1.0, -0.25, 0.5, -0.5, 0.75], np.float32).view(np.uint32)
    inputs[1, 5:] = [1, 0, 1]
    env = capi.Env(1, 1, 1, 42)
    env.reset()
    d = torch.from_numpy(inputs.view(np.int32)).cuda()
    for _ in range(8):
        env.ticks(capi.ACTIONS_DIRECT, d, 1)
    env.synchronize()
    assert (env.read_field("CAR_CONTROLS") == inputs).all()
    assert np.isfinite(env.read_field("CAR_POS").view(np.float32)).all()
    env.close()
