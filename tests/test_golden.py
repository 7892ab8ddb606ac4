"""Golden vectors recorded from the reference (tests/golden/make_golden.py):
the oracle and the product's host build must reproduce them, and the plain-C
restatement of the index paths must reproduce the arena tables, the kickoff
table and rows, and the broadphase cells."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from carl_b200 import capi
from host_tick_lib import HostTick
import parity

GOLDEN = Path(__file__).resolve().parent / "golden"
TICK_CASES = sorted(p.stem[len("tick_"):] for p in GOLDEN.glob("tick_*.npz"))


def load_tick(name):
    z = np.load(GOLDEN / f"tick_{name}.npz")
    n_sim, nb, no, seed = (int(x) for x in z["dims"])
    snaps = {tag: {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(tag + "/")} for tag in ("s0", "s1", "s8", "d1")}
    return (n_sim, nb, no, seed), z["controls"], snaps


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def assert_snap_equal(a: dict, b: dict, what: str):
    bad = {n: int((a[n] != b[n]).sum()) for n in b if n in a and (a[n] != b[n]).any()}
    assert not bad, f"{what}: words differ {bad}"


@pytest.mark.parametrize("name", TICK_CASES)
def test_oracle_reproduces_golden_ticks(oracle_built, name):
    from oracle.refenv import RefCpu

    (n_sim, nb, no, seed), ctl, g = load_tick(name)
    ref = RefCpu(n_sim, nb, no, seed)
    ref.restore(g["s0"])
    ref.ticks(capi.ACTIONS_DIRECT, ctl, 1)
    assert_snap_equal(ref.snapshot(), g["s1"], f"oracle {name} tick 1")
    ref.ticks(capi.ACTIONS_DIRECT, ctl, 7)
    assert_snap_equal(ref.snapshot(), g["s8"], f"oracle {name} tick 8")
    ref.close()


@pytest.mark.parametrize("name", TICK_CASES)
def test_product_host_build_reproduces_golden_ticks(arena_path, name):
    (n_sim, nb, no, seed), ctl, g = load_tick(name)
    ours = HostTick(arena_path, n_sim, nb, no, seed)
    ours.restore(g["s0"])
    ours.ticks(ctl, 1)
    assert_snap_equal(ours.snapshot(), g["s1"], f"host build {name} tick 1")
    for f in ("DIAG_CELL_IDX", "DIAG_NUM_TRIS"):
        assert (ours.read_field(f) == g["d1"][f]).all(), f
    assert parity.compare_sat_pairs(ours.read_field("DIAG_SAT_PAIRS"), g["d1"]["DIAG_SAT_PAIRS"]).size == 0
    ours.ticks(ctl, 7)
    assert_snap_equal(ours.snapshot(), g["s8"], f"host build {name} tick 8")
    ours.close()


def test_c_restatement_arena_tables(arena_path):
    from oracle import port

    golden = json.loads((GOLDEN / "arena.json").read_text())
    t = port.arena(arena_path)
    for k in ("verts", "tris", "prefix", "tri_idx"):
        assert list(t[k].shape) == golden[k]["shape"], k
        assert sha(t[k]) == golden[k]["sha256"], k


def test_product_arena_tables(arena_path):
    golden = json.loads((GOLDEN / "arena.json").read_text())
    ht = HostTick(arena_path, 1, 1, 1, 0)
    t = ht.arena_tables()
    kick = ht.kickoff_table()
    ht.close()
    for k in ("verts", "tris", "prefix", "tri_idx", "edge_angles"):
        assert list(t[k].shape) == golden[k]["shape"], k
        assert sha(t[k]) == golden[k]["sha256"], k
    # Default arena (no native metadata): the ball walks the car's per-cell lists.
    assert golden["ball_tri_idx"]["sha256"] == golden["tri_idx"]["sha256"]
    z = np.load(GOLDEN / "kickoff_4v4.npz")
    assert (kick == z["table"]).all()


def test_c_restatement_kickoff_table():
    from oracle import port

    z = np.load(GOLDEN / "kickoff_4v4.npz")
    assert (port.kickoff_table() == z["table"]).all()


def test_c_restatement_kickoff_rows():
    """Car k of the blue team starts on spot table[row][k]; the row is
    hash32(hash32(seed) ^ hash32(sim) ^ hash32(tick)) % 120 (include/State/Reset.cuh:52-63)."""
    from oracle import port

    z = np.load(GOLDEN / "kickoff_4v4.npz")
    seed, table = int(z["seed"]), z["table"]
    pos = z["car_pos"].view(np.float32).reshape(-1, 8, 3)
    spot_pos: dict[int, tuple] = {}
    for sim in range(pos.shape[0]):
        row = port.kickoff_row(seed, sim, 0)
        for k in range(4):
            key = tuple(pos[sim, k].tolist())
            spot = int(table[row, k])
            assert spot_pos.setdefault(spot, key) == key, (sim, k, spot)
    assert len(spot_pos) == 5 and len(set(spot_pos.values())) == 5


def test_hash32_known_values():
    from oracle import port

    # hash32 is a bijection on 32-bit words; spot-check avalanche and fixed points.
    assert port.hash32(0) == 0
    vals = {port.hash32(v) for v in range(4096)}
    assert len(vals) == 4096


@pytest.mark.parametrize("name", TICK_CASES)
def test_c_restatement_broadphase_cells(name):
    from oracle import port

    (n_sim, nb, no, seed), ctl, g = load_tick(name)
    s0 = g["s0"]
    f = lambda k: s0[k].view(np.float32)
    cells = port.broadphase_cells(f("CAR_POS"), f("CAR_VEL"), f("CAR_ANG"), f("CAR_CEN"), f("CAR_ROT"))
    ref = g["d1"]["DIAG_CELL_IDX"].view(np.int32)[:, 0]
    live = s0["CAR_IS_DEMOED"].view(np.int32)[:, 0] == 0
    assert (cells[live] == ref[live]).all()
