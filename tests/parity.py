"""Field-by-field comparison of snapshots from two implementations.

Tolerance: fp32 values agree within 1e-4 relative or
1e-3 absolute (uu, uu/s, rad/s, ...); integer words must be equal.
TEST INFRASTRUCTURE.
"""

from __future__ import annotations

import numpy as np

from carl_b200 import capi

REL_TOL = 1e-4
ABS_TOL = 1e-3

# Fields that depend on the order the reference's SAT kernel wins atomicAdd
# slots (set semantics) or that it leaves uninitialised until first written.
ORDER_FREE = {"DIAG_SAT_PAIRS"}


def words_to_values(name: str, words: np.ndarray):
    kinds = capi.field_kinds(name, words.shape[1])
    f = words.view(np.float32)
    i = words.view(np.int32)
    is_int = np.array([k == "i" for k in kinds])
    return f, i, is_int


def compare_field(name: str, a: np.ndarray, b: np.ndarray) -> dict:
    """Returns counts of exact / within-tolerance / failing words and rows."""
    assert a.shape == b.shape, (name, a.shape, b.shape)
    fa, ia, is_int = words_to_values(name, a)
    fb, ib, _ = words_to_values(name, b)
    exact = a == b
    ok = exact.copy()
    if (~is_int).any():
        x, y = fa[:, ~is_int].astype(np.float64), fb[:, ~is_int].astype(np.float64)
        close = np.abs(x - y) <= np.maximum(ABS_TOL, REL_TOL * np.maximum(np.abs(x), np.abs(y)))
        close |= np.isnan(x) & np.isnan(y)
        ok[:, ~is_int] |= close
    bad_rows = np.where(~ok.all(axis=1))[0]
    err = 0.0
    if (~is_int).any():
        d = np.abs(fa[:, ~is_int].astype(np.float64) - fb[:, ~is_int].astype(np.float64))
        d = d[np.isfinite(d)]
        err = float(d.max()) if d.size else 0.0
    return {"words": a.size, "rows": a.shape[0], "exact": int(exact.sum()), "ok": int(ok.sum()), "bad_rows": bad_rows,
            "max_abs": err}


SAT_CAP = 32  # pair slots per car (include/RLConstants.cuh MAX_CAR_TRI_PAIRS)


def compare_sat_pairs(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Rows whose SAT pair sets differ (order within a row is free).

    Word 0 of a row is the hit count (at most SAT_CAP), the rest the triangle
    ids.  A car with SAT_CAP or more hits keeps, in the reference's CUDA build,
    the pairs that won its atomicAdd slots (include/Physics/CarArena/
    SAT.cuh:149-150), so for full rows only the counts are compared."""
    ia, ib = a.view(np.int32), b.view(np.int32)
    na, nb = ia[:, 0], ib[:, 0]
    bad = na != nb
    width = ia.shape[1] - 1
    k = np.minimum(np.minimum(na, nb), width)
    cols = np.arange(width)[None, :]
    valid = cols < k[:, None]
    big = np.iinfo(np.int32).max
    sa = np.sort(np.where(valid, ia[:, 1:], big), axis=1)
    sb = np.sort(np.where(valid, ib[:, 1:], big), axis=1)
    sets_differ = (sa != sb).any(axis=1)
    capped = (na >= SAT_CAP) & (nb >= SAT_CAP)
    bad |= sets_differ & ~capped
    return np.where(bad)[0].astype(np.int64)


# The ball's cached integration state is dead while BALL_INT_VALID is 0 (the
# next tick rebuilds it from the exported pose, include/Physics/BallArena/
# Solve.cuh:68-76); the reference leaves it uninitialised until then.
BALL_CACHE = ("BALL_INT_POS", "BALL_INT_VEL", "BALL_EXP_POS", "BALL_EXP_VEL")


def _mask_dead_ball_cache(a: dict, b: dict) -> tuple[dict, dict]:
    if "BALL_INT_VALID" not in a or "BALL_INT_VALID" not in b:
        return a, b
    dead = (a["BALL_INT_VALID"][:, 0] == 0) & (b["BALL_INT_VALID"][:, 0] == 0)
    if not dead.any():
        return a, b
    a, b = dict(a), dict(b)
    for name in BALL_CACHE:
        if name in a and name in b:
            a[name], b[name] = a[name].copy(), b[name].copy()
            a[name][dead] = 0
            b[name][dead] = 0
    return a, b


def _mask_dead_manifold_normal(a: dict, b: dict) -> tuple[dict, dict]:
    """The manifold's first world normal is read only while the car's manifold
    count is non-zero (include/Physics/CarSuspension.cuh:234-265); resets set
    the count to 0 and leave the normal, which the reference's CUDA build
    allocates without clearing (include/Cuda/DeviceArray.cuh:8-12)."""
    if "MAN_COUNT" not in a or "MAN_COUNT" not in b or "MAN_NORMAL0" not in a or "MAN_NORMAL0" not in b:
        return a, b
    dead = (a["MAN_COUNT"][:, 0] == 0) & (b["MAN_COUNT"][:, 0] == 0)
    if not dead.any():
        return a, b
    a, b = dict(a), dict(b)
    a["MAN_NORMAL0"], b["MAN_NORMAL0"] = a["MAN_NORMAL0"].copy(), b["MAN_NORMAL0"].copy()
    a["MAN_NORMAL0"][dead] = 0
    b["MAN_NORMAL0"][dead] = 0
    return a, b


def compare_snapshots(a: dict, b: dict, fields=None) -> dict:
    fields = fields or [f for f in a if f in b]
    a, b = _mask_dead_ball_cache(a, b)
    a, b = _mask_dead_manifold_normal(a, b)
    return {name: compare_field(name, a[name], b[name]) for name in fields}


def summarize(report: dict) -> str:
    lines = []
    for name, r in report.items():
        flag = "" if r["ok"] == r["words"] else "  <-- %d rows" % len(r["bad_rows"])
        lines.append("%-26s exact %6.2f%%  ok %7.3f%%  max|d| %.3g%s" % (
            name, 100.0 * r["exact"] / max(1, r["words"]), 100.0 * r["ok"] / max(1, r["words"]), r["max_abs"], flag))
    return "\n".join(lines)


def all_ok(report: dict) -> bool:
    return all(r["ok"] == r["words"] for r in report.values())


def bad_row_fraction(report: dict, rows: int) -> float:
    """Share of the `rows` records (cars or sims) with any word outside tolerance,
    over every field that has one row per record."""
    bad = set()
    for r in report.values():
        if r["rows"] == rows:
            bad.update(r["bad_rows"].tolist())
    return len(bad) / rows
