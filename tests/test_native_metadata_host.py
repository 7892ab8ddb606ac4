"""The native mesh metadata loader (carl_b200/csrc/arena.cpp, format and
messages of src/ArenaMesh.cu:69-99) on the host: the reference's error
messages, and ball-cell lists re-sorted by the traversal key mesh * 10000 +
order with the same triangles in every cell."""

from __future__ import annotations

import numpy as np
import pytest

from host_tick_lib import HostTick


@pytest.fixture
def host(arena_path):
    h = HostTick(arena_path, 1, 1, 1)
    yield h
    h.close()


def test_metadata_errors(host, tmp_path):
    nt = len(host.arena_tables()["tris"])
    bad = tmp_path / "count.txt"
    bad.write_text("3\n")
    with pytest.raises(RuntimeError, match="CARL arena metadata triangle count mismatch"):
        host.load_metadata(bad)
    short = tmp_path / "short.txt"
    short.write_text(f"{nt}\n" + "0 0 0 0 0 0 0 0 0 0 0 0 0 0 0\n" * 3)
    with pytest.raises(RuntimeError, match="Invalid CARL arena metadata"):
        host.load_metadata(short)
    with pytest.raises(RuntimeError, match="cannot open"):
        host.load_metadata(tmp_path / "missing.txt")


def test_ball_lists_follow_traversal_key(host, tmp_path):
    tables = host.arena_tables()
    nt = len(tables["tris"])
    _, _, _, start0, tris0 = host.ball_grid()
    rng = np.random.default_rng(3)
    mesh = rng.integers(-1, 16, nt)
    order = rng.permutation(nt)
    verts = tables["verts"][tables["tris"]] * np.float32(0.02)
    path = tmp_path / "meta.txt"
    with open(path, "w") as f:
        f.write(f"{nt}\n")
        for t in range(nt):
            f.write(f"{mesh[t]} {order[t]} 0.5 -0.5 6.3 {t % 64} " + " ".join("%.9g" % x for x in verts[t].reshape(-1))
                    + "\n")
    host.load_metadata(path)
    _, _, _, start1, tris1 = host.ball_grid()
    assert (start0 == start1).all()
    key = mesh.astype(np.int64) * 10000 + order
    for c in range(len(start0) - 1):
        a, b = start0[c], start0[c + 1]
        if b - a < 2:
            continue
        cell0, cell1 = tris0[a:b], tris1[a:b]
        assert sorted(cell0.tolist()) == sorted(cell1.tolist())
        k = key[cell1]
        assert (np.diff(k) >= 0).all(), c
