"""Ball-arena contacts with native mesh metadata (CARL_ARENA_METADATA,
src/ArenaMesh.cu:69-99 and BallArena/Contact.cuh:161-593) against the
reference's CUDA build reading the same file.

The metadata is synthetic (the RLGym meshes it is made from are not available):
the default arena's triangles, in the reference's own triangle order, split into
16 native meshes by region, floor triangles and 2 % of the rest marked as not
collidable (mesh -1), a random traversal order inside each mesh, the arena's
edge angles with some edges made concave, random edge flags, and the vertices
in Bullet units.  Balls are placed moving near the floor, walls, corners and
ceiling, where several meshes meet."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, workloads
import parity

pytestmark = pytest.mark.gpu


def write_metadata(path, tables, seed: int) -> None:
    rng = np.random.default_rng(seed)
    verts, tris, angles = tables["verts"], tables["tris"], tables["edge_angles"].copy()
    nt = len(tris)
    tv = verts[tris]                                   # [nt, 3, 3]
    cen = tv.mean(axis=1)
    mesh = ((np.floor((cen[:, 0] + 4200) / 2100).astype(int) * 4
             + np.floor((cen[:, 1] + 6100) / 3050).astype(int)) % 16)
    n = np.cross(tv[:, 1] - tv[:, 0], tv[:, 2] - tv[:, 0])
    n /= np.linalg.norm(n, axis=1, keepdims=True)
    floor = (np.abs(n[:, 2]) > 0.999) & (np.abs(cen[:, 2]) < 1.0)
    mesh[floor | (rng.uniform(size=nt) < 0.02)] = -1
    order = np.zeros(nt, np.int64)
    for m in range(-1, 16):
        idx = np.where(mesh == m)[0]
        order[idx] = rng.permutation(idx.size)
    concave = (rng.uniform(size=angles.shape) < 0.05) & (np.abs(angles) < 2 * np.pi - 1e-3)
    angles[concave] = 0.0
    flags = rng.integers(0, 64, nt)
    native = (tv * np.float32(0.02)).astype(np.float32)
    with open(path, "w") as f:
        f.write(f"{nt}\n")
        for t in range(nt):
            vals = " ".join("%.9g" % x for x in native[t].reshape(-1))
            f.write(f"{mesh[t]} {order[t]} {angles[t, 0]:.9g} {angles[t, 1]:.9g} {angles[t, 2]:.9g} {flags[t]} {vals}\n")


def place_balls(snap: dict, n_sim: int, seed: int) -> dict:
    """Balls moving toward the floor, side walls, back-wall corners and ceiling."""
    rng = np.random.default_rng(seed)
    r = 91.25
    kind = rng.integers(0, 5, n_sim)
    pos = np.stack([rng.uniform(-3000, 3000, n_sim), rng.uniform(-4000, 4000, n_sim),
                    rng.uniform(r, r + 40, n_sim)], 1)
    vel = rng.normal(0, 600, (n_sim, 3))
    vel[:, 2] = -np.abs(vel[:, 2]) - 200
    side = kind == 1
    pos[side, 0] = np.sign(rng.uniform(-1, 1, side.sum())) * (4096 - r - rng.uniform(0, 40, side.sum()))
    pos[side, 2] = rng.uniform(300, 1500, side.sum())
    vel[side, 0] = np.sign(pos[side, 0]) * (np.abs(vel[side, 0]) + 300)
    corner = kind == 2
    pos[corner] = np.stack([np.sign(rng.uniform(-1, 1, corner.sum())) * rng.uniform(3700, 3950, corner.sum()),
                            np.sign(rng.uniform(-1, 1, corner.sum())) * rng.uniform(4700, 4950, corner.sum()),
                            rng.uniform(150, 900, corner.sum())], 1)
    top = kind == 3
    pos[top, 2] = 2044 - r - rng.uniform(0, 40, top.sum())
    vel[top, 2] = np.abs(vel[top, 2]) + 200
    goal = kind == 4
    pos[goal] = np.stack([rng.uniform(-1000, 1000, goal.sum()),
                          np.sign(rng.uniform(-1, 1, goal.sum())) * rng.uniform(5000, 5300, goal.sum()),
                          rng.uniform(r, 700, goal.sum())], 1)
    out = dict(snap)
    out["BALL_POS"] = pos.astype(np.float32).view(np.uint32)
    out["BALL_VEL"] = vel.astype(np.float32).view(np.uint32)
    out["BALL_ANG"] = rng.normal(0, 2, (n_sim, 3)).astype(np.float32).view(np.uint32)
    out["BALL_INT_VALID"] = np.zeros_like(snap["BALL_INT_VALID"])
    return out


BALL_FIELDS = ["BALL_POS", "BALL_VEL", "BALL_ANG"]


def ball_rows_bad(rep: dict) -> set:
    bad = set()
    for name in BALL_FIELDS:
        bad.update(rep[name]["bad_rows"].tolist())
    return bad


@pytest.fixture
def metadata(oracle_built, tmp_path, monkeypatch):
    from oracle.refenv import RefCpu, reference_arena_tables

    ref = RefCpu(1, 1, 1, 0)
    tables = reference_arena_tables(ref)
    ref.close()
    path = tmp_path / "arena_metadata.txt"
    write_metadata(path, tables, 7)
    monkeypatch.setenv("CARL_ARENA_METADATA", str(path))
    return path


def test_native_metadata_matches_reference_cuda_build(metadata, monkeypatch):
    import torch

    from oracle.refenv import RefGpu

    n_sim, nb, no, seed = 512, 1, 1, 11
    env = capi.Env(n_sim, nb, no, seed)
    ref = RefGpu(n_sim, nb, no, seed)
    workloads.mixed_state(env, 12)
    s0 = place_balls(env.snapshot(), n_sim, 13)
    env.restore(s0)
    ref.restore(s0)
    rng = np.random.default_rng(14)
    moved = 0
    for tick in range(8):
        ctl = workloads.controls(rng, n_sim * (nb + no))
        env.ticks(capi.ACTIONS_DIRECT, torch.from_numpy(ctl.view(np.int32)).cuda(), 1)
        ref.ticks(capi.ACTIONS_DIRECT, ctl, 1)
        rep = parity.compare_snapshots(env.snapshot(), ref.snapshot())
        bad = ball_rows_bad(rep)
        if tick == 0:
            assert not bad, parity.summarize({k: rep[k] for k in BALL_FIELDS})
        else:
            assert len(bad) <= n_sim // 50, parity.summarize({k: rep[k] for k in BALL_FIELDS})
    env.close()
    ref.close()

    # The native branch is taken: without the metadata the same 8 ticks differ
    # for the balls that met the arena.
    monkeypatch.delenv("CARL_ARENA_METADATA")
    plain = capi.Env(n_sim, nb, no, seed)
    plain.restore(s0)
    monkeypatch.setenv("CARL_ARENA_METADATA", str(metadata))
    native = capi.Env(n_sim, nb, no, seed)
    native.restore(s0)
    ctl = torch.from_numpy(workloads.controls(np.random.default_rng(15), n_sim * 2).view(np.int32)).cuda()
    plain.ticks(capi.ACTIONS_DIRECT, ctl, 8)
    native.ticks(capi.ACTIONS_DIRECT, ctl, 8)
    moved = (plain.read_field("BALL_VEL") != native.read_field("BALL_VEL")).any(axis=1).sum()
    assert moved > n_sim // 4, moved
    plain.close()
    native.close()


def test_metadata_errors(oracle_built, tmp_path, monkeypatch):
    from oracle.refenv import RefCpu, reference_arena_tables

    ref = RefCpu(1, 1, 1, 0)
    nt = len(reference_arena_tables(ref)["tris"])
    ref.close()
    bad_count = tmp_path / "count.txt"
    bad_count.write_text("3\n0 0 0 0 0 0 0 0 0 0 0 0 0 0 0\n")
    monkeypatch.setenv("CARL_ARENA_METADATA", str(bad_count))
    with pytest.raises(capi.CarlbError, match="triangle count mismatch"):
        capi.Env(4, 1, 1, 0)
    truncated = tmp_path / "short.txt"
    truncated.write_text(f"{nt}\n0 0 0 0 0 0 0 0 0 0 0 0 0 0 0\n")
    monkeypatch.setenv("CARL_ARENA_METADATA", str(truncated))
    with pytest.raises(capi.CarlbError, match="Invalid CARL arena metadata"):
        capi.Env(4, 1, 1, 0)
