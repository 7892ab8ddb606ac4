"""The ball grid used by the device's ball-arena stage: the cell holding a ball
centre lists every triangle that ball can touch (distance below the contact
radius), checked against a brute-force distance over all triangles for seeded
points near the arena surfaces.  The reference gathers from the 48x48x10 car
grid cells around the ball instead; any complete candidate set walked in
ascending triangle order gives the same contacts."""

from __future__ import annotations

import numpy as np

from host_tick_lib import HostTick

CONTACT_RADIUS = 91.25 + 1.905


def closest_point_dist(p, a, b, c):
    """Distance from points p [n,3] to triangles (a, b, c) [m,3] -> [n, m] (float64)."""
    ab, ac = b - a, c - a
    n = np.cross(ab, ac)
    n /= np.linalg.norm(n, axis=1, keepdims=True)
    out = np.empty((p.shape[0], a.shape[0]))
    for i, q in enumerate(p):
        # Project onto the plane, clamp to the triangle via edge distances.
        d_plane = np.einsum("mk,mk->m", q - a, n)
        proj = q - d_plane[:, None] * n
        def inside(u, v, w):
            return np.einsum("mk,mk->m", np.cross(v - u, proj - u), n) >= 0
        ins = inside(a, b, c) & inside(b, c, a) & inside(c, a, b)
        def seg(u, v):
            t = np.clip(np.einsum("mk,mk->m", q - u, v - u) / np.einsum("mk,mk->m", v - u, v - u), 0, 1)
            return np.linalg.norm(q - (u + t[:, None] * (v - u)), axis=1)
        edge = np.minimum(np.minimum(seg(a, b), seg(b, c)), seg(c, a))
        out[i] = np.where(ins, np.abs(d_plane), edge)
    return out


def test_ball_cells_cover_every_touchable_triangle(arena_path):
    ht = HostTick(arena_path, 1, 1, 1, 0)
    origin, cell, dims, start, tris = ht.ball_grid()
    A = ht.arena_tables()
    ht.close()
    v = A["verts"].astype(np.float64)[A["tris"]]
    a, b, c = v[:, 0], v[:, 1], v[:, 2]
    rng = np.random.default_rng(5)
    # Points near surfaces: jitter random triangle points by up to the contact radius.
    pick = rng.integers(0, a.shape[0], 400)
    w = rng.dirichlet([1, 1, 1], 400)
    pts = w[:, :1] * a[pick] + w[:, 1:2] * b[pick] + w[:, 2:] * c[pick]
    pts += rng.normal(0, 40, pts.shape)
    d = closest_point_dist(pts, a, b, c)
    for i, q in enumerate(pts.astype(np.float32)):
        f = (q - origin) / np.float32(cell)
        near = set(np.nonzero(d[i] < CONTACT_RADIUS + 0.5)[0].tolist())
        if not ((f >= 0).all() and (f < dims).all()):
            assert not near, (q, sorted(near)[:5])
            continue
        ci = int(f[0]) + int(dims[0]) * (int(f[1]) + int(dims[1]) * int(f[2]))
        listed = tris[start[ci]:start[ci + 1]]
        assert (np.diff(listed) > 0).all()
        missing = near - set(listed.tolist())
        assert not missing, (q, sorted(missing)[:5])
