"""The boost-pad geometry the device finish stage relies on.

The finish kernel finds, for each car, the one pad whose pickup cylinder holds
it, and then settles every (sim, pad) pair independently.  That equals the
reference's pad-by-pad loop (include/Physics/BoostPads.cuh:70-106) because the
pads' pickup disks are pairwise disjoint: no car is on two pads in one tick.
It looks pads up in 512 uu cells (carl_b200/csrc/tables.cpp); every pad that
can hold a car in a cell must be listed for it, at most 4 per cell.
"""

from __future__ import annotations

import itertools
import math

import numpy as np

import carl_b200

BIG_RADIUS, SMALL_RADIUS = 208.0, 144.0  # cb_consts.cuh BIG_PAD_RADIUS / SMALL_PAD_RADIUS
CELL, NX, NY, X0, Y0 = 512, 16, 20, -4096.0, -5120.0


def _pads():
    pos = np.array(carl_b200.BOOST_PAD_POSITIONS, dtype=np.float64)
    big = pos[:, 2] > 72.0  # the six big pads sit at z = 73, the small ones at z = 70
    assert big.sum() == 6
    return pos, np.where(big, BIG_RADIUS, SMALL_RADIUS)


def test_pickup_disks_are_disjoint():
    pos, rad = _pads()
    gaps = [math.hypot(*(pos[a, :2] - pos[b, :2])) - rad[a] - rad[b]
            for a, b in itertools.combinations(range(len(pos)), 2)]
    assert min(gaps) > 0, min(gaps)


def test_cell_lists_cover_every_pad_reaching_a_cell():
    pos, rad = _pads()
    rng = np.random.default_rng(0)
    pts = np.stack([rng.uniform(-4200, 4200, 200000), rng.uniform(-5200, 5200, 200000)], axis=1)
    for cx in range(NX):
        for cy in range(NY):
            x0, y0 = X0 + cx * CELL, Y0 + cy * CELL
            dx = np.maximum.reduce([x0 - pos[:, 0], np.zeros(len(pos)), pos[:, 0] - x0 - CELL])
            dy = np.maximum.reduce([y0 - pos[:, 1], np.zeros(len(pos)), pos[:, 1] - y0 - CELL])
            listed = set(np.where(dx * dx + dy * dy < (rad + 2.0) ** 2)[0].tolist())
            assert len(listed) <= 4
            inside = pts[(pts[:, 0] >= x0) & (pts[:, 0] < x0 + CELL) & (pts[:, 1] >= y0) & (pts[:, 1] < y0 + CELL)]
            if not len(inside):
                continue
            d2 = ((inside[:, None, :] - pos[None, :, :2]) ** 2).sum(axis=2)
            hit = set(np.where((d2 < rad[None, :] ** 2).any(axis=0))[0].tolist())
            assert hit <= listed, (cx, cy, hit - listed)
