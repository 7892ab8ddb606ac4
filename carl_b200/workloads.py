"""Seeded synthetic workloads (states and controls) for the benchmark and the tests.

States are written field by field into an env that was reset to kickoff, so
every word of the snapshot is defined.  Vector math that feeds derived fields
(the hitbox centre) is done in float32 with the same operation order as the
device code, so the derived values are exactly what the tick would compute.

Distributions (the benchmark configs; no public dataset is involved):
  floor    positions uniform over the field floor, z = 17, velocity N(0, 800)
           in x/y, yaw uniform, boost U[0, 100], ball at rest at centre
  mixed    50 % airborne (z U[100, 1900]), 25 % against walls / ceiling,
           25 % within 300 uu of corners and goal mouths, random unit
           quaternions, angular velocity N(0, 3); ball moving
  crowd    cars packed around the ball at high speed toward it (car-car
           contacts, bumps, demolitions, ball hits)
Controls are redrawn from a seed: throttle/steer/pitch/yaw/roll U[-1, 1],
jump/boost/handbrake Bernoulli(0.3).
"""

from __future__ import annotations

import numpy as np

F = np.float32
CAR_OFFSET = np.array([13.87566, 0.0, 20.755], dtype=F)


def _cross(a, b):
    return np.stack([a[:, 1] * b[:, 2] - a[:, 2] * b[:, 1],
                     a[:, 2] * b[:, 0] - a[:, 0] * b[:, 2],
                     a[:, 0] * b[:, 1] - a[:, 1] * b[:, 0]], axis=1).astype(F)


def _dot(a, b):
    return ((a[:, 0] * b[:, 0] + a[:, 1] * b[:, 1]) + a[:, 2] * b[:, 2]).astype(F)


def rotate(q: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Quaternion (x, y, z, w) rotation, float32, device operation order."""
    q = q.astype(F)
    v = np.broadcast_to(v.astype(F), (q.shape[0], 3)).copy()
    u = q[:, :3]
    qls = ((q[:, 0] * q[:, 0] + q[:, 2] * q[:, 2]) + (q[:, 1] * q[:, 1] + q[:, 3] * q[:, 3])).astype(F)
    t = _cross(u, v) * (F(2.0) / qls)[:, None]
    return ((v + t * q[:, 3:4]) + _cross(u, t)).astype(F)


def yaw_quat(yaw: np.ndarray) -> np.ndarray:
    h = (yaw.astype(F) / F(2)).astype(F)
    return np.stack([np.zeros_like(h), np.zeros_like(h), np.sin(h), np.cos(h)], axis=1).astype(F)


def random_quat(rng, n):
    q = rng.normal(size=(n, 4)).astype(F)
    q /= np.linalg.norm(q, axis=1, keepdims=True).astype(F)
    return q.astype(F)


def controls(rng, n_cars_total: int) -> np.ndarray:
    """Direct controls: [n, 8] words (5 float32 axes, 3 int32 buttons)."""
    out = np.zeros((n_cars_total, 8), dtype=np.uint32)
    axes = rng.uniform(-1, 1, size=(n_cars_total, 5)).astype(F)
    buttons = (rng.uniform(size=(n_cars_total, 3)) < 0.3).astype(np.int32)
    out[:, :5] = axes.view(np.uint32)
    out[:, 5:] = buttons.view(np.uint32)
    return out


def continuous_actions(rng, n_cars_total: int) -> np.ndarray:
    """Continuous actions [n, 7]: horizontal, vertical, throttle in [-1, 1]; buttons in {0, 1}."""
    a = rng.uniform(-1, 1, size=(n_cars_total, 7)).astype(F)
    a[:, [3, 4, 6]] = (rng.uniform(size=(n_cars_total, 3)) < 0.3).astype(F)
    return a


def discrete_actions(rng, n_cars_total: int) -> np.ndarray:
    nvec = np.array([3, 3, 3, 2, 2, 3, 2])
    return (rng.integers(0, 1 << 30, size=(n_cars_total, 7)) % nvec).astype(np.int32)


def _set_cars(env, pos, rot, vel, ang, boost=None, on_ground=None):
    n = pos.shape[0]
    env.write_field("CAR_POS", pos.astype(F))
    env.write_field("CAR_ROT", rot.astype(F))
    env.write_field("CAR_VEL", vel.astype(F))
    env.write_field("CAR_ANG", ang.astype(F))
    cen = (pos.astype(F) + rotate(rot, CAR_OFFSET)).astype(F)
    env.write_field("CAR_CEN", cen)
    internal = env.read_field("CAR_INTERNAL")
    if boost is not None:
        internal[:, 21] = boost.astype(F).view(np.uint32)
    if on_ground is not None:
        internal[:, 0] = on_ground.astype(np.int32).view(np.uint32)
    env.write_field("CAR_INTERNAL", internal)
    assert n == env.n_sim * env.n_cars


def floor_state(env, seed: int) -> None:
    """Config C3 distribution (floor, random yaw and planar velocity)."""
    rng = np.random.default_rng(seed)
    n = env.n_sim * env.n_cars
    pos = np.stack([rng.uniform(-3900, 3900, n), rng.uniform(-4900, 4900, n), np.full(n, 17.0)], axis=1).astype(F)
    vel = np.concatenate([rng.normal(0, 800, (n, 2)), np.zeros((n, 1))], axis=1).astype(F)
    rot = yaw_quat(rng.uniform(-np.pi, np.pi, n).astype(F))
    _set_cars(env, pos, rot, vel, np.zeros((n, 3), F), boost=rng.uniform(0, 100, n), on_ground=np.ones(n))


def mixed_state(env, seed: int) -> None:
    """Config C4 distribution (air, walls/ceiling, corners/goal mouths)."""
    rng = np.random.default_rng(seed)
    n = env.n_sim * env.n_cars
    kind = rng.uniform(size=n)
    pos = np.zeros((n, 3), F)
    air = kind < 0.5
    wall = (kind >= 0.5) & (kind < 0.75)
    corner = kind >= 0.75
    pos[air] = np.stack([rng.uniform(-3800, 3800, air.sum()), rng.uniform(-4800, 4800, air.sum()),
                         rng.uniform(100, 1900, air.sum())], axis=1)
    # Walls: side walls (x = +-4096) and ceiling (z = 2044), just inside the surface.
    w = np.where(wall)[0]
    side = rng.uniform(size=w.size) < 0.7
    pos[w[side]] = np.stack([np.sign(rng.uniform(-1, 1, side.sum())) * rng.uniform(3990, 4040, side.sum()),
                             rng.uniform(-3500, 3500, side.sum()), rng.uniform(200, 1800, side.sum())], axis=1)
    pos[w[~side]] = np.stack([rng.uniform(-3500, 3500, (~side).sum()), rng.uniform(-4500, 4500, (~side).sum()),
                              rng.uniform(1960, 2010, (~side).sum())], axis=1)
    # Corners and goal mouths.
    c = np.where(corner)[0]
    anchors = np.array([[3900, 4900, 60], [-3900, 4900, 60], [3900, -4900, 60], [-3900, -4900, 60],
                        [0, 5100, 100], [0, -5100, 100], [850, 5050, 300], [-850, -5050, 300]], dtype=F)
    a = anchors[rng.integers(0, len(anchors), c.size)]
    off = rng.normal(0, 1, (c.size, 3)).astype(F)
    off /= np.linalg.norm(off, axis=1, keepdims=True)
    pos[c] = a + off * rng.uniform(0, 300, (c.size, 1)).astype(F)
    pos[:, 2] = np.maximum(pos[:, 2], 20)
    rot = random_quat(rng, n)
    vel = rng.normal(0, 800, (n, 3)).astype(F)
    ang = rng.normal(0, 3, (n, 3)).astype(F)
    _set_cars(env, pos, rot, vel, ang, boost=rng.uniform(0, 100, n), on_ground=np.zeros(n))
    ns = env.n_sim
    bpos = np.stack([rng.uniform(-3800, 3800, ns), rng.uniform(-4800, 4800, ns), rng.uniform(95, 1900, ns)], axis=1)
    env.write_field("BALL_POS", bpos.astype(F))
    env.write_field("BALL_VEL", rng.normal(0, 1500, (ns, 3)).astype(F))
    env.write_field("BALL_ANG", rng.normal(0, 2, (ns, 3)).astype(F))


def crowd_state(env, seed: int) -> None:
    """Cars packed around a moving ball, driving at each other and the ball."""
    rng = np.random.default_rng(seed)
    ns, nc = env.n_sim, env.n_cars
    n = ns * nc
    centers = np.stack([rng.uniform(-3000, 3000, ns), rng.uniform(-4000, 4000, ns), np.full(ns, 17.0)], axis=1)
    ang_slots = rng.uniform(0, 2 * np.pi, (ns, nc))
    radius = rng.uniform(60, 260, (ns, nc))
    pos = np.repeat(centers, nc, axis=0).astype(F)
    pos[:, 0] += (np.cos(ang_slots) * radius).ravel()
    pos[:, 1] += (np.sin(ang_slots) * radius).ravel()
    pos[:, 2] = rng.choice([17.0, 17.0, 17.0, 60.0, 120.0], size=n)
    toward = (np.repeat(centers, nc, axis=0) - pos)[:, :2]
    yaw = np.arctan2(toward[:, 1], toward[:, 0]) + rng.normal(0, 0.3, n)
    rot = yaw_quat(yaw.astype(F))
    speed = rng.uniform(500, 2300, n)
    vel = np.stack([np.cos(yaw) * speed, np.sin(yaw) * speed, np.zeros(n)], axis=1).astype(F)
    _set_cars(env, pos, rot, vel, np.zeros((n, 3), F), boost=rng.uniform(0, 100, n), on_ground=np.ones(n))
    bpos = centers.copy()
    bpos[:, 2] = rng.uniform(93.15, 300, ns)
    env.write_field("BALL_POS", bpos.astype(F))
    env.write_field("BALL_VEL", rng.normal(0, 600, (ns, 3)).astype(F))
    env.write_field("BALL_ANG", rng.normal(0, 1, (ns, 3)).astype(F))
