"""The env around the tick, through the C ABI on the device: RL step packing
(obs, state, rewards, dones, auto-reset), kickoff resets, state injection,
sharding by global sim offset, host-buffer stepping and argument errors."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from carl_b200 import capi, workloads
import cuda_copy
import parity

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
NP_DTYPE = {capi.DT_F32: np.float32, capi.DT_I32: np.int32, capi.DT_BOOL: np.uint8, capi.DT_I64: np.int64}
ALL_BUFFERS = [capi.BUF_OBS, capi.BUF_TRANSITION_OBS, capi.BUF_STATE, capi.BUF_TRANSITION_STATE, capi.BUF_REWARDS,
               capi.BUF_DONES, capi.BUF_SCORE_DIFFERENCE, capi.BUF_EPISODE_TICKS,
               capi.BUF_TRANSITION_SCORE_DIFFERENCE, capi.BUF_TRANSITION_EPISODE_TICKS, capi.BUF_OVERTIME,
               capi.BUF_TRANSITION_OVERTIME]


def torch():
    import torch as t

    return t


def read_buffer(env, which) -> np.ndarray:
    ptr, shape, dt = env.buffer(which)
    out = np.empty(shape, dtype=NP_DTYPE[dt])
    env.synchronize()
    cuda_copy.d2h(out, ptr)
    return out


def buffers_close(ours: np.ndarray, theirs: np.ndarray) -> int:
    """Number of entries outside the parity tolerance (exact for integers)."""
    if ours.dtype == np.float32:
        a, b = ours.reshape(-1), theirs.reshape(-1)
        bad = 0
        for i in range(0, a.size, 1 << 24):  # in chunks: the C5 obs buffers hold ~10^8 entries
            x, y = a[i:i + (1 << 24)].astype(np.float64), b[i:i + (1 << 24)].astype(np.float64)
            tol = np.maximum(parity.ABS_TOL, parity.REL_TOL * np.abs(y))
            bad += int((np.abs(x - y) > tol).sum())
        return bad
    return int((ours != theirs.astype(ours.dtype)).sum())


@pytest.mark.parametrize("oracle", ["cuda_build", "host_build"])
@pytest.mark.parametrize("nb, no, kind, frameskip, flags", [
    (2, 2, capi.ACTIONS_DISCRETE, 8, {}),
    (2, 2, capi.ACTIONS_CONTINUOUS, 8, {}),
    (3, 3, capi.ACTIONS_CONTINUOUS, 1, {}),
    (1, 1, capi.ACTIONS_DISCRETE, 2, {"normalize": True}),
    (1, 2, capi.ACTIONS_DISCRETE, 1, {"previous_controls": True, "invert_orange": False}),
])
def test_env_step_matches_reference(oracle_built, nb, no, kind, frameskip, flags, oracle):
    """Env steps in the default mode against the reference's CUDA build, and in
    the source-semantics mode against the reference's host build."""
    from oracle.refenv import RefCpu, RefGpu

    n_sim, seed = 64, 11 + nb + 3 * no
    rng = np.random.default_rng(seed)
    n = n_sim * (nb + no)
    compat = 0 if oracle == "cuda_build" else capi.SOURCE_LAGGED_LATERAL_FRICTION
    env = capi.Env(n_sim, nb, no, seed, frameskip=frameskip, compat_flags=compat, **flags)
    ref = (RefGpu if oracle == "cuda_build" else RefCpu)(n_sim, nb, no, seed, frameskip=frameskip, **flags)
    env.set_limit(capi.LIMIT_MAX_TICKS, 300)
    env.set_limit(capi.LIMIT_NO_TOUCH_TIMEOUT_TICKS, 200)
    ref.set_limits(300, -1, 200, -1)
    worst: dict[int, int] = {}
    steps = 40 if frameskip > 1 else 120
    for _ in range(steps):
        a = workloads.discrete_actions(rng, n) if kind == capi.ACTIONS_DISCRETE else workloads.continuous_actions(rng, n)
        env.env_step(kind, torch().from_numpy(a).cuda())
        ref.env_step(kind, a)
        for b in ALL_BUFFERS:
            worst[b] = max(worst.get(b, 0), buffers_close(read_buffer(env, b), ref.get_buffer(b)))
    env.close()
    ref.close()
    # Early steps must agree exactly in every buffer; over the whole episode a
    # few obs entries may drift past the single-tick tolerance (contact chaos).
    assert worst[capi.BUF_DONES] == 0 and worst[capi.BUF_EPISODE_TICKS] == 0, worst
    assert worst[capi.BUF_REWARDS] == 0 and worst[capi.BUF_SCORE_DIFFERENCE] == 0, worst
    obs_entries = n * env.obs_dim
    assert worst[capi.BUF_OBS] <= 0.01 * obs_entries, worst


def test_c5_shard_env_steps_with_masked_resets_match_reference_cuda_build(oracle_built):
    """C5's per-GPU shard at its size (bench.py --workload c5): 4v4, n_sim =
    131072, frameskip 1, discrete actions, the seeded mixed states, and after every
    env step a masked apply_reset_state that puts a random 1 % of the sims back at
    their kickoff state; default mode against the reference's CUDA build on the
    same inputs.  Rewards, dones and the counters agree exactly; obs within the
    single-tick tolerance except a bounded share (contact chaos)."""
    from oracle.refenv import RefGpu

    import bench

    t = torch()
    n_sim, nb, no, seed = 131072, 4, 4, 0
    n = n_sim * (nb + no)
    rows = bench.kickoff_rows(n_sim, nb, no, seed)
    order = ["ball_position", "ball_velocity", "ball_angular_velocity", "car_position", "car_rotation",
             "car_velocity", "car_angular_velocity", "car_demoed"]
    env = capi.Env(n_sim, nb, no, seed, frameskip=1)
    workloads.mixed_state(env, seed)
    ref = RefGpu(n_sim, nb, no, seed, frameskip=1)
    ref.restore(env.snapshot())
    dev = {k: t.from_numpy(v).cuda() for k, v in rows.items()}
    rng = np.random.default_rng(5)
    worst: dict[int, int] = {}
    for _ in range(4):
        a = workloads.discrete_actions(rng, n)
        mask = (rng.uniform(size=n_sim) < 0.01).astype(np.uint8)
        env.env_step(capi.ACTIONS_DISCRETE, t.from_numpy(a).cuda())
        env.apply_reset_state(n_sim, *[dev[o] for o in order], True, None, None, dev["blue_score"],
                              dev["orange_score"], dev["episode_ticks"], reset_mask=t.from_numpy(mask).cuda())
        ref.env_step(capi.ACTIONS_DISCRETE, a)
        ref.apply_reset_state(n_sim, *[rows[o] for o in order], True, None, None, rows["blue_score"],
                              rows["orange_score"], rows["episode_ticks"], reset_mask=mask)
        for b in ALL_BUFFERS:
            worst[b] = max(worst.get(b, 0), buffers_close(read_buffer(env, b), ref.get_buffer(b)))
    obs_entries = n * env.obs_dim
    env.close()
    ref.close()
    print("C5 shard, 4 env steps with 1 % masked resets: entries outside tolerance per buffer", worst)
    for b in (capi.BUF_DONES, capi.BUF_EPISODE_TICKS, capi.BUF_REWARDS, capi.BUF_SCORE_DIFFERENCE,
              capi.BUF_TRANSITION_EPISODE_TICKS, capi.BUF_TRANSITION_SCORE_DIFFERENCE, capi.BUF_OVERTIME):
        assert worst[b] == 0, (b, worst)
    assert worst[capi.BUF_OBS] <= 0.01 * obs_entries, worst


def test_env_step_golden():
    z = np.load(GOLDEN / "env_step_1v1.npz")
    n_sim, nb, no, seed, frameskip = (int(x) for x in z["dims"])
    # The golden vectors come from the reference's host build (source semantics).
    env = capi.Env(n_sim, nb, no, seed, frameskip=frameskip, compat_flags=capi.SOURCE_LAGGED_LATERAL_FRICTION)
    env.reset()
    names = {"obs": capi.BUF_OBS, "state": capi.BUF_STATE, "rewards": capi.BUF_REWARDS, "dones": capi.BUF_DONES,
             "episode_ticks": capi.BUF_EPISODE_TICKS, "transition_obs": capi.BUF_TRANSITION_OBS}
    for step in range(4):
        env.env_step(capi.ACTIONS_DISCRETE, torch().from_numpy(z[f"actions/{step}"]).cuda())
        for k, b in names.items():
            assert buffers_close(read_buffer(env, b), z[f"{k}/{step}"]) == 0, (step, k)
    env.close()


def test_sharded_envs_equal_one_env():
    """Two shards with global sim offsets reproduce one env over all sims bit for bit."""
    t = torch()
    n_sim, nb, no, seed = 64, 2, 2, 9
    whole = capi.Env(n_sim, nb, no, seed)
    parts = [capi.Env(n_sim // 2, nb, no, seed, sim_offset=r * (n_sim // 2)) for r in range(2)]
    for e in [whole] + parts:
        e.reset()
    rng = np.random.default_rng(3)
    for step in range(6):
        ctl = workloads.controls(rng, n_sim * (nb + no))
        whole.ticks(capi.ACTIONS_DIRECT, t.from_numpy(ctl.view(np.int32)).cuda(), 8)
        half = ctl.shape[0] // 2
        for r, e in enumerate(parts):
            e.ticks(capi.ACTIONS_DIRECT, t.from_numpy(ctl[r * half:(r + 1) * half].view(np.int32)).cuda(), 8)
        # Terminated sims re-kick off with the global sim index in the hash.
        whole.reset_dones()
        for e in parts:
            e.reset_dones()
    a = whole.snapshot()
    b = [e.snapshot() for e in parts]
    for name in a:
        if name == "TICK_COUNT":
            continue
        joined = np.concatenate([b[0][name], b[1][name]], axis=0)
        assert (a[name] == joined).all(), name
    for e in [whole] + parts:
        e.close()


def test_ticks_host_equals_device_path():
    t = torch()
    n_sim, nb, no = 128, 3, 3
    a = capi.Env(n_sim, nb, no, 4)
    b = capi.Env(n_sim, nb, no, 4)
    workloads.floor_state(a, 5)
    b.restore(a.snapshot())
    rng = np.random.default_rng(8)
    rewards = np.zeros(n_sim, np.float32)
    for _ in range(3):
        ctl = workloads.controls(rng, n_sim * (nb + no))
        a.ticks(capi.ACTIONS_DIRECT, t.from_numpy(ctl.view(np.int32)).cuda(), 8)
        b.ticks_host(capi.ACTIONS_DIRECT, ctl, 8, rewards)
    sa, sb = a.snapshot(), b.snapshot()
    assert all((sa[k] == sb[k]).all() for k in sa)
    assert np.isfinite(rewards).all()
    a.close()
    b.close()


def _reset_inputs(rng, k, n_cars, n_sim, with_optional):
    f = np.float32
    car_rot = workloads.random_quat(rng, k * n_cars).reshape(k, n_cars, 4)
    d = {
        "ball_position": np.stack([rng.uniform(-3000, 3000, k), rng.uniform(-4000, 4000, k),
                                   rng.uniform(100, 1500, k)], 1).astype(f),
        "ball_velocity": rng.normal(0, 500, (k, 3)).astype(f),
        "ball_angular_velocity": rng.normal(0, 1, (k, 3)).astype(f),
        "car_position": np.stack([rng.uniform(-3500, 3500, (k, n_cars)), rng.uniform(-4500, 4500, (k, n_cars)),
                                  rng.uniform(17, 600, (k, n_cars))], 2).astype(f),
        "car_rotation": car_rot.astype(f),
        "car_velocity": rng.normal(0, 600, (k, n_cars, 3)).astype(f),
        "car_angular_velocity": rng.normal(0, 2, (k, n_cars, 3)).astype(f),
        "car_demoed": (rng.uniform(size=(k, n_cars)) < 0.1).astype(np.uint8),
    }
    if with_optional:
        d["car_boost"] = rng.uniform(0, 100, (k, n_cars)).astype(f)
        d["blue_score"] = rng.integers(0, 5, k).astype(np.int32)
        d["orange_score"] = rng.integers(0, 5, k).astype(np.int32)
        d["episode_ticks"] = rng.integers(0, 1000, k).astype(np.int32)
    return d


@pytest.mark.parametrize("mode", ["indices", "mask", "all"])
def test_apply_reset_state_matches_reference_cuda_build(oracle_built, mode):
    from oracle.refenv import RefGpu

    t = torch()
    n_sim, nb, no, seed = 48, 2, 2, 6
    n_cars = nb + no
    rng = np.random.default_rng(17)
    env = capi.Env(n_sim, nb, no, seed)
    ref = RefGpu(n_sim, nb, no, seed)
    env.reset()
    ref.reset()
    idx = mask = None
    if mode == "indices":
        idx = np.sort(rng.choice(n_sim, 13, replace=False)).astype(np.int64)
        k = idx.size
    elif mode == "mask":
        mask = (rng.uniform(size=n_sim) < 0.3).astype(np.uint8)
        k = n_sim
    else:
        k = n_sim
    inp = _reset_inputs(rng, k, n_cars, n_sim, with_optional=(mode != "all"))
    dev = {name: t.from_numpy(v).cuda() for name, v in inp.items()}
    order = ["ball_position", "ball_velocity", "ball_angular_velocity", "car_position", "car_rotation",
             "car_velocity", "car_angular_velocity", "car_demoed"]
    opt = ["car_boost", None, "blue_score", "orange_score", "episode_ticks"]
    env.apply_reset_state(k, *[dev[o] for o in order], True,
                          *[dev.get(o) if o else None for o in opt],
                          simulation_indices=None if idx is None else t.from_numpy(idx).cuda(),
                          reset_mask=None if mask is None else t.from_numpy(mask).cuda())
    ref.apply_reset_state(k, *[inp[o] for o in order], True, *[inp.get(o) if o else None for o in opt],
                          simulation_indices=idx, reset_mask=mask)
    env.synchronize()
    rep = parity.compare_snapshots(env.snapshot(), ref.snapshot())
    assert parity.all_ok(rep), parity.summarize(rep)
    # The outputs the reset repacks (the masked path: one fused kernel).
    for b in [capi.BUF_OBS, capi.BUF_STATE, capi.BUF_SCORE_DIFFERENCE, capi.BUF_EPISODE_TICKS, capi.BUF_OVERTIME]:
        assert buffers_close(read_buffer(env, b), ref.get_buffer(b)) == 0, b
    ctl = workloads.controls(rng, n_sim * n_cars)
    env.ticks(capi.ACTIONS_DIRECT, t.from_numpy(ctl.view(np.int32)).cuda(), 1)
    ref.ticks(capi.ACTIONS_DIRECT, ctl, 1)
    env.synchronize()
    rep = parity.compare_snapshots(env.snapshot(), ref.snapshot())
    assert parity.all_ok(rep), parity.summarize(rep)
    env.close()
    ref.close()


def test_errors_leave_state_untouched():
    t = torch()
    env = capi.Env(16, 1, 1, 0)
    env.reset()
    before = env.snapshot()
    ctl = t.zeros((32, 8), dtype=t.int32, device="cuda")
    with pytest.raises(capi.CarlbError) as e:
        env.ticks(7, ctl, 1)
    assert e.value.status == capi.ERR_VALUE
    with pytest.raises(capi.CarlbError):
        env.ticks(capi.ACTIONS_DIRECT, ctl, -1)
    with pytest.raises(capi.CarlbError):
        env.env_step(capi.ACTIONS_DIRECT, ctl)
    with pytest.raises(capi.CarlbError):
        env.set_limit(capi.LIMIT_FRAMESKIP, 0)
    idx = t.arange(17, dtype=t.int64, device="cuda")
    pos = t.zeros((17, 3), dtype=t.float32, device="cuda")
    with pytest.raises(capi.CarlbError, match="too many"):
        env.set_ball(17, pos, pos, pos, idx)
    cars = t.zeros((16, 2, 4), dtype=t.float32, device="cuda")
    mask = t.ones(16, dtype=t.uint8, device="cuda")
    with pytest.raises(capi.CarlbError, match="not both"):
        env.apply_reset_state(16, pos, pos, pos, cars, cars, cars, cars, mask, True,
                              simulation_indices=idx, reset_mask=mask)
    after = env.snapshot()
    assert all((before[k] == after[k]).all() for k in before)
    env.close()


def test_stream_is_the_envs_own():
    t = torch()
    env = capi.Env(8, 1, 1, 0)
    s = env.stream
    assert s != 0
    ext = t.cuda.ExternalStream(s)
    x = t.ones(1024, device="cuda")
    with t.cuda.stream(ext):
        y = x * 2
    ext.synchronize()
    assert float(y.sum()) == 2048.0
    env.close()


def test_sim_slices_equal_single_slice(monkeypatch):
    """The staged tick steps large envs as several sim slices on separate
    streams; the result is bit-identical to stepping them as one slice."""
    t = torch()
    n_sim, nb, no = 16384, 2, 2
    snaps = []
    for groups in ("1", "4"):
        monkeypatch.setenv("CARLB_GROUPS", groups)
        env = capi.Env(n_sim, nb, no, 3)
        workloads.mixed_state(env, 5)
        rng = np.random.default_rng(6)
        for _ in range(3):
            env.ticks(capi.ACTIONS_DIRECT, t.from_numpy(workloads.controls(rng, n_sim * (nb + no)).view(np.int32)).cuda(), 8)
        snaps.append(env.snapshot())
        env.close()
    for name in snaps[0]:
        assert (snaps[0][name] == snaps[1][name]).all(), name
