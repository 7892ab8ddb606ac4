"""Host logic of the multi-GPU path, on CPU with the gloo backend
(world size 2): contiguous slices partition the sims, and the episode
statistics reduction equals the single-process sums."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from carl_b200.shard import episode_stats, shard_range


def test_shard_ranges_partition_the_sims():
    for n, world in [(32768, 8), (10, 3), (7, 7), (1000003, 4)]:
        spans = [shard_range(n, r, world) for r in range(world)]
        assert spans[0][0] == 0
        for (a, na), (b, _) in zip(spans, spans[1:]):
            assert a + na == b
        assert spans[-1][0] + spans[-1][1] == n
        assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)
    with pytest.raises(ValueError):
        shard_range(1, 0, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n_total: int, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        first, count = shard_range(n_total, rank, world)
        g = torch.Generator().manual_seed(1234)
        rewards_all = torch.randn(n_total, generator=g)
        dones_all = torch.rand(n_total, generator=g) < 0.1
        stats = episode_stats(rewards_all[first:first + count], dones_all[first:first + count])
        q.put((rank, first, count, stats.tolist()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_episode_stats_reduce_over_gloo():
    world, n_total = 2, 1001
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(1234)
    rewards = torch.randn(n_total, generator=g)
    dones = torch.rand(n_total, generator=g) < 0.1
    expected = [rewards.double().sum().item(), dones.double().sum().item(), float(n_total)]
    spans = sorted((first, count) for _, first, count, _ in results)
    assert spans == [shard_range(n_total, r, world) for r in range(world)]
    for _, _, _, stats in results:
        assert stats[1] == expected[1] and stats[2] == expected[2]
        assert abs(stats[0] - expected[0]) < 1e-9
