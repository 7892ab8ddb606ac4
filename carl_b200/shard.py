"""Sharding sims over GPUs: one process per GPU, contiguous sim slices.

Sims never interact, so a run over G GPUs is G independent envs whose
`sim_offset` is the global index of their first sim; the kickoff hash and the
demolition respawn seed use global indices, which makes the sharded run
bit-identical to one env over all sims.  The only collective is the optional
reduction of episode statistics at rollout boundaries.
"""

from __future__ import annotations


def shard_range(n_total: int, rank: int, world: int) -> tuple[int, int]:
    """(first global sim, number of sims) of `rank`'s contiguous slice; the
    first n_total % world ranks take one extra sim."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    if n_total < world:
        raise ValueError("fewer sims than ranks")
    base, extra = divmod(n_total, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def make_env(n_total: int, n_blue: int, n_orange: int, seed: int, rank: int, world: int, device: int, **kw):
    """This rank's env over its slice (carl_b200.carl.Env)."""
    from .carl import Env

    first, count = shard_range(n_total, rank, world)
    return Env(count, n_blue, n_orange, seed, device=device, sim_offset=first, **kw)


def episode_stats(rewards, dones, group=None):
    """Sum of rewards, finished episodes and sims over all ranks (float64
    [3] tensor on the inputs' device); a single all-reduce when a process group
    is initialised, local sums otherwise."""
    import torch
    import torch.distributed as dist

    local = torch.stack([rewards.double().sum(), dones.double().sum(),
                         torch.tensor(float(rewards.numel()), dtype=torch.float64, device=rewards.device)])
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(local, op=dist.ReduceOp.SUM, group=group)
    return local
