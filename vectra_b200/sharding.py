"""Multi-GPU plumbing for the operator: one process per GPU, batch shards.

Queries are independent (every (b, h) plane of rbf_attention is computed on
its own, kernels/vectra_kernels/spatial_rbf_attention.py:237 launches one
program per plane and query tile), so a batch splits across ranks with no
collective on the data path. The collectives here are only the host-side
ones a multi-GPU run needs around it: the max-over-ranks time of a timed
region, and gathering the output shards in rank order (to check that N
ranks reproduce the 1-rank result bit for bit).

Everything takes an optional process group and works with any backend
(nccl on GPUs, gloo on CPU, which is how the tests run it).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced rows [lo, hi) of `n` for `rank` of `world`.

    The first n % world ranks take one extra row; concatenating the ranges
    in rank order gives 0..n-1 exactly once.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} outside world of {world}')
    if n < 0:
        raise ValueError(f'negative row count {n}')
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_args(q, k, v, scale, key_bias, world: int, rank: int):
    """This rank's batch rows of the operator's arguments.

    q/k/v (and key_bias when its batch dimension is not broadcast) are
    sliced along dim 0; a scale or bias whose batch dimension is 1 (or
    that has fewer than 4 dimensions, i.e. broadcasts over the batch) is
    shared by every rank.
    """
    lo, hi = shard_range(q.shape[0], world, rank)

    def rows(t):
        if t is None or t.dim() < 4 or t.shape[0] == 1:
            return t
        return t[lo:hi]

    return q[lo:hi], k[lo:hi], v[lo:hi], rows(scale), rows(key_bias)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The largest `value` over all ranks (the slowest rank's time).

    Without an initialised process group this is `value` itself.
    """
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_rows(shard: torch.Tensor, n_total: int, group=None
                ) -> torch.Tensor:
    """All ranks' row shards (split by shard_range) concatenated in rank
    order, on every rank. Shards may differ in length by one row."""
    if not (dist.is_available() and dist.is_initialized()):
        return shard
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_range(n_total, world, rank)
    if shard.shape[0] != hi - lo:
        raise ValueError(f'rank {rank} holds {shard.shape[0]} rows, '
                         f'expected {hi - lo}')
    width = -(-n_total // world) if n_total else 0
    padded = shard.new_zeros((width, *shard.shape[1:]))
    padded[:hi - lo] = shard
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    rows = []
    for r, part in enumerate(parts):
        a, b = shard_range(n_total, world, r)
        rows.append(part[:b - a])
    return torch.cat(rows, dim=0)
