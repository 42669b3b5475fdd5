"""Data-parallel sharding of the KDA op across ranks (one process per GPU).

Every (b, h) sequence of the recurrence is independent (the reference folds heads into the
batch before its chunk loop, nope_gdn_mlx.py:833-838), so a global batch splits into contiguous
batch shards with no collective inside the op.  The only cross-rank step a caller needs is the
timing reduction (the slowest rank sets the step time) and, for training, the data-parallel
gradient all-reduce of the surrounding model, which is not part of this op.
"""
from __future__ import annotations


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank `rank`'s contiguous share of n items; the first n % world ranks
    take one item more.  Every item belongs to exactly one rank."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world of {world}")
    if n < 0:
        raise ValueError("negative item count")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch(x, world: int, rank: int, dim: int = 0):
    """This rank's slice of a global tensor along its batch dimension."""
    a, b = shard_range(x.shape[dim], world, rank)
    return x.narrow(dim, a, b - a)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of `value` over all ranks of the default process group (the step time of
    a data-parallel job); the value itself when no group is initialised."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
