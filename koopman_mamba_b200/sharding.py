"""Partitioning the SKA core across ranks (one process per GPU).

Every SKA quantity belongs to one (batch, head) series: the chunk statistics, the
prefix scan, the chunk operators and the max-key-norm scale are all computed per
series (KLF/koopman_lm/ska.py:73-151 reduce over time and key dimension only).
So the layer splits over batch or heads with no exchange between ranks.  A rank
passes its slice to the C ABI as a strided view: `SkaTensor` carries the batch,
token and head strides, so a head slice of a [B, T, H, D] tensor needs no copy.

The only collective the layer's callers need is the timing reduction
(`max_over_ranks`).  Gradient all-reduce for data-parallel training belongs to
the full language model, not to this layer.
"""
from __future__ import annotations


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced [lo, hi) share of n items for `rank` of `world`.

    The first n % world ranks get one extra item; a rank may get none when
    world > n.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if n < 0:
        raise ValueError(f"negative item count {n}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def batch_shard(x, world: int, rank: int):
    """This rank's batch slice of a [B, T, H, D] tensor (a view)."""
    lo, hi = shard_range(x.shape[0], world, rank)
    return x[lo:hi]


def head_shard(x, world: int, rank: int):
    """This rank's head slice of a [B, T, H, D] tensor (a strided view, no copy)."""
    lo, hi = shard_range(x.shape[2], world, rank)
    return x[:, :, lo:hi]


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar over the default process group.

    Multi-GPU step times are the slowest rank's time.  Without an initialised
    process group this is the identity.
    """
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
