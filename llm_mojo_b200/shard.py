"""Sharding of independent units (sequences, perplexity windows) over the
ranks of one node, and the one gather of their results.

The units of configs 3 and 4 need no data exchange while they run: rank r
takes the contiguous range shard_range(n, world, r), and at the end every
rank joins one all-gather of its equally sized result block (NCCL over
NVLink on the GPUs, gloo on CPU in the tests).
"""

from __future__ import annotations


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of the units of `rank` when n units split evenly over
    `world` ranks (n must divide: every rank's block has the same shape, as
    the all-gather needs)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world size or rank")
    if n % world:
        raise ValueError(f"{n} units do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def gather_blocks(local, world: int):
    """All ranks' equally shaped blocks, stacked in rank order: one
    all_gather_into_tensor (the ranks' process group must be initialised
    when world > 1)."""
    import torch
    import torch.distributed as dist

    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    if world > 1:
        dist.all_gather_into_tensor(out, local.contiguous())
    else:
        out.copy_(local)
    return out
