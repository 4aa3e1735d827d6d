"""Batch sharding across ranks (one process per GPU).

Sequences are independent (each carries its own recurrent state,
yufmusicgen/model.py:403-404), so a batch of ``total`` sequences is split into
contiguous per-rank ranges with no exchange on the data path; results are
gathered on the host if a caller wants them in one place.
"""

from __future__ import annotations


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, start + count) of ``total`` items owned by ``rank``.

    The first ``total % world`` ranks get one extra item; every item is owned by
    exactly one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if total < 0:
        raise ValueError("total must be >= 0")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_sharded(local, world_size: int, group=None):
    """All-gather per-rank host results (a list per rank) into one list in rank
    order, over the process group's backend (gloo on CPU, NCCL on GPUs)."""
    import torch.distributed as dist

    out = [None] * world_size
    dist.all_gather_object(out, local, group=group)
    merged = []
    for part in out:
        merged.extend(part)
    return merged
