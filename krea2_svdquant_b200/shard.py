"""Batch sharding for multi-GPU runs: one process per GPU, each running its own
slice of the image batch with no collective on the data path (images denoise
independently).  The only collective is the max-over-ranks of a device time.
"""
from __future__ import annotations

import torch


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """``(start, count)`` of rank ``rank``'s contiguous share of ``total`` items; shares differ by at most 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device: torch.device | str | None = None) -> float:
    """The maximum of ``value`` over the default process group (the value itself when not distributed)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
