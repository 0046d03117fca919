"""Multi-GPU partitioning of the Gated DeltaNet hot path (one process per GPU).

Batched decode shards by sequence: every rank owns a contiguous range of the
sequences and runs the whole layer on them; there is no collective on the data
path (the reference runs one sequence on one device, gpu_offload.cu:999).
Timing across ranks is the max of the per-rank device times.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the n units rank owns; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device=None) -> float:
    """The max of `value` over the process group (the value itself without one)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
