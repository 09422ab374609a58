"""Multi-GPU partitioning of the hot path: independent units, no collective.

The attention path shards over (batch x head) slices and the paged decode over
sequences (lightserve's kernels treat each (b, h) and each request
independently, kernels/flash_attention.py:100-104, engine/scheduler.py). One
process per GPU owns a contiguous range of units; the only cross-rank
communication is host-side bookkeeping (timing maxima, result gathering for
parity checks), never on the data path.
"""
from __future__ import annotations

import torch


def shard_range(n_units: int, rank: int, world: int) -> tuple[int, int]:
    """[start, end) of the units rank `rank` owns; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(x: float, group=None) -> float:
    """Maximum of a per-rank scalar (device timings are reported as the max over ranks)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(x)
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
