"""Physical KV-block allocator with lightserve's ``BlockManager`` API
(``engine/block_manager.py:47-157``): ``can_allocate`` / ``allocate`` at
admission (the watermark applies only there, ``:75-84``), ``can_append_slot``
/ ``append_slot`` per decode step (a new block exactly when the request's
length exceeds ``len(table) * block_size``, ``:145-157``), idempotent ``free``,
and ``OutOfMemoryError`` when a caller skips the ``can_*`` check.

Free ids are kept in a LIFO list. ``as_tensor`` packs the Python tables into
the int32 ``[S, max_blocks]`` array that ``lsb_paged_decode`` reads (unused
entries are -1, which the kernel treats as "no block").
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .request import Request


class OutOfMemoryError(RuntimeError):
    """allocate()/append_slot() was called with too few free blocks."""


@dataclass
class BlockManager:
    block_size: int
    num_gpu_blocks: int
    watermark_blocks: int = 0
    _free: list = field(init=False, repr=False)
    block_tables: dict = field(init=False, default_factory=dict)

    def __post_init__(self):
        # Reverse order so the first pop hands out block 0.
        self._free = list(range(self.num_gpu_blocks - 1, -1, -1))

    @property
    def num_free_blocks(self) -> int:
        return len(self._free)

    def get_block_table(self, request: Request) -> list:
        return self.block_tables.get(request.request_id, [])

    def can_allocate(self, request: Request) -> bool:
        return self.num_free_blocks - request.num_blocks_needed(self.block_size) >= self.watermark_blocks

    def allocate(self, request: Request) -> None:
        if request.request_id in self.block_tables:
            raise ValueError(f"{request.request_id} is already allocated; use append_slot")
        need = request.num_blocks_needed(self.block_size)
        if need > self.num_free_blocks:
            raise OutOfMemoryError(
                f"{request.request_id} needs {need} blocks, {self.num_free_blocks} free "
                "(check can_allocate first)")
        table = [self._free.pop() for _ in range(need)]
        self.block_tables[request.request_id] = table
        request.block_table = table

    def _needs_new_block(self, request: Request) -> bool:
        table = self.block_tables.get(request.request_id, [])
        return request.get_len() > len(table) * self.block_size

    def can_append_slot(self, request: Request) -> bool:
        return (not self._needs_new_block(request)) or self.num_free_blocks >= 1

    def append_slot(self, request: Request) -> bool:
        """Reserves a block for the newest token if needed; returns True if one was added."""
        table = self.block_tables.get(request.request_id)
        if table is None:
            raise ValueError(f"{request.request_id} has no block table; allocate first")
        if not self._needs_new_block(request):
            return False
        if not self._free:
            raise OutOfMemoryError(f"{request.request_id} needs a new block and none is free")
        table.append(self._free.pop())
        return True

    def free(self, request: Request) -> None:
        table = self.block_tables.pop(request.request_id, None)
        if table is None:
            return
        self._free.extend(reversed(table))
        request.block_table = []

    def as_tensor(self, requests, max_blocks: int, device=None):
        """int32 [len(requests), max_blocks] block-table array (-1 padded)."""
        import torch

        out = torch.full((len(requests), max_blocks), -1, dtype=torch.int32)
        for i, r in enumerate(requests):
            t = self.block_tables.get(r.request_id, [])
            if len(t) > max_blocks:
                raise ValueError(f"{r.request_id} holds {len(t)} blocks > max_blocks={max_blocks}")
            if t:
                out[i, : len(t)] = torch.tensor(t, dtype=torch.int32)
        return out if device is None else out.to(device)
