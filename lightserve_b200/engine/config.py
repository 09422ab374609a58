"""KV-cache sizing config, same fields and checks as lightserve's
``engine/config.py:16-43`` ``CacheConfig`` (block_size defaults to 16, ``:34``),
and the scheduler limits of ``engine/config.py:46-68`` ``SchedulerConfig``.

``kv_cache_bytes_per_block`` adds the physical-size arithmetic the reference
leaves to the deployment (``engine/config.py:7-11``): a block stores K and V for
block_size tokens of every layer and head.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class CacheConfig:
    block_size: int = 16
    num_gpu_blocks: int = 0
    watermark_blocks: int = 0

    def __post_init__(self):
        assert self.block_size > 0, "block_size must be positive"
        assert self.num_gpu_blocks >= 0, "num_gpu_blocks must be non-negative"
        assert 0 <= self.watermark_blocks <= self.num_gpu_blocks, (
            "watermark_blocks must fit within num_gpu_blocks"
        )


@dataclass(frozen=True)
class SchedulerConfig:
    """max_num_seqs: most requests RUNNING at once (the decode batch);
    max_num_batched_tokens: tokens one schedule() call may hand to the model
    (whole prompts of admitted requests plus one per decoding request)."""
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 2048

    def __post_init__(self):
        assert self.max_num_seqs > 0, "max_num_seqs must be positive"
        assert self.max_num_batched_tokens > 0, "max_num_batched_tokens must be positive"


def kv_cache_bytes_per_block(block_size: int, n_layers: int, n_heads: int, head_dim: int,
                             dtype_bytes: int) -> int:
    """Bytes one physical block occupies across all layers (K and V)."""
    return 2 * n_layers * n_heads * block_size * head_dim * dtype_bytes
