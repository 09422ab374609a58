"""Operators of lightserve's attention hot path, backed by liblightserve_b200.so."""
from .flash_attention import flash_attention_forward
from .flash_attention_backward import flash_attention
from .fused_rmsnorm_residual import fused_add_rmsnorm
from .paged_attention import paged_decode_attention, write_kv_cache

__all__ = ["flash_attention_forward", "flash_attention", "fused_add_rmsnorm",
           "paged_decode_attention", "write_kv_cache"]
