"""Operators of lightserve's attention hot path, backed by liblightserve_b200.so."""
from .flash_attention import flash_attention_forward, flash_attention_forward_host, flash_attention_varlen
from .flash_attention_backward import flash_attention
from .fused_rmsnorm_residual import fused_add_rmsnorm
from .fused_swiglu import silu_and_mul
from .linear import PackedWeight, linear, pack_linear_weight
from .sampling import greedy_next
from .paged_attention import paged_decode_attention, rope_kv_write_slots, write_kv_cache

__all__ = ["flash_attention_forward", "flash_attention_forward_host", "flash_attention_varlen",
           "flash_attention", "fused_add_rmsnorm", "silu_and_mul", "linear", "pack_linear_weight", "PackedWeight", "paged_decode_attention",
           "rope_kv_write_slots", "write_kv_cache", "greedy_next"]
