"""Autograd FlashAttention, drop-in for lightserve's
``kernels/flash_attention_backward.py:400`` ``flash_attention(q, k, v, causal=False)``.

Mirrors the reference's structure (``:172-420``):

* ``_flash_attention_forward_lse(q, k, v, causal) -> (o, L)``: the forward
  that also writes the fp32 per-row log-sum-exp ``L = m + ln(l)``, shape
  ``[B, H, N]`` (``:172-199``);
* ``_flash_attention_backward(do, q, k, v, o, L, causal) -> (dq, dk, dv)``:
  ``Dsum = rowsum(dO * O)``, then per K/V tile a sweep over Q tiles that
  recomputes ``P = exp(S - L)`` and accumulates dV, dK and an fp32 dQ, which
  is rounded to q's dtype at the end (``:333-382``);
* ``_FlashAttentionFunction`` saves ``(q, k, v, o, L)`` (``:385-397``).

Computation: ``lsb_attn_fwd`` (with an LSE output) and ``lsb_attn_bwd`` in
liblightserve_b200.so. The backward's fp32 scratch (Dsum and the dQ
accumulator) is allocated here with torch and handed to the C ABI, which never
allocates.
"""
from __future__ import annotations

import math

import torch

from .. import _lib
from .flash_attention import _attn_fwd, _check_qkv


def _flash_attention_forward_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool):
    B, H, N, D = q.shape
    o = torch.empty_like(q)
    L = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
    _attn_fwd(q, k, v, o, L, causal)
    return o, L


def _flash_attention_backward(do: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                              o: torch.Tensor, L: torch.Tensor, causal: bool,
                              impl: int = _lib.IMPL_AUTO):
    B, H, N, D = q.shape
    assert do.shape == q.shape and do.dtype == q.dtype, "dO must match q's shape and dtype"
    assert L.shape == (B, H, N) and L.dtype == torch.float32 and L.is_contiguous()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    lib = _lib.load()
    ws_bytes = lib.lsb_attn_bwd_workspace_size(B, H, N, D)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    with _lib.device_guard(q.device):
        rc = lib.lsb_attn_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), L.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, H, N, D,
            _lib.strides4(q), _lib.strides4(k), _lib.strides4(v), _lib.strides4(o),
            _lib.strides4(do), _lib.strides4(dq), _lib.strides4(dk), _lib.strides4(dv),
            1.0 / math.sqrt(D), int(bool(causal)), _lib.dtype_code(q.dtype), impl,
            ws.data_ptr(), ws_bytes, _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "lsb_attn_bwd")
    return dq, dk, dv


class _FlashAttentionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal):
        o, L = _flash_attention_forward_lse(q, k, v, causal)
        ctx.save_for_backward(q, k, v, o, L)
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, L = ctx.saved_tensors
        dq, dk, dv = _flash_attention_backward(do, q, k, v, o, L, ctx.causal)
        return dq, dk, dv, None


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """Autograd-enabled FlashAttention over [B, H, N, D] q, k, v (same checks as the forward)."""
    _check_qkv(q, k, v)
    return _FlashAttentionFunction.apply(q, k, v, causal)
