"""Forward-only FlashAttention, drop-in for lightserve's
``kernels/flash_attention.py:182`` ``flash_attention_forward(q, k, v, causal=False)``.

Same contract as the reference: q, k, v are ``[B, H, N, D]`` CUDA tensors of
one shape and one dtype (any strides); the scale is ``1/sqrt(D)``
(``kernels/flash_attention.py:203``); the output is ``torch.empty_like(q)``
(``:202``); bad inputs raise ``AssertionError`` before anything launches
(``:192-199``).

Computation: ``lsb_attn_fwd`` in liblightserve_b200.so. bf16/fp16 inputs with
D in {64, 128} run the tcgen05/TMEM kernel (TMA-staged K/V tiles, QK^T and PV
on the 5th-generation tensor cores, online softmax in fp32); fp32 and other
head dims run the CUDA-core kernel of the same library.
"""
from __future__ import annotations

import math

import torch

from .. import _lib


def _check_qkv(q, k, v):
    assert q.ndim == 4 and k.ndim == 4 and v.ndim == 4, (
        f"expected q/k/v as [B, H, N, D], got {q.ndim}D/{k.ndim}D/{v.ndim}D"
    )
    assert q.shape == k.shape == v.shape, (
        f"q/k/v shapes must match, got {tuple(q.shape)}/{tuple(k.shape)}/{tuple(v.shape)}"
    )
    assert q.is_cuda and k.is_cuda and v.is_cuda, "lightserve_b200 kernels need CUDA tensors"
    assert q.dtype == k.dtype == v.dtype, f"dtype mismatch: q={q.dtype} k={k.dtype} v={v.dtype}"
    assert q.device == k.device == v.device, "q/k/v must be on one device"
    _lib.dtype_code(q.dtype)


def _attn_fwd(q, k, v, o, lse, causal: bool, impl: int = _lib.IMPL_AUTO):
    B, H, N, D = q.shape
    lib = _lib.load()
    with _lib.device_guard(q.device):
        rc = lib.lsb_attn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), _lib.ptr(lse),
            B, H, N, D, _lib.strides4(q), _lib.strides4(k), _lib.strides4(v), _lib.strides4(o),
            1.0 / math.sqrt(D), int(bool(causal)), _lib.dtype_code(q.dtype), impl,
            _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "lsb_attn_fwd")


def flash_attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            causal: bool = False) -> torch.Tensor:
    """O = softmax(Q @ K^T / sqrt(D) [causal]) @ V for q, k, v of shape [B, H, N, D]."""
    _check_qkv(q, k, v)
    o = torch.empty_like(q)
    _attn_fwd(q, k, v, o, None, causal)
    return o
