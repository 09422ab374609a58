"""Fused residual-add + RMSNorm, drop-in for lightserve's
``kernels/fused_rmsnorm_residual.py:73`` ``fused_add_rmsnorm(x, residual, weight, eps=1e-6)``.

Returns ``(rmsnorm(x + residual) * weight, x + residual)`` with the reference's
rounding: ``h = x + residual`` in the input dtype, the mean of squares of
``float(h)`` in fp32, ``out = (float(h) * rrms * float(weight))`` rounded to
the input dtype (``kernels/fused_rmsnorm_residual.py:55-70``). The same
assertions guard the call (``:86-97``): 2-D equal shapes, matching weight,
CUDA tensors, one dtype, unit stride along the last dim.

Computation: ``lsb_rmsnorm_residual`` in liblightserve_b200.so (one CTA per
row, the row held in registers as 16-byte vectors).
"""
from __future__ import annotations

import torch

from .. import _lib


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                      eps: float = 1e-6):
    assert x.shape == residual.shape and x.ndim == 2, (
        f"x {tuple(x.shape)} and residual {tuple(residual.shape)} must both be 2D and equal-shaped"
    )
    assert weight.ndim == 1 and weight.shape[0] == x.shape[1], (
        f"weight shape {tuple(weight.shape)} must match x's last dim {x.shape[1]}"
    )
    assert x.is_cuda and residual.is_cuda and weight.is_cuda, "lightserve_b200 kernels need CUDA tensors"
    assert x.dtype == residual.dtype == weight.dtype, (
        f"dtype mismatch: x={x.dtype} residual={residual.dtype} weight={weight.dtype}"
    )
    assert x.stride(1) == 1 and residual.stride(1) == 1, (
        "x and residual must be contiguous along the last dim (row-major, no transposed views)"
    )
    assert weight.stride(0) == 1 or weight.shape[0] <= 1, "weight must be contiguous"
    M, N = x.shape
    out = torch.empty_like(x)
    residual_out = torch.empty_like(x)
    if M == 0 or N == 0:
        return out, residual_out
    def ld(t):  # a single row's stride is meaningless; report a dense one
        return t.stride(0) if M > 1 else N

    lib = _lib.load()
    with _lib.device_guard(x.device):
        rc = lib.lsb_rmsnorm_residual(
            x.data_ptr(), residual.data_ptr(), weight.data_ptr(), out.data_ptr(),
            residual_out.data_ptr(), M, N, ld(x), ld(residual), ld(out), ld(residual_out), float(eps), _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device),
        )
    _lib.check(rc, "lsb_rmsnorm_residual")
    return out, residual_out
