"""Fused add+RMSNorm oracle (test infrastructure only; see oracle/__init__.py).

Restates _fused_add_rmsnorm_kernel (kernels/fused_rmsnorm_residual.py:31-70)
and the reference's test oracle rmsnorm_residual_reference
(kernels/tests/test_fused_rmsnorm_residual.py:24-29):
h = x + residual rounded to the input dtype (:55-56); variance = mean of
float(h)^2 in fp32 (:64-65); out = (float(h) * rsqrt(var + eps) * float(w))
rounded to the input dtype (:66-70).
"""
from __future__ import annotations

import torch


def rmsnorm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    x, residual, weight = (t.detach().cpu() for t in (x, residual, weight))
    h = x + residual
    hf = h.float()
    var = hf.pow(2).mean(-1, keepdim=True)
    out = (hf * torch.rsqrt(var + eps) * weight.float()).to(x.dtype)
    return out, h


def rmsnorm_bytes(M: int, N: int, itemsize: int) -> int:
    """Algorithmic bytes: read x, residual; write out, h
    (kernels/benchmark_fused_rmsnorm_residual.py:59-64)."""
    return 4 * M * N * itemsize
