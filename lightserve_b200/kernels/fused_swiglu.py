"""Fused SwiGLU activation: ``silu(gate) * up`` from one fused gate|up GEMM output.

Replaces lightserve's ``F.silu(gate_proj(h)) * up_proj(h)``
(``model/minimal_llama.py:231-233``) with the same roundings: silu computed in
fp32 and rounded to the input dtype, then the product of the two dtype
values rounded again. ``gu`` is ``[S, 2I]`` (gate in the first ``I`` columns,
up in the last ``I``); the result is ``[S, I]``.

Computation: ``lsb_swiglu`` in liblightserve_b200.so (one pass, 16-byte
vectors).
"""
from __future__ import annotations

import torch

from .. import _lib


def silu_and_mul(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    assert gu.ndim == 2 and gu.shape[1] % 2 == 0, f"expected gu as [S, 2I], got {tuple(gu.shape)}"
    assert gu.is_cuda, "lightserve_b200 kernels need CUDA tensors"
    assert gu.stride(1) == 1, "gu must be contiguous along the last dim"
    S, I2 = gu.shape
    I = I2 // 2
    if out is None:
        out = torch.empty(S, I, dtype=gu.dtype, device=gu.device)
    assert out.shape == (S, I) and out.dtype == gu.dtype and out.device == gu.device
    assert out.stride(1) == 1, "out must be contiguous along the last dim"
    if S == 0 or I == 0:
        return out
    lib = _lib.load()
    with _lib.device_guard(gu.device):
        rc = lib.lsb_swiglu(gu.data_ptr(), out.data_ptr(), S, I,
                            gu.stride(0) if S > 1 else I2, out.stride(0) if S > 1 else I,
                            _lib.dtype_code(gu.dtype), _lib.stream_ptr(gu.device))
    _lib.check(rc, "lsb_swiglu")
    return out
