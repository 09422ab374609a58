"""Weight-streaming linear layer for decode batches: ``y = x @ w``.

Replaces the projections of lightserve's decode step (``h @ w`` in
``model/minimal_llama.py:216-234`` and ``:249``; lightserve's own GEMM kernel is
``kernels/tiled_matmul.py:55-151``): bf16/fp16 operands, fp32 accumulation,
one rounding to the operand dtype. Serves up to 128 rows of ``x`` (decode
batches); larger batches (prefill) stay on cuBLAS.

The weight is packed once (``pack_linear_weight``) from its transpose
``w_t = w.t()`` (``[N, K]``) into 16 KiB tiles that the kernel streams with
sequential bulk copies.

Computation: ``lsb_linear`` in liblightserve_b200.so (tcgen05 MMAs with the
weight tile as the A operand, K split across the CTAs of a thread-block
cluster and reduced in distributed shared memory, weight ring that starts
before the previous kernel of the stream has finished). No scratch memory;
the summation order is fixed, so results are reproducible.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib

MAX_ROWS = 128


@dataclass
class PackedWeight:
    """A weight W [K, N] packed for ``linear`` (from W^T [N, K])."""
    data: torch.Tensor  # uint8, lsb_linear_packed_bytes(N, K)
    N: int
    K: int
    dtype: torch.dtype

    @property
    def device(self):
        return self.data.device


def pack_linear_weight(w_t: torch.Tensor) -> PackedWeight:
    """Packs ``w_t`` = W^T ([N, K], K contiguous, bf16/fp16, CUDA)."""
    assert w_t.ndim == 2 and w_t.is_cuda and w_t.stride(1) == 1, "expected a CUDA [N, K] tensor, K contiguous"
    assert w_t.dtype in (torch.bfloat16, torch.float16), f"bf16/fp16 expected, got {w_t.dtype}"
    N, K = w_t.shape
    assert K % 8 == 0, f"K={K} must be a multiple of 8"
    lib = _lib.load()
    nbytes = int(lib.lsb_linear_packed_bytes(N, K))
    data = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=w_t.device)
    if nbytes:
        with _lib.device_guard(w_t.device):
            rc = lib.lsb_linear_pack(w_t.data_ptr(), w_t.stride(0) if N > 1 else K, N, K,
                                     _lib.dtype_code(w_t.dtype), data.data_ptr(), nbytes,
                                     _lib.stream_ptr(w_t.device))
        _lib.check(rc, "lsb_linear_pack")
    return PackedWeight(data, N, K, w_t.dtype)


def linear(x: torch.Tensor, w: PackedWeight | torch.Tensor, out: torch.Tensor | None = None,
           pdl: bool = True) -> torch.Tensor:
    """``x [S, K] @ W`` -> ``[S, N]``; ``w`` is a PackedWeight or W^T [N, K]
    (packed on the fly)."""
    if not isinstance(w, PackedWeight):
        w = pack_linear_weight(w)
    assert x.ndim == 2 and x.shape[1] == w.K, f"expected x [S, {w.K}], got {tuple(x.shape)}"
    assert x.is_cuda and x.device == w.device, "lightserve_b200 kernels need CUDA tensors on the weight's device"
    assert x.dtype == w.dtype, f"dtype mismatch: x={x.dtype} w={w.dtype}"
    assert x.stride(1) == 1, "x must be contiguous along K"
    S, K = x.shape
    N = w.N
    assert S <= MAX_ROWS, f"at most {MAX_ROWS} rows (decode batches); got {S}"
    if out is None:
        out = torch.empty(S, N, dtype=x.dtype, device=x.device)
    assert out.shape == (S, N) and out.dtype == x.dtype and out.stride(1) == 1
    if S == 0 or N == 0:
        return out
    lib = _lib.load()
    with _lib.device_guard(x.device):
        rc = lib.lsb_linear(x.data_ptr(), x.stride(0) if S > 1 else K, w.data.data_ptr(),
                            out.data_ptr(), out.stride(0) if S > 1 else N, S, N, K,
                            _lib.dtype_code(x.dtype), 1 if pdl else 0, _lib.stream_ptr(x.device))
    _lib.check(rc, "lsb_linear")
    return out
