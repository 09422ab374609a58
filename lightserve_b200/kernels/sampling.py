"""Greedy next-token selection: ``argmax`` over each row of the logits, the
next id written in place, optionally each sequence's position advanced.

Replaces ``logits[:, -1, :].argmax(dim=-1)`` and the write of the next id in
lightserve's decode loop (``model/cuda_graph_decode.py:114-118``), with
torch.argmax's order (the first index of the maximum; NaN counts as the
maximum). Computation: ``lsb_greedy_next`` (one CTA per row).
"""
from __future__ import annotations

import torch

from .. import _lib


def greedy_next(logits: torch.Tensor, tokens: torch.Tensor | None = None,
                positions: torch.Tensor | None = None) -> torch.Tensor:
    """logits [S, V] (unit stride along V) -> int64 [S] argmax, written into
    ``tokens`` when given; ``positions`` (int64 [S]) is incremented."""
    assert logits.ndim == 2 and logits.is_cuda and logits.stride(1) == 1, "expected CUDA logits [S, V]"
    S, V = logits.shape
    if tokens is None:
        tokens = torch.empty(S, dtype=torch.int64, device=logits.device)
    assert tokens.shape == (S,) and tokens.dtype == torch.int64 and tokens.is_contiguous()
    if positions is not None:
        assert positions.shape == (S,) and positions.dtype == torch.int64 and positions.is_contiguous()
    if S == 0:
        return tokens
    assert V > 0, "empty vocabulary"
    lib = _lib.load()
    with _lib.device_guard(logits.device):
        rc = lib.lsb_greedy_next(logits.data_ptr(), S, V, logits.stride(0) if S > 1 else V,
                                 _lib.dtype_code(logits.dtype), tokens.data_ptr(),
                                 None if positions is None else positions.data_ptr(),
                                 _lib.stream_ptr(logits.device))
    _lib.check(rc, "lsb_greedy_next")
    return tokens
