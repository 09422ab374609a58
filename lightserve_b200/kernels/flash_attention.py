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

import ctypes
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


def flash_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           cu_seqlens: torch.Tensor, max_seqlen: int, causal: bool = False,
                           out: torch.Tensor | None = None,
                           lse: torch.Tensor | None = None) -> torch.Tensor:
    """Attention over sequences packed along the token axis.

    q, k, v: ``[T, H, D]`` (bf16/fp16, D in {64, 128}, unit last stride, any
    16-byte aligned token/head strides, e.g. views into a fused QKV
    projection); ``cu_seqlens``: int32 ``[num_seqs + 1]`` on the same device,
    sequence s = tokens ``[cu_seqlens[s], cu_seqlens[s+1])``; ``max_seqlen``:
    an upper bound on the longest sequence. Each sequence attends only to
    itself (causally when ``causal``) with scale ``1/sqrt(D)``, as
    ``flash_attention_forward`` on that sequence alone would. Returns ``out``
    (default ``empty_like(q)``); ``lse`` (optional, fp32 ``[H, T]``) receives
    the per-row log-sum-exp. lightserve's forward has no variable-length form
    (``kernels/flash_attention.py:192-199`` requires one N for the batch);
    this is the packed prefill a paged-KV server needs for prompts of
    different lengths (``engine/request.py:86-93``)."""
    assert q.ndim == 3 and k.ndim == 3 and v.ndim == 3, "expected q/k/v as [T, H, D]"
    assert q.shape == k.shape == v.shape, (
        f"q/k/v shapes must match, got {tuple(q.shape)}/{tuple(k.shape)}/{tuple(v.shape)}"
    )
    assert q.is_cuda and k.is_cuda and v.is_cuda, "lightserve_b200 kernels need CUDA tensors"
    assert q.dtype == k.dtype == v.dtype, f"dtype mismatch: q={q.dtype} k={k.dtype} v={v.dtype}"
    assert q.dtype in (torch.bfloat16, torch.float16), "varlen attention needs bf16 or fp16"
    assert q.device == k.device == v.device == cu_seqlens.device, "tensors must be on one device"
    assert cu_seqlens.ndim == 1 and cu_seqlens.dtype == torch.int32 and cu_seqlens.is_contiguous(), (
        "cu_seqlens must be a contiguous int32 vector [num_seqs + 1]"
    )
    assert cu_seqlens.numel() >= 1, "cu_seqlens needs at least one entry"
    T, H, D = q.shape
    assert D in (64, 128), f"varlen attention supports D in {{64, 128}}, got {D}"
    assert 0 <= int(max_seqlen) <= T, f"max_seqlen {max_seqlen} outside [0, {T}]"
    if out is None:
        out = torch.empty_like(q)
    assert out.shape == q.shape and out.dtype == q.dtype and out.device == q.device
    if lse is not None:
        assert lse.shape == (H, T) and lse.dtype == torch.float32 and lse.is_contiguous()
    lib = _lib.load()
    s3 = lambda t: (ctypes.c_int64 * 3)(*t.stride())  # noqa: E731
    with _lib.device_guard(q.device):
        rc = lib.lsb_attn_fwd_varlen(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), _lib.ptr(lse),
            cu_seqlens.data_ptr(), cu_seqlens.numel() - 1, int(max_seqlen), T, H, D,
            s3(q), s3(k), s3(v), s3(out), 1.0 / math.sqrt(D), int(bool(causal)),
            _lib.dtype_code(q.dtype), _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "lsb_attn_fwd_varlen")
    return out


def flash_attention_forward_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                 causal: bool = False, out: torch.Tensor | None = None,
                                 device: torch.device | str = "cuda",
                                 chunk_slices: int = 16) -> torch.Tensor:
    """flash_attention_forward for q, k, v held in (pinned) host memory.

    The (batch, head) slices stream through the GPU in chunks of
    ``chunk_slices``: host-to-device copies, the attention kernel and the
    device-to-host copy of the output run on three streams, double-buffered,
    so the copies in both directions overlap each other and the compute.
    Returns ``out`` (default: a new pinned host tensor like ``q``). The
    calling stream of ``device`` waits for the last copy."""
    assert q.ndim == 4 and q.shape == k.shape == v.shape, "expected q/k/v as [B, H, N, D] of one shape"
    assert q.device.type == k.device.type == v.device.type == "cpu", "host tensors expected"
    assert q.dtype == k.dtype == v.dtype, f"dtype mismatch: q={q.dtype} k={k.dtype} v={v.dtype}"
    assert q.is_contiguous() and k.is_contiguous() and v.is_contiguous(), "contiguous host tensors expected"
    assert chunk_slices >= 1
    _lib.dtype_code(q.dtype)
    B, H, N, D = q.shape
    BH = B * H
    dev = torch.device(device)
    if out is None:
        out = torch.empty_like(q).pin_memory()
    assert out.shape == q.shape and out.dtype == q.dtype and out.is_contiguous()
    if BH == 0 or N == 0:
        return out
    hq, hk, hv, ho = (t.view(BH, N, D) for t in (q, k, v, out))
    cs = min(chunk_slices, BH)
    cur = torch.cuda.current_stream(dev)
    s_in, s_comp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    for s in (s_in, s_comp, s_out):
        s.wait_stream(cur)
    nbuf = 2
    bufs = [[torch.empty(cs, N, D, dtype=q.dtype, device=dev) for _ in range(4)] for _ in range(nbuf)]
    in_done = [torch.cuda.Event() for _ in range(nbuf)]
    comp_done = [torch.cuda.Event() for _ in range(nbuf)]
    out_done = [torch.cuda.Event() for _ in range(nbuf)]
    for ci, s0 in enumerate(range(0, BH, cs)):
        bi, n = ci % nbuf, min(cs, BH - s0)
        dq, dk, dv, do = bufs[bi]
        with torch.cuda.stream(s_in):
            if ci >= nbuf:
                s_in.wait_event(comp_done[bi])  # chunk ci - nbuf has read its inputs
            for d, h in ((dq, hq), (dk, hk), (dv, hv)):
                d[:n].copy_(h[s0:s0 + n], non_blocking=True)
            in_done[bi].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done[bi])
            if ci >= nbuf:
                s_comp.wait_event(out_done[bi])  # its output buffer has been copied out
            x = [t[:n].unsqueeze(0) for t in (dq, dk, dv, do)]
            _attn_fwd(x[0], x[1], x[2], x[3], None, causal)
            comp_done[bi].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[bi])
            ho[s0:s0 + n].copy_(do[:n], non_blocking=True)
            out_done[bi].record(s_out)
    cur.wait_stream(s_out)
    for bl in bufs:  # keep the device buffers alive until the streams are done with them
        for t in bl:
            t.record_stream(s_in); t.record_stream(s_comp); t.record_stream(s_out)
    return out
