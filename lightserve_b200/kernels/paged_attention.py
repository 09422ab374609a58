"""Paged-KV decode attention and KV-cache write.

lightserve has no decode-shaped attention operator: ``engine/README.md:142-147``
and ``engine/request.py:86-93`` note that an incremental decode call
(Nq = 1 against a paged Nkv) "is not yet supported by any kernel", and
``model/cuda_graph_decode.py:11-31`` re-runs the full causal forward instead.
These two operators fill that gap. Their results equal the last row of the
reference's causal attention over the cached prefix, and the cache is addressed
through the block tables of ``engine/block_manager.py`` (block i of a request
holds its tokens ``[i*block_size, (i+1)*block_size)``, ``:58-61``).

Cache layout per layer: ``k_cache, v_cache: [num_blocks, H, block_size, D]``.
"""
from __future__ import annotations

import math

import torch

from .. import _lib


def write_kv_cache(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   slot_mapping: torch.Tensor) -> None:
    """Scatters new rows ``k[t], v[t]`` (``[T, H, D]``) into cache slot ``slot_mapping[t]``
    (``block_id * block_size + offset``; negative slots are skipped)."""
    assert k.ndim == 3 and k.shape == v.shape, f"k/v must be [T, H, D], got {tuple(k.shape)}/{tuple(v.shape)}"
    assert k_cache.ndim == 4 and k_cache.shape == v_cache.shape, "caches must be [num_blocks, H, block_size, D]"
    T, H, D = k.shape
    nb, Hc, bs, Dc = k_cache.shape
    assert (Hc, Dc) == (H, D), f"cache heads/dim {(Hc, Dc)} do not match k {(H, D)}"
    assert k.dtype == v.dtype == k_cache.dtype == v_cache.dtype, "k/v/cache dtypes must match"
    assert k.is_cuda and v.is_cuda and k_cache.is_cuda and v_cache.is_cuda and slot_mapping.is_cuda
    assert k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous"
    assert k.stride(2) == 1 and v.stride(2) == 1, "k/v must be contiguous along D"
    assert slot_mapping.dtype == torch.int64 and slot_mapping.shape == (T,) and slot_mapping.is_contiguous()
    lib = _lib.load()
    with _lib.device_guard(k.device):
        rc = lib.lsb_kv_cache_write(
            k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(),
            T, H, D, nb, bs, k.stride(0), k.stride(1), v.stride(0), v.stride(1),
            _lib.dtype_code(k.dtype), _lib.stream_ptr(k.device),
        )
    _lib.check(rc, "lsb_kv_cache_write")


def paged_decode_workspace(q_shape, max_blocks_per_seq: int, block_size: int, device) -> torch.Tensor:
    """fp32 scratch for split-context partials (empty when none is needed)."""
    S, H, D = q_shape
    nbytes = _lib.load().lsb_paged_decode_workspace_size(S, H, D, max_blocks_per_seq, block_size)
    return torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=device)


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor,
                           scale: float | None = None, out: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """o[s, h] = softmax(q[s, h] . K[s, h, :L_s]^T * scale) V[s, h, :L_s].

    q: [S, H, D]; k_cache, v_cache: [num_blocks, H, block_size, D];
    block_tables: int32 [S, max_blocks]; context_lens: int32 [S] (tokens already
    in the cache, including the current one). scale defaults to 1/sqrt(D).
    Passing ``out`` and ``workspace`` makes the call allocation-free (for CUDA
    graph capture).
    """
    assert q.ndim == 3, f"q must be [S, H, D], got {q.ndim}D"
    S, H, D = q.shape
    assert k_cache.ndim == 4 and k_cache.shape == v_cache.shape, "caches must be [num_blocks, H, block_size, D]"
    nb, Hc, bs, Dc = k_cache.shape
    assert (Hc, Dc) == (H, D), f"cache heads/dim {(Hc, Dc)} do not match q {(H, D)}"
    assert q.dtype == k_cache.dtype == v_cache.dtype, "q/cache dtypes must match"
    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda and block_tables.is_cuda and context_lens.is_cuda
    assert k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous"
    assert q.stride(2) == 1, "q must be contiguous along D"
    assert block_tables.dtype == torch.int32 and block_tables.ndim == 2 and block_tables.shape[0] == S
    assert block_tables.is_contiguous(), "block_tables must be contiguous"
    assert context_lens.dtype == torch.int32 and context_lens.shape == (S,) and context_lens.is_contiguous()
    assert bs > 0 and (bs & (bs - 1)) == 0, "block_size must be a power of two"
    max_blocks = block_tables.shape[1]
    if out is None:
        out = torch.empty_like(q)
    assert out.shape == q.shape and out.dtype == q.dtype and out.stride(2) == 1
    lib = _lib.load()
    need = lib.lsb_paged_decode_workspace_size(S, H, D, max_blocks, bs)
    if workspace is None:
        workspace = paged_decode_workspace((S, H, D), max_blocks, bs, q.device)
    assert workspace.numel() * workspace.element_size() >= need, "workspace too small"
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    with _lib.device_guard(q.device):
        rc = lib.lsb_paged_decode(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_tables.data_ptr(),
            context_lens.data_ptr(), out.data_ptr(), S, H, D, max_blocks, bs, nb,
            q.stride(0), q.stride(1), out.stride(0), out.stride(1), float(scale),
            _lib.dtype_code(q.dtype), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
            _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "lsb_paged_decode")
    return out


def rope_kv_write(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor,
                  block_tables: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, context_lens: torch.Tensor | None = None) -> torch.Tensor:
    """One decode step's RoPE + KV-cache write, fused.

    qkv: [S, 3, H, D] (the fused QKV projection); cos/sin: [max_pos, D] tables in
    the model dtype; positions: int64 [S] (position of each sequence's new token);
    block_tables: int32 [S, max_blocks]. Writes rotated q into q_out [S, H, D],
    rotated k and v into the caches at the token's slot, and context_lens[s] =
    positions[s] + 1 when given. Rounding matches lightserve's apply_rope
    (model/minimal_llama.py:167-182) computed with torch ops in the model dtype.
    """
    assert qkv.ndim == 4 and qkv.shape[1] == 3 and qkv.stride(3) == 1, "qkv must be [S, 3, H, D]"
    S, _, H, D = qkv.shape
    assert k_cache.ndim == 4 and k_cache.shape == v_cache.shape and k_cache.is_contiguous()
    nb, Hc, bs, Dc = k_cache.shape
    assert (Hc, Dc) == (H, D)
    assert cos.shape == sin.shape and cos.shape[1] == D and cos.stride() == sin.stride() and cos.stride(1) == 1
    assert qkv.dtype == cos.dtype == sin.dtype == k_cache.dtype == q_out.dtype
    assert q_out.shape == (S, H, D) and q_out.is_contiguous()
    assert positions.dtype == torch.int64 and positions.shape == (S,) and positions.is_contiguous()
    assert block_tables.dtype == torch.int32 and block_tables.is_contiguous() and block_tables.shape[0] == S
    if context_lens is not None:
        assert context_lens.dtype == torch.int32 and context_lens.shape == (S,) and context_lens.is_contiguous()
    lib = _lib.load()
    with _lib.device_guard(qkv.device):
        rc = lib.lsb_rope_kv_write(
            qkv.data_ptr(), qkv.stride(0), qkv.stride(1), qkv.stride(2), cos.data_ptr(), sin.data_ptr(),
            cos.stride(0), positions.data_ptr(), block_tables.data_ptr(), block_tables.shape[1],
            q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(context_lens),
            S, H, D, nb, bs, _lib.dtype_code(qkv.dtype), _lib.stream_ptr(qkv.device),
        )
    _lib.check(rc, "lsb_rope_kv_write")
    return q_out


def rope_kv_write_slots(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                        positions: torch.Tensor, slot_mapping: torch.Tensor, q_out: torch.Tensor,
                        k_out: torch.Tensor | None, k_cache: torch.Tensor,
                        v_cache: torch.Tensor) -> torch.Tensor:
    """Packed-prefill RoPE + KV-cache write: ``rope_kv_write`` for T tokens of any
    sequences, each with its own position (int64 [T]) and cache slot
    (``slot_mapping`` int64 [T], ``block * block_size + offset``; < 0 skips the
    write). Rotated q goes to ``q_out`` and rotated k to ``k_out`` (both
    [T, H, D] contiguous; ``k_out`` optional), as inputs of
    ``flash_attention_varlen``. Same rounding as ``rope_kv_write``."""
    assert qkv.ndim == 4 and qkv.shape[1] == 3 and qkv.stride(3) == 1, "qkv must be [T, 3, H, D]"
    T, _, H, D = qkv.shape
    assert k_cache.ndim == 4 and k_cache.shape == v_cache.shape and k_cache.is_contiguous()
    assert v_cache.is_contiguous()
    nb, Hc, bs, Dc = k_cache.shape
    assert (Hc, Dc) == (H, D)
    assert cos.shape == sin.shape and cos.shape[1] == D and cos.stride() == sin.stride() and cos.stride(1) == 1
    assert qkv.dtype == cos.dtype == sin.dtype == k_cache.dtype == v_cache.dtype == q_out.dtype
    assert q_out.shape == (T, H, D) and q_out.is_contiguous()
    if k_out is not None:
        assert k_out.shape == (T, H, D) and k_out.is_contiguous() and k_out.dtype == q_out.dtype
    assert positions.dtype == torch.int64 and positions.shape == (T,) and positions.is_contiguous()
    assert slot_mapping.dtype == torch.int64 and slot_mapping.shape == (T,) and slot_mapping.is_contiguous()
    lib = _lib.load()
    with _lib.device_guard(qkv.device):
        rc = lib.lsb_rope_kv_write_slots(
            qkv.data_ptr(), qkv.stride(0), qkv.stride(1), qkv.stride(2), cos.data_ptr(), sin.data_ptr(),
            cos.stride(0), positions.data_ptr(), slot_mapping.data_ptr(), q_out.data_ptr(),
            _lib.ptr(k_out), k_cache.data_ptr(), v_cache.data_ptr(), T, H, D, nb, bs,
            _lib.dtype_code(qkv.dtype), _lib.stream_ptr(qkv.device),
        )
    _lib.check(rc, "lsb_rope_kv_write_slots")
    return q_out
