"""Attention oracle (test infrastructure only; see oracle/__init__.py).

Two restatements of lightserve's attention:

* ``flash_fwd_tiled`` / ``flash_bwd_tiled`` -- numpy, loop-for-loop the tiled
  algorithm of lightserve's Triton kernels: online softmax over K/V tiles with
  causal early exit (kernels/flash_attention.py:129-175; with the LSE write of
  kernels/flash_attention_backward.py:162-169), and the recomputation backward
  (kernels/flash_attention_backward.py:202-330). Exact fp32 arithmetic; for
  small cases.
* ``attention_ref`` / ``attention_ref_grads`` -- dense PyTorch-CPU fp32
  (materialised softmax), the reference's own comparison target
  (F.scaled_dot_product_attention in kernels/tests/test_flash_attention.py:47
  and kernels/tests/test_flash_attention_backward.py:79-87). Used at larger
  sizes and as the timed CPU baseline.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def flash_fwd_tiled(q, k, v, causal: bool, block_m: int = 32, block_n: int = 32):
    """q, k, v: float arrays [B, H, N, D]. Returns (o [B,H,N,D] f32, lse [B,H,N] f32).

    Follows _flash_attn_fwd_lse_kernel (kernels/flash_attention_backward.py:
    88-169): s = q.k * scale (:135), mask outside [0,N) and above the diagonal
    (:137-140), m_new = max(m, rowmax) (:142-143), p = exp(s - m_new),
    alpha = exp(m - m_new) (:144-145), l = alpha*l + rowsum(p) (:147),
    acc = acc*alpha + p.v (:153), o = acc / l (:156), L = m + log(l) (:161).
    """
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32); v = np.asarray(v, np.float32)
    B, H, N, D = q.shape
    scale = np.float32(1.0 / math.sqrt(D))
    o = np.zeros((B, H, N, D), np.float32)
    lse = np.zeros((B, H, N), np.float32)
    for b in range(B):
        for h in range(H):
            for m0 in range(0, N, block_m):
                rows = np.arange(m0, min(m0 + block_m, N))
                qi = q[b, h, rows]
                m_i = np.full(len(rows), -np.inf, np.float32)
                l_i = np.zeros(len(rows), np.float32)
                acc = np.zeros((len(rows), D), np.float32)
                hi = min(N, m0 + block_m) if causal else N  # causal early exit (:133)
                for n0 in range(0, hi, block_n):
                    cols = np.arange(n0, min(n0 + block_n, N))
                    s = (qi @ k[b, h, cols].T) * scale
                    if causal:
                        s = np.where(rows[:, None] >= cols[None, :], s, -np.inf)
                    m_new = np.maximum(m_i, s.max(axis=1))
                    p = np.exp(s - m_new[:, None])
                    alpha = np.exp(m_i - m_new)
                    l_i = alpha * l_i + p.sum(axis=1)
                    acc = acc * alpha[:, None] + p @ v[b, h, cols]
                    m_i = m_new
                o[b, h, rows] = acc / l_i[:, None]
                lse[b, h, rows] = m_i + np.log(l_i)
    return o, lse


def flash_bwd_tiled(q, k, v, o, do, lse, causal: bool, block_m: int = 32, block_n: int = 32):
    """Returns (dq, dk, dv) as f32 arrays [B,H,N,D].

    Follows kernels/flash_attention_backward.py: Dsum = rowsum(dO*O) (:226);
    per K/V tile j, Q tiles from lo = floor(j*BN/BM)*BM when causal (:290);
    P = exp(s - L) with masked entries 0 (:314); dV += P^T dO (:316);
    dP = dO V^T (:318); dS = P (dP - Dsum) (:319); dK += dS^T Q * scale (:321);
    dQ += dS K * scale (:323-325).
    """
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32); v = np.asarray(v, np.float32)
    o = np.asarray(o, np.float32); do = np.asarray(do, np.float32); lse = np.asarray(lse, np.float32)
    B, H, N, D = q.shape
    scale = np.float32(1.0 / math.sqrt(D))
    dsum = (o * do).sum(axis=-1)
    dq = np.zeros_like(q); dk = np.zeros_like(k); dv = np.zeros_like(v)
    for b in range(B):
        for h in range(H):
            for n0 in range(0, N, block_n):
                cols = np.arange(n0, min(n0 + block_n, N))
                kj, vj = k[b, h, cols], v[b, h, cols]
                dk_acc = np.zeros((len(cols), D), np.float32)
                dv_acc = np.zeros((len(cols), D), np.float32)
                lo = (n0 // block_m) * block_m if causal else 0
                for m0 in range(lo, N, block_m):
                    rows = np.arange(m0, min(m0 + block_m, N))
                    s = (q[b, h, rows] @ kj.T) * scale
                    p = np.exp(s - lse[b, h, rows][:, None])
                    if causal:
                        p = np.where(rows[:, None] >= cols[None, :], p, 0.0).astype(np.float32)
                    dv_acc += p.T @ do[b, h, rows]
                    dp = do[b, h, rows] @ vj.T
                    ds = p * (dp - dsum[b, h, rows][:, None])
                    dk_acc += (ds.T @ q[b, h, rows]) * scale
                    dq[b, h, rows] += (ds @ kj) * scale
                dk[b, h, cols] = dk_acc
                dv[b, h, cols] = dv_acc
    return dq, dk, dv


def attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                  return_lse: bool = False):
    """Dense fp32 attention on CPU tensors [B,H,N,D] (any float dtype in, fp32 out)."""
    q32, k32, v32 = (t.detach().to("cpu", torch.float32) for t in (q, k, v))
    D = q32.shape[-1]
    s = (q32 @ k32.transpose(-1, -2)) * (1.0 / math.sqrt(D))
    if causal:
        N = s.shape[-1]
        mask = torch.ones(N, N, dtype=torch.bool).tril()
        s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ v32
    return (o, lse) if return_lse else o


def attention_ref_grads(q, k, v, do, causal: bool):
    """(dq, dk, dv) of attention_ref under upstream gradient do, fp32 on CPU."""
    q32, k32, v32 = (t.detach().to("cpu", torch.float32).requires_grad_() for t in (q, k, v))
    o = _dense(q32, k32, v32, causal)
    o.backward(do.detach().to("cpu", torch.float32))
    return q32.grad, k32.grad, v32.grad


def _dense(q, k, v, causal):
    D = q.shape[-1]
    s = (q @ k.transpose(-1, -2)) * (1.0 / math.sqrt(D))
    if causal:
        N = s.shape[-1]
        s = s.masked_fill(~torch.ones(N, N, dtype=torch.bool).tril(), float("-inf"))
    return torch.softmax(s, dim=-1) @ v


def attn_fwd_flops(B, H, N, D, causal: bool) -> float:
    """lightserve's convention (kernels/benchmark_flash_attention.py:55-64)."""
    f = 4.0 * B * H * N * N * D
    return f / 2 if causal else f


def attn_bwd_flops(B, H, N, D, causal: bool) -> float:
    """2.5 x forward (kernels/benchmark_flash_attention_backward.py:59-68)."""
    return 2.5 * attn_fwd_flops(B, H, N, D, causal)
