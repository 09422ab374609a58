"""Decode oracle (test infrastructure only; see oracle/__init__.py).

* ``reference_forward`` restates lightserve's ``reference_llama_forward``
  (model/minimal_llama.py:253-293): F.linear with the [in, out] weights
  transposed, rotate-half RoPE (:146-182), SDPA-equivalent causal attention,
  ``rmsnorm(h) = (float(h) * rsqrt(mean(float(h)^2) + eps)).to(dtype) * w``
  (:265-268), ``residual = residual + x`` after each sublayer (:281, :288).
* ``greedy_full_recompute`` restates the decode loop of
  model/cuda_graph_decode.py:108-118: every step re-runs the full forward over
  the whole sequence and appends ``argmax`` of the newest position's logits.
* ``paged_decode_ref`` is the single-query attention of one decode step,
  gathering each sequence's K/V from a paged cache through its block table
  (engine/block_manager.py:58-61: block i holds tokens [i*bs, (i+1)*bs)).

Weights are any object with lightserve's LlamaWeights / LayerWeights fields.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _rope_tables(cfg, device="cpu"):
    half = cfg.head_dim // 2
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, half, dtype=torch.float32) / half))
    pos = torch.arange(cfg.max_seq_len, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    cos = torch.cat([freqs.cos(), freqs.cos()], dim=-1).to(cfg.dtype)
    sin = torch.cat([freqs.sin(), freqs.sin()], dim=-1).to(cfg.dtype)
    return cos.to(device), sin.to(device)


def _rot(x):
    a, b = x.chunk(2, dim=-1)
    return torch.cat([-b, a], dim=-1)


def _attn(q, k, v):
    N, D = q.shape[-2], q.shape[-1]
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(D)
    s = s.masked_fill(~torch.ones(N, N, dtype=torch.bool, device=q.device).tril(), float("-inf"))
    return (torch.softmax(s, dim=-1) @ v.float()).to(q.dtype)


def reference_forward(weights, cfg, input_ids: torch.Tensor) -> torch.Tensor:
    """input_ids [B, N] (CPU) -> logits [B, N, vocab] in cfg.dtype."""
    B, N = input_ids.shape
    dev = input_ids.device
    cos, sin = _rope_tables(cfg, dev)
    cos_n, sin_n = cos[:N].view(1, 1, N, -1), sin[:N].view(1, 1, N, -1)

    def rmsnorm(h, w):
        hf = h.float()
        return (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + cfg.rms_eps)).to(h.dtype) * w

    def lin(x, w):
        return F.linear(x, w.t())

    residual = F.embedding(input_ids, weights.embed_tokens)
    for layer in weights.layers:
        h = rmsnorm(residual, layer.input_layernorm_weight)
        q = lin(h, layer.q_proj).view(B, N, cfg.n_heads, cfg.head_dim).transpose(1, 2)
        k = lin(h, layer.k_proj).view(B, N, cfg.n_heads, cfg.head_dim).transpose(1, 2)
        v = lin(h, layer.v_proj).view(B, N, cfg.n_heads, cfg.head_dim).transpose(1, 2)
        q, k = q * cos_n + _rot(q) * sin_n, k * cos_n + _rot(k) * sin_n
        a = _attn(q, k, v).transpose(1, 2).reshape(B, N, cfg.hidden_size)
        residual = residual + lin(a, layer.o_proj)
        h2 = rmsnorm(residual, layer.post_attention_layernorm_weight)
        residual = residual + lin(F.silu(lin(h2, layer.gate_proj)) * lin(h2, layer.up_proj),
                                  layer.down_proj)
    return lin(rmsnorm(residual, weights.norm_weight), weights.lm_head)


def greedy_full_recompute(weights, cfg, prompt: list, num_tokens: int, return_margins=False):
    """Greedy tokens after `prompt` by full recompute each step (CPU)."""
    ids = list(prompt)
    out, margins = [], []
    for _ in range(num_tokens):
        logits = reference_forward(weights, cfg, torch.tensor([ids], dtype=torch.int64))[0, -1].float()
        top2 = torch.topk(logits, 2).values
        margins.append(float(top2[0] - top2[1]))
        t = int(logits.argmax())
        out.append(t)
        ids.append(t)
    return (out, margins) if return_margins else out


def paged_decode_ref(q, k_cache, v_cache, block_tables, context_lens, scale=None):
    """q [S,H,D]; caches [num_blocks,H,bs,D]; returns fp32 [S,H,D] on CPU."""
    q = q.detach().cpu().float()
    kc, vc = k_cache.detach().cpu().float(), v_cache.detach().cpu().float()
    bt, cl = block_tables.detach().cpu(), context_lens.detach().cpu()
    S, H, D = q.shape
    bs = kc.shape[2]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    out = torch.zeros(S, H, D)
    for s in range(S):
        L = int(cl[s])
        if L == 0:
            continue
        pos = torch.arange(L)
        blk = bt[s, pos // bs].long()
        off = pos % bs
        K = kc[blk, :, off]  # [L, H, D]
        V = vc[blk, :, off]
        sc = torch.einsum("hd,lhd->hl", q[s], K) * scale
        p = torch.softmax(sc, dim=-1)
        out[s] = torch.einsum("hl,lhd->hd", p, V)
    return out
