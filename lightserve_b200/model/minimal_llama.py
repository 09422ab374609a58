"""LLaMA-shaped decoder (plain MHA) built on lightserve_b200's operators.

Same architecture, weight layout and arithmetic order as lightserve's
``model/minimal_llama.py``:

* ``LlamaConfig`` (``:50-69``): MHA only, ``hidden == n_heads * head_dim``;
* weights stored ``[in_features, out_features]`` (``:20-24``), N(0, 0.02)
  projections and unit norm weights (``:109-143``);
* rotate-half RoPE with cos/sin tables in the model dtype (``:146-175``);
* pre-norm residual stream driven through ``fused_add_rmsnorm`` starting from a
  zero ``x`` (``:199-205``), final norm over ``x + residual`` (``:236-249``).

Differences, on purpose:

* ``init_weights`` draws from a CPU ``torch.Generator`` and then moves the
  tensors, so the same seed gives bit-identical weights on any device (the
  reference seeds a device generator, ``:113``, so CPU and CUDA differ);
* the Linears are ``torch.matmul`` (cuBLAS): lightserve's Triton GEMM is not
  part of this hot path.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..kernels.flash_attention import flash_attention_forward
from ..kernels.fused_rmsnorm_residual import fused_add_rmsnorm


@dataclass
class LlamaConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    n_layers: int
    n_heads: int
    head_dim: int
    max_seq_len: int
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5
    dtype: torch.dtype = torch.bfloat16

    def __post_init__(self):
        assert self.hidden_size == self.n_heads * self.head_dim, (
            f"hidden_size ({self.hidden_size}) must equal n_heads*head_dim "
            f"({self.n_heads}*{self.head_dim}) -- plain MHA only"
        )


TOY_CONFIG = LlamaConfig(
    vocab_size=256, hidden_size=256, intermediate_size=688,
    n_layers=2, n_heads=4, head_dim=64, max_seq_len=64,
)


def decode_bench_config(max_seq_len: int = 4224, dtype: torch.dtype = torch.bfloat16) -> LlamaConfig:
    """The paged-decode benchmark model: 8 layers, hidden 2048 (16 x 128),
    SwiGLU 5632, vocab 32000, RoPE theta 10000."""
    return LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632, n_layers=8,
                       n_heads=16, head_dim=128, max_seq_len=max_seq_len, rope_theta=10000.0,
                       dtype=dtype)


@dataclass
class LayerWeights:
    input_layernorm_weight: torch.Tensor
    q_proj: torch.Tensor
    k_proj: torch.Tensor
    v_proj: torch.Tensor
    o_proj: torch.Tensor
    post_attention_layernorm_weight: torch.Tensor
    gate_proj: torch.Tensor
    up_proj: torch.Tensor
    down_proj: torch.Tensor


@dataclass
class LlamaWeights:
    embed_tokens: torch.Tensor
    layers: list = field(default_factory=list)
    norm_weight: torch.Tensor = None
    lm_head: torch.Tensor = None


def init_weights(config: LlamaConfig, device="cuda", seed: int = 0) -> LlamaWeights:
    """N(0, 0.02) projections, unit norm weights; drawn in the reference's order
    (per layer q, k, v, o, gate, up, down; then embedding, then lm_head)."""
    g = torch.Generator(device="cpu").manual_seed(seed)

    def randn(*shape):
        t = torch.randn(*shape, generator=g, dtype=torch.float32) * 0.02
        return t.to(config.dtype).to(device)

    def ones(*shape):
        return torch.ones(*shape, dtype=config.dtype, device=device)

    H, I, V = config.hidden_size, config.intermediate_size, config.vocab_size
    qkv = config.n_heads * config.head_dim
    layers = []
    for _ in range(config.n_layers):
        layers.append(LayerWeights(
            input_layernorm_weight=ones(H),
            q_proj=randn(H, qkv), k_proj=randn(H, qkv), v_proj=randn(H, qkv),
            o_proj=randn(qkv, H),
            post_attention_layernorm_weight=ones(H),
            gate_proj=randn(H, I), up_proj=randn(H, I), down_proj=randn(I, H),
        ))
    return LlamaWeights(embed_tokens=randn(V, H), layers=layers, norm_weight=ones(H),
                        lm_head=randn(H, V))


def precompute_rope(config: LlamaConfig, device):
    """cos/sin tables [max_seq_len, head_dim] in the model dtype."""
    half = config.head_dim // 2
    inv_freq = 1.0 / (config.rope_theta ** (
        torch.arange(0, half, device=device, dtype=torch.float32) / half))
    pos = torch.arange(config.max_seq_len, device=device, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    cos = torch.cat([freqs.cos(), freqs.cos()], dim=-1).to(config.dtype)
    sin = torch.cat([freqs.sin(), freqs.sin()], dim=-1).to(config.dtype)
    return cos, sin


def rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([-x2, x1], dim=-1)


def apply_rope(q, k, cos_n, sin_n):
    """q, k and cos_n/sin_n broadcastable to each other (head_dim last)."""
    return q * cos_n + rotate_half(q) * sin_n, k * cos_n + rotate_half(k) * sin_n


def llama_forward(weights: LlamaWeights, config: LlamaConfig, input_ids: torch.Tensor,
                  causal: bool = True, kv_sink=None, last_only: bool = False) -> torch.Tensor:
    """Prefill forward: input_ids [B, N] -> logits [B, N, vocab] ([B, 1, vocab]
    with ``last_only``, which applies the final norm and lm_head to the last
    position only).

    ``kv_sink(layer_idx, k, v)``, when given, receives each layer's post-RoPE
    keys and values ``[B, H, N, D]`` (used to fill the paged KV cache).
    """
    B, N = input_ids.shape
    Hd = config.hidden_size
    cos, sin = precompute_rope(config, input_ids.device)
    cos_n = cos[:N].view(1, 1, N, -1)
    sin_n = sin[:N].view(1, 1, N, -1)

    residual = F.embedding(input_ids, weights.embed_tokens).reshape(B * N, Hd)
    x = torch.zeros_like(residual)
    for li, layer in enumerate(weights.layers):
        normed, residual = fused_add_rmsnorm(x, residual, layer.input_layernorm_weight, eps=config.rms_eps)
        q = (normed @ layer.q_proj).view(B, N, config.n_heads, config.head_dim).transpose(1, 2)
        k = (normed @ layer.k_proj).view(B, N, config.n_heads, config.head_dim).transpose(1, 2)
        v = (normed @ layer.v_proj).view(B, N, config.n_heads, config.head_dim).transpose(1, 2)
        q, k = apply_rope(q, k, cos_n, sin_n)
        if kv_sink is not None:
            kv_sink(li, k, v)
        attn = flash_attention_forward(q, k, v, causal=causal)
        attn = attn.transpose(1, 2).reshape(B * N, Hd)
        x = attn @ layer.o_proj
        normed2, residual = fused_add_rmsnorm(x, residual, layer.post_attention_layernorm_weight,
                                              eps=config.rms_eps)
        x = (F.silu(normed2 @ layer.gate_proj) * (normed2 @ layer.up_proj)) @ layer.down_proj
    if last_only:
        x = x.view(B, N, Hd)[:, -1].contiguous()
        residual = residual.view(B, N, Hd)[:, -1].contiguous()
        N = 1
    final, _ = fused_add_rmsnorm(x, residual, weights.norm_weight, eps=config.rms_eps)
    return (final @ weights.lm_head).view(B, N, config.vocab_size)
