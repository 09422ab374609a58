"""Generates the golden fixtures in tests/golden/ from lightserve's own code.

Run in a container where the lightserve sources are available (path given by
--reference, a required argument); the fixtures it writes are small .npz
files committed next to this script, so tests never need the reference.

What it records:
* attn_*.npz -- lightserve's Triton kernels _flash_attn_fwd_lse_kernel,
  _flash_attn_bwd_preprocess_kernel and _flash_attn_bwd_kernel
  (kernels/flash_attention_backward.py), and the autotuned
  _flash_attn_fwd_kernel (kernels/flash_attention.py), executed by the Triton
  CPU interpreter (TRITON_INTERPRET=1) in fp32 on seeded inputs.
* rmsnorm_*.npz -- _fused_add_rmsnorm_kernel
  (kernels/fused_rmsnorm_residual.py) under the interpreter, fp32.
* llama_toy.npz -- reference_llama_forward (model/minimal_llama.py:253) logits
  and a greedy full-recompute decode on a 2-layer toy config in fp32, with
  weights drawn from a CPU generator in init_weights' order.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent

ATTN_CASES = [  # (B, H, N, D, causal)
    (1, 1, 17, 32, False),
    (1, 1, 17, 32, True),
    (1, 2, 40, 16, True),
    (2, 1, 33, 64, False),
    (1, 1, 70, 64, True),
]
RMS_CASES = [(1, 1), (4, 17), (3, 300), (2, 1024)]


def _seeded(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g, dtype=torch.float32)


def gen_attention(ref):
    from kernels import flash_attention as fa
    from kernels import flash_attention_backward as fab
    import triton

    for i, (B, H, N, D, causal) in enumerate(ATTN_CASES):
        q, k, v, do = (_seeded((B, H, N, D), 100 * i + j) for j in range(4))
        o, L = fab._flash_attention_forward_lse(q, k, v, causal)
        dq, dk, dv = fab._flash_attention_backward(do, q, k, v, o, L, causal)
        # Forward-only autotuned kernel (its wrapper asserts CUDA, so launch directly).
        o2 = torch.empty_like(q)
        BLOCK_D = max(16, triton.next_power_of_2(D))
        # The autotuner cannot benchmark under the interpreter: run the jitted
        # function with the config its fp32 prune keeps (32x32, kernels/flash_attention.py:71-72).
        fa._flash_attn_fwd_kernel.fn[(triton.cdiv(N, 32), B * H)](
            q, k, v, o2, *q.stride(), *k.stride(), *v.stride(), *o2.stride(), H, N, D,
            1.0 / D ** 0.5, CAUSAL=causal, BLOCK_M=32, BLOCK_N=32, BLOCK_D=BLOCK_D)
        name = f"attn_b{B}h{H}n{N}d{D}{'_causal' if causal else ''}.npz"
        np.savez_compressed(HERE / name, q=q.numpy(), k=k.numpy(), v=v.numpy(), do=do.numpy(),
                            o=o.numpy(), lse=L.numpy(), o_fwd_only=o2.numpy(), dq=dq.numpy(),
                            dk=dk.numpy(), dv=dv.numpy(), causal=np.array(causal))
        print("wrote", name)


def gen_rmsnorm(ref):
    from kernels import fused_rmsnorm_residual as fr
    import triton

    for i, (M, N) in enumerate(RMS_CASES):
        x, r = _seeded((M, N), 7 * i), _seeded((M, N), 7 * i + 1)
        w = 1.0 + 0.02 * _seeded((N,), 7 * i + 2)
        out, h = torch.empty_like(x), torch.empty_like(x)
        BLOCK_N = triton.next_power_of_2(N)
        fr._fused_add_rmsnorm_kernel[(M,)](x, r, w, out, h, N, x.stride(0), r.stride(0),
                                           out.stride(0), h.stride(0), 1e-6, BLOCK_N=BLOCK_N)
        name = f"rmsnorm_m{M}n{N}.npz"
        np.savez_compressed(HERE / name, x=x.numpy(), r=r.numpy(), w=w.numpy(), out=out.numpy(),
                            h=h.numpy(), eps=np.array(1e-6))
        print("wrote", name)


def toy_weights(mm, cfg, seed=0):
    """init_weights' draw order with a CPU generator (fp32)."""
    g = torch.Generator().manual_seed(seed)

    def randn(*s):
        return (torch.randn(*s, generator=g, dtype=torch.float32) * 0.02).to(cfg.dtype)

    def ones(*s):
        return torch.ones(*s, dtype=cfg.dtype)

    H, I, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    layers = [mm.LayerWeights(ones(H), randn(H, H), randn(H, H), randn(H, H), randn(H, H), ones(H),
                              randn(H, I), randn(H, I), randn(I, H)) for _ in range(cfg.n_layers)]
    return mm.LlamaWeights(embed_tokens=randn(V, H), layers=layers, norm_weight=ones(H),
                           lm_head=randn(H, V))


def gen_llama(ref):
    from model import minimal_llama as mm

    cfg = mm.LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=688, n_layers=2,
                         n_heads=4, head_dim=64, max_seq_len=64, rope_theta=10000.0,
                         dtype=torch.float32)
    w = toy_weights(mm, cfg)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 19, 33)]
    steps = 12
    tokens, margins = [], []
    with torch.no_grad():
        for p in prompts:
            ids = list(p)
            out, marg = [], []
            for _ in range(steps):
                logits = mm.reference_llama_forward(w, cfg, torch.tensor([ids]))[0, -1]
                t2 = torch.topk(logits, 2).values
                marg.append(float(t2[0] - t2[1]))
                out.append(int(logits.argmax()))
                ids.append(out[-1])
            tokens.append(out)
            margins.append(marg)
        logits0 = mm.reference_llama_forward(w, cfg, torch.tensor([prompts[1]]))
    pad = max(len(p) for p in prompts)
    P = np.full((len(prompts), pad), -1, np.int64)
    for i, p in enumerate(prompts):
        P[i, : len(p)] = p
    np.savez_compressed(HERE / "llama_toy.npz", prompts=P, prompt_lens=np.array([len(p) for p in prompts]),
                        tokens=np.array(tokens), margins=np.array(margins),
                        logits_prompt1=logits0.numpy())
    print("wrote llama_toy.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the lightserve source tree")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    gen_attention(args.reference)
    gen_rmsnorm(args.reference)
    gen_llama(args.reference)


if __name__ == "__main__":
    main()
