"""Seeded single-kernel workloads for profiler captures.

``python -m lightserve_b200.profile_cases CASE [--reps R] [shape options]``
runs one operator R times on seeded N(0,1) inputs and synchronises, so a
profiler (e.g. ``ncu -k regex:<kernel> -s 1 -c 1``) can capture a warm
launch of exactly that kernel. Cases:

* ``fwd``     causal flash_attention_forward, [B, H, N, D] bf16
* ``bwd``     causal backward (_flash_attention_backward), LSE from the forward
* ``varlen``  causal flash_attention_varlen over ``--lens`` packed sequences
* ``rmsnorm`` fused_add_rmsnorm on [M, N] bf16
* ``decode``  paged_decode_attention, S sequences with contexts U[lo, hi]
* ``linear``  lsb_linear, x [S, K] @ W [K, N] bf16 (weight packed once)
* ``greedy``  greedy_next over [S, N] bf16 logits
"""
from __future__ import annotations

import argparse

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["fwd", "bwd", "varlen", "rmsnorm", "decode", "linear", "greedy"])
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--B", type=int, default=2)
    ap.add_argument("--H", type=int, default=32)
    ap.add_argument("--N", type=int, default=2048)
    ap.add_argument("--D", type=int, default=128)
    ap.add_argument("--M", type=int, default=16384)
    ap.add_argument("--lens", default="4096,1000,3000,77,2048,4096,513,1")
    ap.add_argument("--S", type=int, default=64)
    ap.add_argument("--ctx", default="512,4096")
    a = ap.parse_args(argv)
    from lightserve_b200.kernels import (flash_attention_forward, flash_attention_varlen, fused_add_rmsnorm,
                                         paged_decode_attention)
    from lightserve_b200.kernels.flash_attention_backward import (_flash_attention_backward,
                                                                  _flash_attention_forward_lse)
    g = torch.Generator(device="cuda").manual_seed(0)
    bf = torch.bfloat16

    def rn(*shape):
        return torch.randn(*shape, device="cuda", dtype=bf, generator=g)

    if a.case in ("fwd", "bwd"):
        q, k, v = (rn(a.B, a.H, a.N, a.D) for _ in range(3))
        if a.case == "fwd":
            run = lambda: flash_attention_forward(q, k, v, causal=True)  # noqa: E731
        else:
            do = rn(a.B, a.H, a.N, a.D)
            o, L = _flash_attention_forward_lse(q, k, v, True)
            run = lambda: _flash_attention_backward(do, q, k, v, o, L, True)  # noqa: E731
    elif a.case == "varlen":
        lens = [int(x) for x in a.lens.split(",")]
        T = sum(lens)
        q, k, v = (rn(T, a.H, a.D) for _ in range(3))
        cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
        run = lambda: flash_attention_varlen(q, k, v, cu, max(lens), causal=True)  # noqa: E731
    elif a.case == "linear":
        from lightserve_b200.kernels import linear, pack_linear_weight
        x = rn(a.S, a.D)  # K = --D
        pw = pack_linear_weight((0.02 * rn(a.N, a.D)).contiguous())
        out = torch.empty(a.S, a.N, device="cuda", dtype=bf)
        run = lambda: linear(x, pw, out=out)  # noqa: E731
    elif a.case == "greedy":
        from lightserve_b200.kernels import greedy_next
        logits = rn(a.S, a.N)
        tok = torch.empty(a.S, dtype=torch.int64, device="cuda")
        run = lambda: greedy_next(logits, tok)  # noqa: E731
    elif a.case == "rmsnorm":
        x, r = rn(a.M, a.N), rn(a.M, a.N)
        w = (1 + 0.02 * torch.randn(a.N, device="cuda", generator=g)).to(bf)
        run = lambda: fused_add_rmsnorm(x, r, w, 1e-6)  # noqa: E731
    else:
        lo, hi = (int(x) for x in a.ctx.split(","))
        bs, H, D = 16, a.H, a.D
        lens = torch.randint(lo, hi + 1, (a.S,), generator=torch.Generator().manual_seed(0))
        mb = -(-hi // bs)
        nb = a.S * mb
        kc, vc = rn(nb, H, bs, D), rn(nb, H, bs, D)
        table = torch.randperm(nb, generator=torch.Generator().manual_seed(1)).view(a.S, mb)
        table = table.to(torch.int32).cuda()
        ctx = lens.to(torch.int32).cuda()
        q = rn(a.S, H, D)
        run = lambda: paged_decode_attention(q, kc, vc, table, ctx)  # noqa: E731
    for _ in range(a.reps):
        run()
    torch.cuda.synchronize()
    print(f"{a.case}: {a.reps} launches done")


if __name__ == "__main__":
    main()
