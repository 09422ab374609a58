"""Benchmark of lightserve_b200's attention hot path on B200.

Headline: causal FlashAttention forward, bf16,
B=4 H=32 N=4096 D=128, seeded N(0,1) inputs, TFLOP/s with lightserve's FLOP
convention 4*B*H*N^2*D/2 (kernels/benchmark_flash_attention.py:55-64).
Secondary lines in the same JSON object: FA backward (config 3), fused
add+RMSNorm (config 4) and paged greedy decode tokens/s (config 5).

Multi-GPU: one process per GPU (torchrun); every rank runs the full per-GPU
workload on its own (batch x head) slices -- independent units, no
collective on the data path ("scaling": "weak"); times are the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FWD_CFG = dict(B=4, H=32, N=4096, D=128, causal=True)
BWD_CFG = dict(B=4, H=32, N=2048, D=128, causal=True)
RMS_CFG = dict(M=16384, N=4096)
DEC_CFG = dict(S=64, steps=128, ctx_lo=512, ctx_hi=4096, block_size=16)


# ----------------------------------------------------------------- plumbing --
@contextlib.contextmanager
def _stdout_to_stderr():
    """Sends file-descriptor-level stdout to stderr (NCCL prints its version
    banner on stdout when the communicator comes up; stdout carries only the
    JSON line)."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        with _stdout_to_stderr():
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            dist.barrier()
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, ws, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    from lightserve_b200.sharding import max_over_ranks as _m

    return _m(x) if ws > 1 else x


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic():
    """Per-launch DRAM bytes from committed ncu summaries (profiles/traffic.json)."""
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while a region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx, self.samples, self._stop = gpu_index, [], threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([s.strip() for s in out.split(",")])
            except Exception:  # noqa: BLE001 -- sampling is best effort
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 4 + i and s[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def time_cuda(fn, steps: int, warmup: int, ws: int):
    """Warm-up, then EXACTLY `steps` calls bracketed by barrier + synchronize;
    returns (max-over-ranks total ms, per-call event ms list)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s)
    for a, b in evs:
        a.record(s)
        fn()
        b.record(s)
    t1.record(s)
    torch.cuda.synchronize()
    barrier(ws)
    total = max_over_ranks(t0.elapsed_time(t1), ws)
    return total, [a.elapsed_time(b) for a, b in evs]


# ---------------------------------------------------------------- workloads --
def attn_fwd_flops(B, H, N, D, causal: bool) -> float:
    """lightserve's convention (kernels/benchmark_flash_attention.py:55-64)."""
    f = 4.0 * B * H * N * N * D
    return f / 2 if causal else f


def attn_bwd_flops(B, H, N, D, causal: bool) -> float:
    """2.5 x forward (kernels/benchmark_flash_attention_backward.py:59-68)."""
    return 2.5 * attn_fwd_flops(B, H, N, D, causal)


def rmsnorm_bytes(M, N, elem_bytes) -> int:
    """Read x, residual; write out, h (kernels/benchmark_fused_rmsnorm_residual.py:59-64)."""
    return 4 * M * N * elem_bytes


def _randn(shape, dtype, gen):
    return torch.randn(*shape, device="cuda", dtype=torch.float32, generator=gen).to(dtype)


def bench_fwd(steps, warmup, ws, rank, peaks, e2e_steps, strong=False):
    from lightserve_b200.kernels import flash_attention_forward, flash_attention_forward_host
    from lightserve_b200.sharding import shard_range

    c = FWD_CFG
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    if strong:  # this rank's contiguous share of the B*H (b, h) slices
        a, b = shard_range(c["B"] * c["H"], rank, ws)
        shape = (1, b - a, c["N"], c["D"])
    else:       # every rank runs the full config on its own slices
        shape = (c["B"], c["H"], c["N"], c["D"])
    q, k, v = (_randn(shape, torch.bfloat16, gen) for _ in range(3))
    flops = attn_fwd_flops(shape[0], shape[1], c["N"], c["D"], c["causal"])
    mult = 1 if strong else ws  # whole-job work = per-rank work x ranks (weak)
    total_ms, per = time_cuda(lambda: flash_attention_forward(q, k, v, causal=True), steps, warmup, ws)
    ms = total_ms / steps
    kern_ms = statistics.mean(per)

    # End to end through the public API with host buffers: pinned q, k, v in
    # host memory, the output back in host memory (flash_attention_forward_host
    # streams (b, h) chunks: copies in both directions overlap the kernel).
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = torch.empty_like(hq).pin_memory()

    def e2e_step():
        flash_attention_forward_host(hq, hk, hv, causal=True, out=ho, device=q.device)

    e2e_total, _ = time_cuda(e2e_step, e2e_steps, 1, ws)
    nb = q.numel() * q.element_size()
    return {
        "ms": ms, "kernel_ms": kern_ms, "flops": flops,
        "value": (attn_fwd_flops(c["B"], c["H"], c["N"], c["D"], True) if strong else mult * flops)
        / (ms * 1e-3) / 1e12,
        "kernel_tflops": flops / (kern_ms * 1e-3) / 1e12,
        "e2e": {"value": (attn_fwd_flops(c["B"], c["H"], c["N"], c["D"], True) if strong else mult * flops)
                / (e2e_total / e2e_steps * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": 3 * nb, "d2h_bytes_per_step": nb, "steps": e2e_steps},
        "launches_per_step": 1,
    }


def bench_bwd(steps, warmup, ws, rank):
    from lightserve_b200.kernels.flash_attention_backward import (_flash_attention_backward,
                                                                  _flash_attention_forward_lse)

    c = BWD_CFG
    gen = torch.Generator(device="cuda").manual_seed(2000 + rank)
    q, k, v, do = (_randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen) for _ in range(4))
    o, L = _flash_attention_forward_lse(q, k, v, True)
    flops = attn_bwd_flops(c["B"], c["H"], c["N"], c["D"], True)
    total_ms, per = time_cuda(lambda: _flash_attention_backward(do, q, k, v, o, L, True), steps, warmup, ws)
    ms = total_ms / steps
    return {"ms": ms, "flops": flops, "value": ws * flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "launches_per_step": 3}


def bench_rmsnorm(steps, warmup, ws, rank):
    from lightserve_b200.kernels import fused_add_rmsnorm

    c = RMS_CFG
    gen = torch.Generator(device="cuda").manual_seed(3000 + rank)
    x = _randn((c["M"], c["N"]), torch.bfloat16, gen)
    r = _randn((c["M"], c["N"]), torch.bfloat16, gen)
    w = (1 + 0.02 * torch.randn(c["N"], device="cuda", generator=gen)).to(torch.bfloat16)
    nbytes = rmsnorm_bytes(c["M"], c["N"], 2)
    total_ms, per = time_cuda(lambda: fused_add_rmsnorm(x, r, w, 1e-6), steps, warmup, ws)
    ms = total_ms / steps
    return {"ms": ms, "bytes": nbytes, "value": ws * nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "kernel_ms": statistics.mean(per), "launches_per_step": 1}


def bench_serving(ws, rank, max_tokens=64):
    """Continuous batching end to end (ServingEngine: scheduler, packed
    prefill, CUDA-graph paged decode, host-side token handling each step) on
    config 5's model and prompt set: all 64 requests submitted at once, each
    generating max_tokens tokens. Timed on the host around run(), after one
    warm-up run of the same requests."""
    from lightserve_b200.engine import CacheConfig, Request, SamplingParams, SchedulerConfig
    from lightserve_b200.model.minimal_llama import decode_bench_config, init_weights
    from lightserve_b200.model.serving import ServingEngine

    c = DEC_CFG
    cfg = decode_bench_config()
    w = init_weights(cfg, device="cuda", seed=0)
    g = torch.Generator().manual_seed(rank)
    lens = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["S"],), generator=g).tolist()
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    bs = c["block_size"]
    blocks = sum(-(-(n + max_tokens) // bs) for n in lens) + 8
    eng = ServingEngine(w, cfg, CacheConfig(block_size=bs, num_gpu_blocks=blocks),
                        SchedulerConfig(max_num_seqs=c["S"], max_num_batched_tokens=sum(lens)))
    times = []
    for it in range(2):
        for i, p in enumerate(prompts):
            eng.add_request(Request(f"run{it}-{i}", p, SamplingParams(max_tokens=max_tokens)))
        torch.cuda.synchronize()
        barrier(ws)
        t0 = time.perf_counter()
        out = eng.run()
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
        assert len(out) == c["S"] and all(len(v) == max_tokens for v in out.values())
    el = max_over_ranks(times[-1], ws)
    gen = c["S"] * max_tokens
    return {"seconds": el, "requests": c["S"], "prompt_tokens": sum(lens), "generated_tokens": gen,
            "value": ws * gen / el, "unit": "generated tokens/s",
            "total_tokens_per_s": ws * (gen + sum(lens)) / el,
            "note": "host-timed ServingEngine.run(): prefill of every prompt, then decode steps"}


def bench_varlen(steps, warmup, ws, rank):
    """Packed (variable-length) causal attention over config 5's prompt set:
    64 sequences with lengths U[512, 4096], 16 heads x 128, bf16 -- one
    layer's prefill attention."""
    from lightserve_b200.kernels import flash_attention_varlen

    c = DEC_CFG
    g = torch.Generator().manual_seed(rank)
    lens = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["S"],), generator=g).tolist()
    T, H, D = sum(lens), 16, 128
    gen = torch.Generator(device="cuda").manual_seed(2000 + rank)
    q, k, v = (_randn((T, H, D), torch.bfloat16, gen) for _ in range(3))
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    total_ms, _ = time_cuda(lambda: flash_attention_varlen(q, k, v, cu, max(lens), causal=True, out=out),
                            steps, warmup, ws)
    ms = total_ms / steps
    flops = sum(attn_fwd_flops(1, H, n, D, True) for n in lens)
    return {"ms": ms, "flops": flops, "tokens": T, "value": ws * flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "launches_per_step": 1}


def bench_decode(steps, warmup, ws, rank):
    from lightserve_b200.engine import BlockManager, Request
    from lightserve_b200.model.minimal_llama import decode_bench_config, init_weights
    from lightserve_b200.model.paged_decode import PagedDecoder, PagedKVCache

    c = DEC_CFG
    cfg = decode_bench_config()
    w = init_weights(cfg, device="cuda", seed=0)
    g = torch.Generator().manual_seed(rank)
    lens = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["S"],), generator=g).tolist()
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    bs = c["block_size"]
    max_blocks = -(-(c["ctx_hi"] + c["steps"] + warmup + 2) // bs)
    num_blocks = sum(-(-(n + c["steps"] + warmup + 2) // bs) for n in lens) + 8
    cache = PagedKVCache(cfg, num_blocks, bs)
    bm = BlockManager(block_size=bs, num_gpu_blocks=num_blocks)
    dec = PagedDecoder(w, cfg, cache, bm, max_batch=c["S"], max_blocks_per_seq=max_blocks)
    reqs = [Request(f"r{i}", p) for i, p in enumerate(prompts)]
    dec.admit(reqs, c["steps"] + warmup + 1)
    # Packed prefill of all prompts (already run once by admit), timed again
    # on the same inputs: it rewrites the same cache slots with the same values.
    tables = [bm.get_block_table(r) for r in reqs]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    dec.prefill_packed(reqs, tables)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    dec.capture()
    torch.cuda.nvtx.range_push("decode_steps")  # lets ncu select the timed replays
    total_ms, _ = time_cuda(dec.graph.replay, steps, warmup, ws)
    torch.cuda.nvtx.range_pop()
    ms = total_ms / steps
    ctx = sum(lens) / len(lens) + warmup + steps / 2
    layers = cfg.n_layers
    kv_bytes = c["S"] * ctx * layers * 2 * cfg.hidden_size * 2
    w_bytes = sum(t.numel() * t.element_size() for t in
                  [w.lm_head] + [getattr(l, n) for l in w.layers for n in
                                 ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")])
    return {"ms_per_step": ms, "value": ws * c["S"] / (ms * 1e-3), "unit": "tokens/s",
            "hbm_bytes_per_step": kv_bytes + w_bytes, "achieved_gbs": (kv_bytes + w_bytes) / (ms * 1e-3) / 1e9,
            "seqs_per_gpu": c["S"], "mean_prompt": sum(lens) / len(lens),
            "prefill": {"ms": prefill_ms, "tokens": sum(lens),
                        "tokens_per_s": sum(lens) / (prefill_ms * 1e-3),
                        "note": "packed prefill of the 64 prompts (varlen attention), CUDA-event timed outside the decode steps"}}


def bench_torch_sdpa(steps, warmup):
    """Context, not the product: PyTorch's own scaled_dot_product_attention
    (whatever backend it dispatches to on this GPU) on config 2 (forward) and
    config 3 (backward through autograd), same FLOP conventions."""
    import torch.nn.functional as F

    gen = torch.Generator(device="cuda").manual_seed(4000)
    c = FWD_CFG
    q, k, v = (_randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen) for _ in range(3))
    with torch.no_grad():
        total, _ = time_cuda(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), steps, warmup, 1)
    fwd = attn_fwd_flops(c["B"], c["H"], c["N"], c["D"], True) / (total / steps * 1e-3) / 1e12
    del q, k, v
    c = BWD_CFG
    q, k, v = (_randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen).requires_grad_()
               for _ in range(3))
    do = _randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    total, _ = time_cuda(lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True),
                         steps, warmup, 1)
    bwd = attn_bwd_flops(c["B"], c["H"], c["N"], c["D"], True) / (total / steps * 1e-3) / 1e12
    return {"fwd_tflops": fwd, "bwd_tflops": bwd,
            "note": "torch.nn.functional.scaled_dot_product_attention, bf16, causal; context only"}


# ------------------------------------------------------------- CPU baseline --
def cpu_attention_sample(target_s: float = 10.0):
    """The reference's CPU path for config 2 (dense fp32 causal attention, the
    oracle in oracle/attention.py) on a bounded sample of (b, h) slices of the
    same shape, all host threads. Returns (TFLOP/s, cores, sample text)."""
    from oracle.attention import attention_ref, attn_fwd_flops

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    c = FWD_CFG
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 1, c["N"], c["D"], generator=g) for _ in range(3))
    slices, t0 = 0, time.perf_counter()
    while True:
        attention_ref(q, k, v, True)
        slices += 1
        el = time.perf_counter() - t0
        if el >= target_s or slices >= c["B"] * c["H"]:
            break
    flops = attn_fwd_flops(1, slices, c["N"], c["D"], True)
    return flops / el / 1e12, cores, (f"{slices} of {c['B'] * c['H']} (b,h) slices of N={c['N']} D={c['D']} "
                                      f"causal, fp32 dense softmax(QK^T)V, {el:.1f} s")


def run_reference(args, rank, ws):
    """--impl reference: the reference's CPU implementation of the path (the
    oracle port: lightserve's GPU code is Triton and its CPU path is PyTorch
    SDPA), timed on this host on config 2's metric. Rank 0 only."""
    if rank != 0:
        return
    from oracle.attention import attention_ref, attn_fwd_flops

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    c = FWD_CFG
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 1, c["N"], c["D"], generator=g) for _ in range(3))
    for _ in range(max(args.warmup, 1)):
        attention_ref(q, k, v, True)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        attention_ref(q, k, v, True)
    el = time.perf_counter() - t0
    flops = attn_fwd_flops(1, args.steps, c["N"], c["D"], True)
    val = flops / el / 1e12
    sample = f"1 (b,h) slice of config 2 per step (N={c['N']} D={c['D']} causal fp32)"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": CONFIG,
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


METRIC = "FA fwd causal bf16 TFLOP/s (B=4,H=32,N=4096,D=128)"
CONFIG = {"workload": "causal FlashAttention forward, BASELINE config 2", "B": 4, "H": 32, "N": 4096,
          "D": 128, "causal": True, "l2": "inputs (4 x 134 MB) larger than L2"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--only", default="fwd,bwd,rmsnorm,varlen,decode,serving,context",
                    help="comma list of workloads (fwd is always run: it is the headline)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--strong", action="store_true",
                    help="split config 2's (b,h) slices across ranks instead of one full config per rank")
    args = ap.parse_args()
    rank, ws, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, rank, ws)
        return
    args.warmup = max(args.warmup, 3)
    peaks = load_peaks()
    traffic = load_traffic()
    only = set(args.only.split(","))
    with ClockSampler(local) as clk:
        fwd = bench_fwd(args.steps, args.warmup, ws, rank, peaks, e2e_steps=min(args.steps, 5),
                        strong=args.strong)
    secondary = {}
    if "bwd" in only:
        secondary["fa_bwd"] = bench_bwd(args.steps, args.warmup, ws, rank)
        secondary["fa_bwd"]["frac_of_peak"] = secondary["fa_bwd"]["value"] / ws / peaks["bf16_tflops"]
    if "rmsnorm" in only:
        secondary["rmsnorm"] = bench_rmsnorm(args.steps, args.warmup, ws, rank)
        secondary["rmsnorm"]["frac_of_peak"] = secondary["rmsnorm"]["value"] / ws / peaks["hbm_gbs"]
    if "varlen" in only:
        secondary["varlen_prefill_attn"] = bench_varlen(args.steps, args.warmup, ws, rank)
        secondary["varlen_prefill_attn"]["frac_of_peak"] = (secondary["varlen_prefill_attn"]["value"] / ws
                                                             / peaks["bf16_tflops"])
    if "decode" in only:
        secondary["paged_decode"] = bench_decode(min(args.steps * 4, 128), args.warmup, ws, rank)
    if "serving" in only:
        secondary["serving"] = bench_serving(ws, rank)
    if ws == 1 and "context" in only:
        try:
            secondary["torch_sdpa_context"] = bench_torch_sdpa(args.steps, args.warmup)
        except Exception as e:  # context only: never fail the bench on it
            secondary["torch_sdpa_context"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    if rank != 0:
        return
    cpu = None
    if not args.no_cpu_baseline:
        v, cores, sample = cpu_attention_sample()
        cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}
    achieved = fwd["kernel_tflops"]
    tr = traffic.get("attn_fwd", {}).get("dram_bytes_per_launch")
    line = {
        "metric": METRIC, "value": fwd["value"], "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": fwd["ms"], "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))", "config": CONFIG,
        "e2e": {k: v for k, v in fwd["e2e"].items() if k != "steps"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"], "traffic": tr,
                     "peak_source": peaks["source"] + " (burst bf16)"},
        "cpu_baseline": cpu,
        "gpu_launches": fwd["launches_per_step"] * args.steps,
        "clocks": clk.summary(),
        "secondary": secondary,
    }
    print(json.dumps(line))


def _shutdown():
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    try:
        main()
    finally:
        _shutdown()
