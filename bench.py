"""Benchmark of lightserve_b200's attention hot path on B200.

Headline: causal FlashAttention forward, bf16,
B=4 H=32 N=4096 D=128, seeded N(0,1) inputs, TFLOP/s with lightserve's FLOP
convention 4*B*H*N^2*D/2 (kernels/benchmark_flash_attention.py:55-64).
Secondary lines in the same JSON object: FA backward (config 3), fused
add+RMSNorm (config 4) and paged greedy decode tokens/s (config 5).

Multi-GPU: one process per GPU (torchrun). By default each configuration's
fixed total work is partitioned across the ranks ("scaling": "strong"):
config 2's and config 3's 128 (batch x head) slices, config 4's rows, config
5's 64 sequences (each rank holds a full weight replica, its own paged KV
pool and its own CUDA graph). The units are independent, so there is no
collective on the data path; times are the max over ranks and every value is
the whole configuration's work divided by that time. `--scaling weak` gives
every rank a full configuration instead.

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


def _sum_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64, device="cuda")
    dist.all_reduce(t)
    return float(t.item())


DEVICE_ERRORS: dict = {}


def check_device_errors(what: str) -> None:
    """Reads (and clears) the library's device error words after a workload:
    a kernel that gave up on a bounded on-chip wait fails the bench loudly
    instead of reporting a speed for partial output."""
    from lightserve_b200 import _lib

    code = int(_lib.load().lsb_device_error_reset())
    DEVICE_ERRORS[what] = code
    if code:
        raise RuntimeError(f"{what}: a kernel gave up on a bounded wait (device error {code:#x})")


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


def time_cuda(fn, steps: int, warmup: int, ws: int, per_call: bool = True):
    """Warm-up, then EXACTLY `steps` calls bracketed by barrier + synchronize;
    returns (max-over-ranks total ms, per-call event ms list). With
    per_call=False only the two bracketing events are recorded (no event
    records between the calls); the list is then empty."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps if per_call else 0)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s)
    if per_call:
        for a, b in evs:
            a.record(s)
            fn()
            b.record(s)
    else:
        for _ in range(steps):
            fn()
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


def bench_fwd(steps, warmup, ws, rank, peaks, e2e_steps, strong=True):
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
    job_flops = attn_fwd_flops(c["B"], c["H"], c["N"], c["D"], True) * (1 if strong else ws)
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
    check_device_errors("attention forward")
    return {
        "ms": ms, "kernel_ms": kern_ms, "flops": flops, "slices_per_rank": shape[0] * shape[1],
        "value": job_flops / (ms * 1e-3) / 1e12,
        "kernel_tflops": flops / (kern_ms * 1e-3) / 1e12,
        "e2e": {"value": job_flops / (e2e_total / e2e_steps * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": 3 * nb, "d2h_bytes_per_step": nb, "steps": e2e_steps},
        "launches_per_step": 1,
    }


def bench_bwd(steps, warmup, ws, rank, strong=True):
    from lightserve_b200.kernels.flash_attention_backward import (_flash_attention_backward,
                                                                  _flash_attention_forward_lse)
    from lightserve_b200.sharding import shard_range

    c = BWD_CFG
    gen = torch.Generator(device="cuda").manual_seed(2000 + rank)
    if strong:
        a, b = shard_range(c["B"] * c["H"], rank, ws)
        shape = (1, b - a, c["N"], c["D"])
    else:
        shape = (c["B"], c["H"], c["N"], c["D"])
    q, k, v, do = (_randn(shape, torch.bfloat16, gen) for _ in range(4))
    o, L = _flash_attention_forward_lse(q, k, v, True)
    job_flops = attn_bwd_flops(c["B"], c["H"], c["N"], c["D"], True) * (1 if strong else ws)
    total_ms, _ = time_cuda(lambda: _flash_attention_backward(do, q, k, v, o, L, True), steps, warmup, ws,
                            per_call=False)
    ms = total_ms / steps
    check_device_errors("attention backward")
    return {"ms": ms, "flops": job_flops, "value": job_flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "launches_per_step": 3, "slices_per_rank": shape[0] * shape[1]}


def bench_rmsnorm(steps, warmup, ws, rank, strong=True):
    from lightserve_b200.kernels import fused_add_rmsnorm
    from lightserve_b200.sharding import shard_range

    c = RMS_CFG
    gen = torch.Generator(device="cuda").manual_seed(3000 + rank)
    a, b = shard_range(c["M"], rank, ws) if strong else (0, c["M"])
    x = _randn((b - a, c["N"]), torch.bfloat16, gen)
    r = _randn((b - a, c["N"]), torch.bfloat16, gen)
    w = (1 + 0.02 * torch.randn(c["N"], device="cuda", generator=gen)).to(torch.bfloat16)
    job_bytes = rmsnorm_bytes(c["M"], c["N"], 2) * (1 if strong else ws)
    total_ms, _ = time_cuda(lambda: fused_add_rmsnorm(x, r, w, 1e-6), steps, warmup, ws, per_call=False)
    ms = total_ms / steps
    check_device_errors("rmsnorm")
    return {"ms": ms, "bytes": job_bytes, "value": job_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "launches_per_step": 1, "rows_per_rank": b - a}


def _prompt_set(cfg, rank, ws, strong):
    """Config 5's prompt set: 64 lengths U[512, 4096] and token ids U[0, 32000)
    from seed 0. Strong scaling: this rank's contiguous share of the 64
    sequences; weak: a full set of its own (seed = rank)."""
    from lightserve_b200.sharding import shard_range

    c = DEC_CFG
    g = torch.Generator().manual_seed(0 if strong else rank)
    lens = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["S"],), generator=g).tolist()
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    a, b = shard_range(c["S"], rank, ws) if strong else (0, c["S"])
    return prompts[a:b]


def bench_serving(ws, rank, strong=True, max_tokens=64):
    """Continuous batching end to end (ServingEngine: scheduler, packed
    prefill, CUDA-graph paged decode, host-side token handling each step) on
    config 5's model and prompt set (this rank's share of it): all requests
    submitted at once, each generating max_tokens tokens. Timed on the host
    around run(), after one warm-up run of the same requests."""
    from lightserve_b200.engine import CacheConfig, Request, SamplingParams, SchedulerConfig
    from lightserve_b200.model.minimal_llama import decode_bench_config, init_weights
    from lightserve_b200.model.serving import ServingEngine

    c = DEC_CFG
    cfg = decode_bench_config()
    w = init_weights(cfg, device="cuda", seed=0)
    prompts = _prompt_set(cfg, rank, ws, strong)
    lens = [len(p) for p in prompts]
    bs = c["block_size"]
    blocks = sum(-(-(n + max_tokens) // bs) for n in lens) + 8
    eng = ServingEngine(w, cfg, CacheConfig(block_size=bs, num_gpu_blocks=blocks),
                        SchedulerConfig(max_num_seqs=len(prompts), max_num_batched_tokens=sum(lens)))
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
        assert len(out) == len(prompts) and all(len(v) == max_tokens for v in out.values())
    el = max_over_ranks(times[-1], ws)
    mult = 1 if strong else ws
    n_req = c["S"] * mult
    gen = n_req * max_tokens
    total_prompt = _sum_over_ranks(sum(lens), ws)
    return {"seconds": el, "requests": n_req, "prompt_tokens": total_prompt, "generated_tokens": gen,
            "value": gen / el, "unit": "generated tokens/s",
            "total_tokens_per_s": (gen + total_prompt) / el,
            "note": "host-timed ServingEngine.run(): prefill of every prompt, then decode steps"}


def bench_varlen(steps, warmup, ws, rank, strong=True):
    """Packed (variable-length) causal attention over config 5's prompt set
    (this rank's share): lengths U[512, 4096], 16 heads x 128, bf16 -- one
    layer's prefill attention."""
    from lightserve_b200.kernels import flash_attention_varlen
    from lightserve_b200.model.minimal_llama import decode_bench_config

    lens = [len(p) for p in _prompt_set(decode_bench_config(), rank, ws, strong)]
    T, H, D = sum(lens), 16, 128
    gen = torch.Generator(device="cuda").manual_seed(2000 + rank)
    q, k, v = (_randn((T, H, D), torch.bfloat16, gen) for _ in range(3))
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    total_ms, _ = time_cuda(lambda: flash_attention_varlen(q, k, v, cu, max(lens), causal=True, out=out),
                            steps, warmup, ws, per_call=False)
    ms = total_ms / steps
    flops = _sum_over_ranks(sum(attn_fwd_flops(1, H, n, D, True) for n in lens), ws)
    check_device_errors("varlen attention")
    return {"ms": ms, "flops": flops, "tokens": _sum_over_ranks(T, ws),
            "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "launches_per_step": 1}


def bench_decode(steps, warmup, ws, rank, strong=True):
    from lightserve_b200.engine import BlockManager, Request
    from lightserve_b200.model.minimal_llama import decode_bench_config, init_weights
    from lightserve_b200.model.paged_decode import PagedDecoder, PagedKVCache

    c = DEC_CFG
    cfg = decode_bench_config()
    w = init_weights(cfg, device="cuda", seed=0)
    prompts = _prompt_set(cfg, rank, ws, strong)
    lens = [len(p) for p in prompts]
    S = len(prompts)
    bs = c["block_size"]
    max_blocks = -(-(c["ctx_hi"] + c["steps"] + warmup + 2) // bs)
    num_blocks = sum(-(-(n + c["steps"] + warmup + 2) // bs) for n in lens) + 8
    cache = PagedKVCache(cfg, num_blocks, bs)
    bm = BlockManager(block_size=bs, num_gpu_blocks=num_blocks)
    dec = PagedDecoder(w, cfg, cache, bm, max_batch=S, max_blocks_per_seq=max_blocks)
    reqs = [Request(f"r{i}", p) for i, p in enumerate(prompts)]
    dec.admit(reqs, c["steps"] + warmup + 1)
    # Packed prefill of all prompts (already run once by admit), timed again
    # on the same inputs: it rewrites the same cache slots with the same values.
    tables = [bm.get_block_table(r) for r in reqs]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(ws)
    e0.record()
    dec.prefill_packed(reqs, tables)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(e0.elapsed_time(e1), ws)
    dec.capture()
    torch.cuda.nvtx.range_push("decode_steps")  # lets ncu select the timed replays
    total_ms, _ = time_cuda(dec.graph.replay, steps, warmup, ws)
    torch.cuda.nvtx.range_pop()
    ms = total_ms / steps
    check_device_errors("paged decode")
    mult = 1 if strong else ws
    n_seq = c["S"] * mult
    # HBM bytes per step over the whole job: every rank streams the weights
    # once and its own sequences' K/V.
    ctx_sum = _sum_over_ranks(sum(lens) + S * (warmup + steps / 2), ws)
    layers = cfg.n_layers
    kv_bytes = ctx_sum * layers * 2 * cfg.hidden_size * 2
    w_bytes = sum(t.numel() * t.element_size() for t in
                  [w.lm_head] + [getattr(l, n) for l in w.layers for n in
                                 ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")])
    job_bytes = kv_bytes + ws * w_bytes
    total_prompt = _sum_over_ranks(sum(lens), ws)
    return {"ms_per_step": ms, "value": n_seq / (ms * 1e-3), "unit": "tokens/s",
            "hbm_bytes_per_step": job_bytes, "achieved_gbs": job_bytes / (ms * 1e-3) / 1e9,
            "achieved_gbs_per_gpu": job_bytes / ws / (ms * 1e-3) / 1e9,
            "seqs_per_gpu": S, "mean_prompt": total_prompt / n_seq,
            "prefill": {"ms": prefill_ms, "tokens": total_prompt,
                        "tokens_per_s": total_prompt / (prefill_ms * 1e-3),
                        "note": "packed prefill of every prompt (varlen attention), CUDA-event timed "
                                "outside the decode steps, max over ranks"}}


def bench_torch_sdpa(steps, warmup):
    """Context, not the product: PyTorch's own scaled_dot_product_attention
    (whatever backend it dispatches to on this GPU) on config 2 (forward) and
    config 3 (backward through autograd), same FLOP conventions."""
    import torch.nn.functional as F

    gen = torch.Generator(device="cuda").manual_seed(4000)
    c = FWD_CFG
    q, k, v = (_randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen) for _ in range(3))
    with torch.no_grad():
        total, _ = time_cuda(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), steps, warmup, 1, False)
    fwd = attn_fwd_flops(c["B"], c["H"], c["N"], c["D"], True) / (total / steps * 1e-3) / 1e12
    del q, k, v
    c = BWD_CFG
    q, k, v = (_randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen).requires_grad_()
               for _ in range(3))
    do = _randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    total, _ = time_cuda(lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True),
                         steps, warmup, 1, False)
    bwd = attn_bwd_flops(c["B"], c["H"], c["N"], c["D"], True) / (total / steps * 1e-3) / 1e12
    return {"fwd_tflops": fwd, "bwd_tflops": bwd,
            "note": "torch.nn.functional.scaled_dot_product_attention, bf16, causal; context only"}


# ------------------------------------------------------------- CPU baseline --
def _cpu_threads():
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    return cores


def _sdpa_cpu(q, k, v):
    """lightserve's CPU comparison path for attention: PyTorch SDPA, causal,
    implicit 1/sqrt(D) scale (kernels/tests/test_flash_attention.py:47)."""
    import torch.nn.functional as F

    return F.scaled_dot_product_attention(q, k, v, is_causal=True)


def cpu_attention_sample(target_s: float = 8.0):
    """Config 2 on the host cores through the reference's CPU path (fp32 SDPA)
    over as many (b, h) slices of the config's shape as fit in ~target_s.
    Returns (TFLOP/s, cores, sample text)."""
    cores = _cpu_threads()
    c = FWD_CFG
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 4, c["N"], c["D"], generator=g) for _ in range(3))
    with torch.no_grad():
        _sdpa_cpu(q, k, v)  # warm-up
        slices, t0 = 0, time.perf_counter()
        while True:
            _sdpa_cpu(q, k, v)
            slices += 4
            el = time.perf_counter() - t0
            if el >= target_s or slices >= c["B"] * c["H"]:
                break
    flops = attn_fwd_flops(1, slices, c["N"], c["D"], True)
    return flops / el / 1e12, cores, (f"{slices} of {c['B'] * c['H']} (b,h) slices of N={c['N']} "
                                      f"D={c['D']} causal, fp32 torch SDPA on the host, {el:.1f} s")


def cpu_backward_sample(target_s: float = 5.0):
    """Config 3 on the host: SDPA autograd fp32 (the reference's gradient
    oracle, kernels/tests/test_flash_attention_backward.py:69-90), backward
    only timed, over (b, h) slices of the config's shape."""
    cores = _cpu_threads()
    c = BWD_CFG
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 4, c["N"], c["D"], generator=g).requires_grad_() for _ in range(3))
    do = torch.randn(1, 4, c["N"], c["D"], generator=g)
    slices, el = 0, 0.0
    while el < target_s and slices < c["B"] * c["H"]:
        o = _sdpa_cpu(q, k, v)
        t0 = time.perf_counter()
        torch.autograd.grad(o, (q, k, v), do)
        el += time.perf_counter() - t0
        slices += 4
    flops = attn_bwd_flops(1, slices, c["N"], c["D"], True)
    return {"value": flops / el / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
            "sample": f"{slices} of {c['B'] * c['H']} (b,h) slices, fp32 SDPA autograd backward on the "
                      f"host, {el:.1f} s"}


def cpu_rmsnorm_sample(target_s: float = 3.0):
    """Config 4 on the host: lightserve's eager add+RMSNorm
    (rmsnorm_residual_reference, kernels/tests/test_fused_rmsnorm_residual.py:24-29)
    in fp32 over row blocks of the config; GB/s counts the config's bf16
    bytes for the rows processed (same work as the GPU line)."""
    from oracle.rmsnorm import rmsnorm_residual

    cores = _cpu_threads()
    c = RMS_CFG
    g = torch.Generator().manual_seed(0)
    rows = 1024
    x, r = (torch.randn(rows, c["N"], generator=g) for _ in range(2))
    w = 1 + 0.02 * torch.randn(c["N"], generator=g)
    done, t0 = 0, time.perf_counter()
    while True:
        rmsnorm_residual(x, r, w, 1e-6)
        done += rows
        el = time.perf_counter() - t0
        if el >= target_s or done >= c["M"]:
            break
    return {"value": rmsnorm_bytes(done, c["N"], 2) / el / 1e9, "unit": "GB/s", "cores": cores,
            "kind": "port", "sample": f"{done} of {c['M']} rows, fp32 eager add+RMSNorm, {el:.1f} s"}


def cpu_decode_sample(steps: int = 2):
    """Config 5 on the host: lightserve's decode is a full recompute of
    reference_llama_forward per step (model/cuda_graph_decode.py:108-118);
    this times `steps` greedy steps of ONE sequence at the prompt set's mean
    length in fp32 and extrapolates tokens/s for the batch of 64 as 64
    sequences at that per-sequence rate run one after another (the forward is
    compute-bound on the host, so batching does not change the total)."""
    from lightserve_b200.model.minimal_llama import decode_bench_config, init_weights
    from oracle.llama import reference_forward

    cores = _cpu_threads()
    cfg = decode_bench_config(dtype=torch.float32)
    w = init_weights(cfg, device="cpu", seed=0)
    g = torch.Generator().manual_seed(0)
    n = 2400
    ids = torch.randint(0, cfg.vocab_size, (1, n), generator=g)
    t0 = time.perf_counter()
    with torch.no_grad():
        for _ in range(steps):
            nxt = reference_forward(w, cfg, ids)[0, -1].argmax().view(1, 1)
            ids = torch.cat([ids, nxt], dim=1)
    el = time.perf_counter() - t0
    return {"value": steps / el, "unit": "tokens/s", "cores": cores, "kind": "port",
            "extrapolated": True,
            "sample": f"{steps} full-recompute greedy steps of 1 sequence at {n} tokens, fp32, "
                      f"{el:.1f} s; the batch of {DEC_CFG['S']} is extrapolated at this per-sequence rate"}


def bench_reference_triton(steps, warmup):
    """Context, not the product: lightserve's own Triton kernels (staged
    unmodified under baseline/_ref by tests/stage_reference_kernels.py) on
    configs 2, 3 and 4 on this GPU, same FLOP/byte conventions."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "kernels" / "flash_attention.py").exists():
        return {"unavailable": "reference kernels not staged (tests/stage_reference_kernels.py)"}
    sys.path.insert(0, str(ref))
    try:
        from kernels import flash_attention as rfa
        from kernels import flash_attention_backward as rfb
        from kernels import fused_rmsnorm_residual as rrn
    finally:
        sys.path.remove(str(ref))
    out = {}
    gen = torch.Generator(device="cuda").manual_seed(4000)
    c = FWD_CFG
    q, k, v = (_randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen) for _ in range(3))
    total, _ = time_cuda(lambda: rfa.flash_attention_forward(q, k, v, causal=True), steps, warmup, 1, False)
    out["fwd_tflops"] = attn_fwd_flops(c["B"], c["H"], c["N"], c["D"], True) / (total / steps * 1e-3) / 1e12
    del q, k, v
    c = BWD_CFG
    q, k, v, do = (_randn((c["B"], c["H"], c["N"], c["D"]), torch.bfloat16, gen) for _ in range(4))
    o, L = rfb._flash_attention_forward_lse(q, k, v, True)
    total, _ = time_cuda(lambda: rfb._flash_attention_backward(do, q, k, v, o, L, True), steps, warmup, 1, False)
    out["bwd_tflops"] = attn_bwd_flops(c["B"], c["H"], c["N"], c["D"], True) / (total / steps * 1e-3) / 1e12
    del q, k, v, do, o, L
    c = RMS_CFG
    x, r = (_randn((c["M"], c["N"]), torch.bfloat16, gen) for _ in range(2))
    w = (1 + 0.02 * torch.randn(c["N"], device="cuda", generator=gen)).to(torch.bfloat16)
    total, _ = time_cuda(lambda: rrn.fused_add_rmsnorm(x, r, w, 1e-6), steps, warmup, 1, False)
    out["rmsnorm_gbs"] = rmsnorm_bytes(c["M"], c["N"], 2) / (total / steps * 1e-3) / 1e9
    out["note"] = "lightserve's Triton kernels (JIT for sm_100 by Triton) on this GPU; context only"
    return out


def run_reference(args, rank, ws):
    """--impl reference: the reference's CPU implementation of the path,
    PyTorch SDPA in fp32 (lightserve's own comparison target,
    kernels/tests/test_flash_attention.py:47; its GPU code is Triton), on
    this host's cores, on config 2's metric. Each step is a bounded sample
    of 8 (b, h) slices of config 2. Rank 0 only."""
    if rank != 0:
        return
    cores = _cpu_threads()
    c = FWD_CFG
    g = torch.Generator().manual_seed(0)
    per_step = 8
    q, k, v = (torch.randn(1, per_step, c["N"], c["D"], generator=g) for _ in range(3))
    with torch.no_grad():
        for _ in range(max(args.warmup, 1)):
            _sdpa_cpu(q, k, v)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _sdpa_cpu(q, k, v)
        el = time.perf_counter() - t0
    flops = attn_fwd_flops(1, per_step * args.steps, c["N"], c["D"], True)
    val = flops / el / 1e12
    sample = (f"{per_step} (b,h) slices of config 2 per step (N={c['N']} D={c['D']} causal), "
              f"fp32 torch SDPA on {cores} host threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": CONFIG,
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                         "sample": sample},
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
    ap.add_argument("--only", default="fwd,bwd,rmsnorm,varlen,decode,serving,context,triton",
                    help="comma list of workloads (fwd is always run: it is the headline)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: each configuration's fixed work is split across the ranks; "
                         "weak: every rank runs a full configuration")
    args = ap.parse_args()
    rank, ws, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, rank, ws)
        return
    args.warmup = max(args.warmup, 3)
    strong = args.scaling == "strong"
    peaks = load_peaks()
    traffic = load_traffic()
    only = set(args.only.split(","))
    with ClockSampler(local) as clk:
        fwd = bench_fwd(args.steps, args.warmup, ws, rank, peaks, e2e_steps=min(args.steps, 5),
                        strong=strong)
    secondary = {}
    if "bwd" in only:
        secondary["fa_bwd"] = bench_bwd(args.steps, args.warmup, ws, rank, strong)
        secondary["fa_bwd"]["frac_of_peak"] = secondary["fa_bwd"]["value"] / ws / peaks["bf16_tflops"]
    if "rmsnorm" in only:
        secondary["rmsnorm"] = bench_rmsnorm(args.steps, args.warmup, ws, rank, strong)
        secondary["rmsnorm"]["frac_of_peak"] = secondary["rmsnorm"]["value"] / ws / peaks["hbm_gbs"]
    if "varlen" in only:
        secondary["varlen_prefill_attn"] = bench_varlen(args.steps, args.warmup, ws, rank, strong)
        secondary["varlen_prefill_attn"]["frac_of_peak"] = (secondary["varlen_prefill_attn"]["value"] / ws
                                                             / peaks["bf16_tflops"])
    if "decode" in only:
        secondary["paged_decode"] = bench_decode(min(args.steps * 4, 128), args.warmup, ws, rank, strong)
        secondary["paged_decode"]["frac_of_peak"] = (secondary["paged_decode"]["achieved_gbs_per_gpu"]
                                                     / peaks["hbm_gbs"])
    if "serving" in only:
        secondary["serving"] = bench_serving(ws, rank, strong)
    if ws == 1 and "context" in only:
        try:
            secondary["torch_sdpa_context"] = bench_torch_sdpa(args.steps, args.warmup)
        except Exception as e:  # context only: never fail the bench on it
            secondary["torch_sdpa_context"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    if ws == 1 and "triton" in only:
        try:
            secondary["reference_triton_context"] = bench_reference_triton(args.steps, args.warmup)
        except Exception as e:  # context only: never fail the bench on it
            secondary["reference_triton_context"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    if rank != 0:
        return
    cpu = None
    if not args.no_cpu_baseline:
        v, cores, sample = cpu_attention_sample()
        cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "reference", "sample": sample}
        if ws == 1:
            if "bwd" in secondary:
                secondary["fa_bwd"]["cpu_baseline"] = cpu_backward_sample()
            if "rmsnorm" in secondary:
                secondary["rmsnorm"]["cpu_baseline"] = cpu_rmsnorm_sample()
            if "paged_decode" in secondary:
                secondary["paged_decode"]["cpu_baseline"] = cpu_decode_sample()
    achieved = fwd["kernel_tflops"]
    tr = traffic.get("attn_fwd", {}).get("dram_bytes_per_launch")
    config = dict(CONFIG)
    config["parallelism"] = (f"(b,h) slices split over {ws} GPU(s), {fwd['slices_per_rank']} per rank"
                             if strong else f"{ws} replica(s) of the full config")
    line = {
        "metric": METRIC, "value": fwd["value"], "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": fwd["ms"], "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))", "config": config,
        "e2e": {k: v for k, v in fwd["e2e"].items() if k != "steps"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"], "traffic": tr,
                     "peak_source": peaks["source"] + " (burst bf16)"},
        "cpu_baseline": cpu,
        "gpu_launches": fwd["launches_per_step"] * args.steps,
        "clocks": clk.summary(),
        "device_errors": DEVICE_ERRORS,
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
