"""Continuous-batching greedy serving: lightserve's scheduler policy
(``engine/scheduler.py``, here ``lightserve_b200.engine.Scheduler``) driving
this package's kernels, the model-runner wiring lightserve leaves open
(``engine/README.md:134-141``: "What's not wired up").

Each ``step()``:

1. ``Scheduler.schedule()`` decides the batch (and preempts by recompute when
   the KV pool runs out);
2. requests admitted this step (``scheduled_new``, a whole sequence each:
   the prompt, or prompt + tokens generated before a preemption) get one
   packed prefill (``PagedDecoder.prefill``: varlen attention, RoPE + cache
   write by slot) that also yields their next token;
3. running requests (``scheduled_running``, one token each) get one decode
   step over the paged cache in batch rows ("slots") they keep while running
   (``PagedDecoder.decode_slots``: a CUDA graph replay);
4. sampled tokens are appended, ``Request.maybe_finish`` applies the length
   cap / EOS, and ``free_finished_requests`` returns finished requests' blocks.
"""
from __future__ import annotations

import torch

from .._lib import check_device_errors
from ..engine import CacheConfig, Request, Scheduler, SchedulerConfig
from .minimal_llama import LlamaConfig, LlamaWeights
from .paged_decode import PagedDecoder, PagedKVCache


class ServingEngine:
    def __init__(self, weights: LlamaWeights, config: LlamaConfig, cache_config: CacheConfig,
                 scheduler_config: SchedulerConfig, device="cuda", use_graph: bool = True,
                 check_every: int = 64):
        self.cfg = config
        # Every `check_every` steps (and at the end of run()) the device error
        # words are read: a kernel that gave up on a bounded wait raises
        # lightserve_b200.DeviceWaitError instead of yielding tokens silently.
        self.check_every = check_every
        self._steps = 0
        self.scheduler = Scheduler(cache_config, scheduler_config)
        bs = cache_config.block_size
        self.cache = PagedKVCache(config, cache_config.num_gpu_blocks, bs, device=device)
        max_blocks = -(-config.max_seq_len // bs)
        self.runner = PagedDecoder(weights, config, self.cache, self.scheduler.block_manager,
                                   max_batch=scheduler_config.max_num_seqs,
                                   max_blocks_per_seq=max_blocks, device=device)
        self.use_graph = use_graph
        self.slot_of: dict = {}
        self._free_slots = list(range(scheduler_config.max_num_seqs - 1, -1, -1))
        self.num_prefill_tokens = 0
        self.num_decode_tokens = 0
        self.num_preemptions = 0
        self._next_id = 0

    def add_request(self, request: Request) -> None:
        need = len(request.prompt_token_ids) + request.sampling_params.max_tokens
        assert 0 < len(request.prompt_token_ids) and need <= self.cfg.max_seq_len, (
            f"{request.request_id}: prompt + max_tokens = {need} exceeds max_seq_len "
            f"{self.cfg.max_seq_len}")
        self.scheduler.add_request(request)

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished_requests()

    def _release(self, req: Request) -> None:
        slot = self.slot_of.pop(req.request_id, None)
        if slot is not None:
            self._free_slots.append(slot)

    def _emit(self, req: Request, token: int) -> None:
        req.output_token_ids.append(int(token))
        req.maybe_finish()

    def step(self) -> list:
        """One scheduling step; returns the requests that finished in it."""
        out = self.scheduler.schedule()
        self.num_preemptions += len(out.preempted)
        for r in out.preempted:
            self._release(r)
        bm = self.scheduler.block_manager
        new = [x.request for x in out.scheduled_new]
        if new:
            for r in new:
                self.slot_of[r.request_id] = self._free_slots.pop()
            seqs = [r.all_token_ids() for r in new]
            self.num_prefill_tokens += sum(len(t) for t in seqs)
            toks = self.runner.prefill(seqs, [bm.get_block_table(r) for r in new])
            for r, t in zip(new, toks):
                self._emit(r, t)
        run = [x.request for x in out.scheduled_running]
        if run:
            toks = self.runner.decode_slots(
                [self.slot_of[r.request_id] for r in run],
                [r.output_token_ids[-1] if r.output_token_ids else r.prompt_token_ids[-1] for r in run],
                [r.get_len() - 1 for r in run], [bm.get_block_table(r) for r in run],
                use_graph=self.use_graph)
            self.num_decode_tokens += len(run)
            for r, t in zip(run, toks):
                self._emit(r, t)
        done = self.scheduler.free_finished_requests()
        for r in done:
            self._release(r)
        self._steps += 1
        if self.check_every and self._steps % self.check_every == 0:
            check_device_errors()
        return done

    def run(self, max_steps: int = 1_000_000) -> dict:
        """Steps until every request has finished; returns {request_id: output tokens}."""
        results = {}
        for _ in range(max_steps):
            if not self.has_unfinished_requests():
                break
            for r in self.step():
                results[r.request_id] = list(r.output_token_ids)
        assert not self.has_unfinished_requests(), "max_steps reached with requests unfinished"
        check_device_errors()
        return results

    def generate(self, prompts, max_tokens: int, eos_token_id=None) -> list:
        """Adds one request per prompt and runs them all; outputs in prompt order."""
        from ..engine import SamplingParams

        ids = []
        for p in prompts:
            rid = f"gen-{self._next_id}"
            self._next_id += 1
            self.add_request(Request(rid, list(p), SamplingParams(max_tokens=max_tokens,
                                                                  eos_token_id=eos_token_id)))
            ids.append(rid)
        res = self.run()
        return [res[r] for r in ids]
