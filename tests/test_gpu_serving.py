"""Continuous-batching serving (scheduler -> packed prefill / paged decode)
against lightserve's full-recompute greedy decode: the fp32 golden token ids
(reference_llama_forward, tests/golden/llama_toy.npz) must come out exactly,
also when requests queue behind max_num_seqs and when the KV pool is so small
that requests are preempted and recomputed; bf16 against the oracle's
teacher-forced argmax."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.llama import reference_forward
from lightserve_b200.engine import CacheConfig, Request, SamplingParams, SchedulerConfig
from lightserve_b200.model.minimal_llama import LlamaConfig, init_weights
from lightserve_b200.model.serving import ServingEngine

pytestmark = pytest.mark.gpu


def _toy(dtype, head_dim=64, max_seq_len=64):
    return LlamaConfig(vocab_size=256, hidden_size=4 * head_dim, intermediate_size=688, n_layers=2,
                       n_heads=4, head_dim=head_dim, max_seq_len=max_seq_len, rope_theta=10000.0,
                       dtype=dtype)


def _golden():
    g = np.load(GOLDEN / "llama_toy.npz")
    prompts = [list(map(int, row[:n])) for row, n in zip(g["prompts"], g["prompt_lens"])]
    return prompts, [list(map(int, t)) for t in g["tokens"]]


# (block_size, blocks, max_num_seqs, graph): ample pool; requests queueing
# behind max_num_seqs; a pool of 11 four-token blocks, where the longest
# request alone fits but not beside the others (one recompute preemption).
@pytest.mark.parametrize("bs,blocks,seqs,use_graph", [(16, 64, 3, True), (16, 64, 2, True),
                                                      (4, 11, 3, True), (4, 11, 3, False)])
def test_fp32_serving_matches_reference_tokens(bs, blocks, seqs, use_graph):
    prompts, tokens = _golden()
    cfg = _toy(torch.float32)
    eng = ServingEngine(init_weights(cfg, device="cuda", seed=0), cfg,
                        CacheConfig(block_size=bs, num_gpu_blocks=blocks),
                        SchedulerConfig(max_num_seqs=seqs, max_num_batched_tokens=512), use_graph=use_graph)
    out = eng.generate(prompts, max_tokens=len(tokens[0]))
    assert out == tokens
    bm = eng.scheduler.block_manager
    assert bm.num_free_blocks == blocks and not bm.block_tables and not eng.slot_of
    if blocks == 11:
        assert eng.num_preemptions > 0


def test_bf16_serving_teacher_forced_argmax_matches_oracle():
    cfg = _toy(torch.bfloat16, head_dim=64, max_seq_len=128)
    w = init_weights(cfg, device="cuda", seed=0)
    eng = ServingEngine(w, cfg, CacheConfig(block_size=16, num_gpu_blocks=12),
                        SchedulerConfig(max_num_seqs=3, max_num_batched_tokens=256))
    gen = torch.Generator().manual_seed(11)
    lens = (9, 40, 70, 3, 25)
    prompts = [torch.randint(0, 256, (n,), generator=gen).tolist() for n in lens]
    reqs = [Request(f"q{i}", p, SamplingParams(max_tokens=12)) for i, p in enumerate(prompts)]
    for r in reqs:
        eng.add_request(r)
    res = eng.run()
    assert sorted(res) == sorted(r.request_id for r in reqs)
    w_cpu = init_weights(cfg, device="cpu", seed=0)
    checked = 0
    for r in reqs:
        toks = res[r.request_id]
        assert len(toks) == 12
        ids = list(r.prompt_token_ids)
        for t in toks:
            with torch.no_grad():
                logits = reference_forward(w_cpu, cfg, torch.tensor([ids]))[0, -1].float()
            top2 = torch.topk(logits, 2)
            if float(top2.values[0] - top2.values[1]) > 0.05:
                assert t == int(top2.indices[0])
                checked += 1
            ids.append(t)
    assert checked >= 20
    assert eng.scheduler.block_manager.num_free_blocks == 12


def test_eos_stops_a_request_early():
    prompts, tokens = _golden()
    cfg = _toy(torch.float32)
    eng = ServingEngine(init_weights(cfg, device="cuda", seed=0), cfg,
                        CacheConfig(block_size=16, num_gpu_blocks=64),
                        SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=512))
    eos = tokens[1][4]  # request 1 emits this token fifth
    out = eng.generate(prompts, max_tokens=len(tokens[0]), eos_token_id=eos)
    for o, t in zip(out, tokens):
        n = t.index(eos) + 1 if eos in t else len(t)
        assert o == t[:n]
