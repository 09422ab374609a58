"""Variable-length (packed) attention and the packed prefill that uses it.

Each packed sequence must get exactly the attention it would get alone:
checked against the oracle per sequence (bf16/fp16 tolerance 2e-2, as the
dense forward), bit-for-bit against the dense kernel where the dense
kernel computes the same thing (one sequence, or sequences of one length),
and with q/k/v as strided views into one fused QKV buffer (the prefill's
layout). Ragged lengths cover 1, tile edges (127/128/129, 255/256/257) and
empty sequences."""
import pytest
import torch

from oracle.attention import attention_ref
from lightserve_b200.engine import BlockManager, Request
from lightserve_b200.kernels import (flash_attention_forward, flash_attention_varlen,
                                     rope_kv_write_slots)
from lightserve_b200.model.minimal_llama import LlamaConfig, apply_rope, init_weights, precompute_rope
from lightserve_b200.model.paged_decode import PagedDecoder, PagedKVCache, slots_for_positions

pytestmark = pytest.mark.gpu


def _pack(lens, H, D, dtype, seed, fused=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = sum(lens)
    if fused:
        qkv = torch.randn(T, 3, H, D, device="cuda", dtype=dtype, generator=g)
        q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
    else:
        q, k, v = (torch.randn(T, H, D, device="cuda", dtype=dtype, generator=g) for _ in range(3))
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    return q, k, v, cu


LENS = [[1], [300], [5, 128, 129, 1, 300], [127, 255, 256, 257, 0, 64], [1000, 3, 513]]


@pytest.mark.parametrize("lens", LENS)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_varlen_matches_oracle_per_sequence(lens, D, causal, dtype):
    H = 3
    q, k, v, cu = _pack(lens, H, D, dtype, seed=sum(lens) + D, fused=(D == 128))
    lse = torch.empty(H, q.shape[0], device="cuda", dtype=torch.float32)
    o = flash_attention_varlen(q, k, v, cu, max(lens), causal=causal, lse=lse)
    for s, n in enumerate(lens):
        if n == 0:
            continue
        a, b = int(cu[s]), int(cu[s + 1])
        sl = lambda t: t[a:b].transpose(0, 1).unsqueeze(0)  # noqa: E731  [1, H, n, D]
        ref = attention_ref(sl(q), sl(k), sl(v), causal)
        torch.testing.assert_close(sl(o).float().cpu(), ref, atol=2e-2, rtol=2e-2)
        # LSE of the packed rows = logsumexp of the sequence's own scaled scores.
        qf, kf = sl(q).float().cpu()[0], sl(k).float().cpu()[0]
        sc = qf @ kf.transpose(-1, -2) / D ** 0.5
        if causal:
            sc = sc.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
        torch.testing.assert_close(lse[:, a:b].cpu(), torch.logsumexp(sc, -1), atol=2e-2, rtol=1e-3)


@pytest.mark.parametrize("n", [1, 200, 1024])
def test_single_sequence_is_bit_identical_to_dense(n):
    H, D = 4, 128
    q, k, v, cu = _pack([n], H, D, torch.bfloat16, seed=n)
    o = flash_attention_varlen(q, k, v, cu, n, causal=True)
    dense = flash_attention_forward(*(t.transpose(0, 1).unsqueeze(0) for t in (q, k, v)), causal=True)
    assert torch.equal(o, dense[0].transpose(0, 1))


def test_equal_lengths_bit_identical_to_dense_batch():
    B, H, N, D = 3, 2, 384, 64
    q, k, v, cu = _pack([N] * B, H, D, torch.bfloat16, seed=7)
    o = flash_attention_varlen(q, k, v, cu, N, causal=True)
    to4 = lambda t: t.view(B, N, H, D).transpose(1, 2)  # noqa: E731
    dense = flash_attention_forward(to4(q), to4(k), to4(v), causal=True)
    assert torch.equal(to4(o), dense)


def test_max_seqlen_zero_and_empty_batch_are_noops():
    q, k, v, cu = _pack([0, 0], 2, 64, torch.bfloat16, seed=1)
    assert flash_attention_varlen(q, k, v, cu, 0).shape == (0, 2, 64)


def test_rope_kv_write_slots_matches_apply_rope():
    """Rotated q/k equal lightserve's apply_rope (bit-exact: same roundings),
    and every token's k/v lands in its cache slot."""
    cfg = LlamaConfig(vocab_size=16, hidden_size=256, intermediate_size=64, n_layers=1, n_heads=2,
                      head_dim=128, max_seq_len=600, rope_theta=10000.0, dtype=torch.bfloat16)
    H, D, bs, nb = cfg.n_heads, cfg.head_dim, 16, 80
    cos, sin = precompute_rope(cfg, "cuda")
    lens = [37, 1, 520]
    T = sum(lens)
    qkv = torch.randn(T, 3, H, D, device="cuda", dtype=cfg.dtype)
    pos = torch.cat([torch.arange(n) for n in lens]).cuda()
    perm = torch.randperm(nb)
    tables, start = [], 0
    for n in lens:
        nblk = -(-n // bs)
        tables.append(perm[start:start + nblk].tolist())
        start += nblk
    slots = torch.cat([slots_for_positions(t, range(n), bs) for t, n in zip(tables, lens)]).cuda()
    slots[5] = -1  # skipped write
    kc = torch.zeros(nb, H, bs, D, device="cuda", dtype=cfg.dtype)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(T, H, D, device="cuda", dtype=cfg.dtype)
    k_out = torch.empty_like(q_out)
    rope_kv_write_slots(qkv, cos, sin, pos, slots, q_out, k_out, kc, vc)
    c, s_ = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
    eq, ek = apply_rope(qkv[:, 0], qkv[:, 1], c, s_)
    assert torch.equal(q_out, eq) and torch.equal(k_out, ek)
    flat_k = kc.transpose(1, 2).reshape(nb * bs, H, D)
    flat_v = vc.transpose(1, 2).reshape(nb * bs, H, D)
    keep = slots >= 0
    assert torch.equal(flat_k[slots[keep]], ek[keep]) and torch.equal(flat_v[slots[keep]], qkv[keep, 2])


def test_packed_prefill_matches_per_request_prefill():
    """The packed prefill fills the cache like one llama_forward per request
    (within bf16 GEMM-order noise) and returns the same first tokens wherever
    the per-request logits are not a near tie."""
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=688, n_layers=2, n_heads=2,
                      head_dim=128, max_seq_len=700, rope_theta=10000.0, dtype=torch.bfloat16)
    w = init_weights(cfg, device="cuda", seed=0)
    gen = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 512, (n,), generator=gen).tolist() for n in (1, 130, 600, 17)]
    caches, firsts = [], []
    for packed in (True, False):
        cache = PagedKVCache(cfg, num_blocks=128, block_size=16)
        bm = BlockManager(block_size=16, num_gpu_blocks=128)
        dec = PagedDecoder(w, cfg, cache, bm, max_batch=4, max_blocks_per_seq=48)
        firsts.append(dec.admit([Request(f"r{i}", p) for i, p in enumerate(prompts)], 4, packed=packed))
        caches.append(cache)
    for a, b in zip(caches[0].k + caches[0].v, caches[1].k + caches[1].v):
        assert (a.float() - b.float()).norm() <= 2e-2 * b.float().norm()
    assert torch.equal(firsts[0], firsts[1])


# Work numbering in variable-length mode: up to 128 groups of 16 (sequence,
# head) slices and 512 sequences, only the 256-row blocks inside each
# sequence are numbered (a table built in shared memory); above either
# limit every slice gets max_seqlen / 256 blocks and those past its end are
# skipped. Every item is computed the same way in both, so each sequence's
# rows must equal the dense kernel's output for that sequence alone, bit for
# bit.
@pytest.mark.parametrize("lens,H,max_seqlen", [
    ([4096, 1, 300, 0, 513, 256, 257, 2000, 17], 16, None),   # compact, many skipped blocks
    ([513, 40, 1, 256], 4, 800),                              # max_seqlen above the longest
    ([(37 * i) % 300 + 1 for i in range(130)], 16, None),     # 130 groups: uncompacted
    ([(53 * i) % 200 + 1 for i in range(600)], 2, None),      # 600 sequences: uncompacted
])
@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16)])
def test_varlen_numbering_bit_identical_to_dense(lens, H, max_seqlen, D, dtype):
    q, k, v, cu = _pack(lens, H, D, dtype, seed=len(lens) + H)
    o = flash_attention_varlen(q, k, v, cu, max_seqlen or max(lens), causal=True)
    for s, n in enumerate(lens):
        if n == 0:
            continue
        a, b = int(cu[s]), int(cu[s + 1])
        sl = lambda t: t[a:b].transpose(0, 1).unsqueeze(0)  # noqa: E731  [1, H, n, D]
        dense = flash_attention_forward(sl(q).contiguous(), sl(k).contiguous(), sl(v).contiguous(),
                                        causal=True)
        assert torch.equal(sl(o), dense), f"sequence {s} (length {n})"
