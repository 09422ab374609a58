"""Paged decode attention and KV write on the GPU vs the oracle: ragged and
empty contexts, multi-partition contexts, shuffled block tables, bad block
ids, and equality with the last row of causal attention."""
import pytest
import torch

from oracle.attention import attention_ref
from oracle.llama import paged_decode_ref
from lightserve_b200.kernels import paged_decode_attention, write_kv_cache

pytestmark = pytest.mark.gpu


def _build(S, H, D, bs, lens, dtype, nb_extra=7, seed=0):
    g = torch.Generator().manual_seed(seed)
    max_blocks = max(1, max(-(-l // bs) for l in lens))
    nb = S * max_blocks + nb_extra
    perm = torch.randperm(nb, generator=g)
    bt = torch.full((S, max_blocks), -1, dtype=torch.int32)
    for s, l in enumerate(lens):
        nblk = -(-l // bs)
        bt[s, :nblk] = perm[s * max_blocks: s * max_blocks + nblk].to(torch.int32)
    kc = torch.randn(nb, H, bs, D, generator=g).to(dtype)
    vc = torch.randn(nb, H, bs, D, generator=g).to(dtype)
    q = torch.randn(S, H, D, generator=g).to(dtype)
    return q, kc, vc, bt, torch.tensor(lens, dtype=torch.int32)


CASES = [  # S, H, D, bs, lens
    (4, 2, 128, 16, [1, 15, 16, 17]),
    (3, 4, 64, 16, [0, 33, 100]),
    (5, 2, 128, 16, [511, 512, 513, 1500, 4224]),
    (2, 3, 128, 8, [1000, 7]),
    (2, 2, 256, 16, [700, 31]),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("S,H,D,bs,lens", CASES)
def test_matches_oracle(S, H, D, bs, lens, dtype):
    if dtype == torch.float32 and D == 256:
        pytest.skip("fp32 paged decode supports D <= 128")
    q, kc, vc, bt, cl = _build(S, H, D, bs, lens, dtype)
    out = paged_decode_attention(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda())
    exp = paged_decode_ref(q, kc, vc, bt, cl)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(out.float().cpu(), exp, atol=tol, rtol=tol)


def test_bad_block_ids_read_nothing():
    q, kc, vc, bt, cl = _build(2, 2, 128, 16, [40, 40], torch.bfloat16)
    bt2 = bt.clone()
    bt2[1, 1] = 10_000  # out of range: its 16 tokens are skipped
    out = paged_decode_attention(q.cuda(), kc.cuda(), vc.cuda(), bt2.cuda(), cl.cuda())
    # tokens 32..39 live in block bt[1,2]; build the expected result from positions 0-15 and 32-39
    keep = [(int(bt[1, 0]), list(range(16))), (int(bt[1, 2]), list(range(8)))]
    K = torch.cat([kc[b][:, offs] for b, offs in keep], dim=1).float()  # [H, 24, D]
    V = torch.cat([vc[b][:, offs] for b, offs in keep], dim=1).float()
    s = torch.einsum("hd,hld->hl", q[1].float(), K) / 128 ** 0.5
    exp = torch.einsum("hl,hld->hd", s.softmax(-1), V)
    torch.testing.assert_close(out[1].float().cpu(), exp, atol=2e-2, rtol=2e-2)


def test_equals_last_row_of_causal_attention():
    torch.manual_seed(0)
    H, L, D, bs = 4, 777, 128, 16
    q, k, v = (torch.randn(1, H, L, D, dtype=torch.bfloat16) for _ in range(3))
    nblk = -(-L // bs)
    kc = torch.zeros(nblk + 3, H, bs, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    table = torch.randperm(nblk + 3)[:nblk]
    pos = torch.arange(L)
    slots = (table[pos // bs] * bs + pos % bs).cuda()
    write_kv_cache(k[0].transpose(0, 1).cuda(), v[0].transpose(0, 1).cuda(), kc, vc, slots)
    out = paged_decode_attention(q[0, :, -1].contiguous().cuda().unsqueeze(0), kc, vc,
                                 table.to(torch.int32).view(1, -1).cuda(),
                                 torch.tensor([L], dtype=torch.int32, device="cuda"))
    exp = attention_ref(q, k, v, causal=True)[0, :, -1]
    torch.testing.assert_close(out[0].float().cpu(), exp, atol=2e-2, rtol=2e-2)


def test_kv_write_exact_and_skips_negative_slots():
    torch.manual_seed(0)
    T, H, D, bs, nb = 37, 3, 64, 16, 8
    k = torch.randn(T, H, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, H, D, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(nb, H, bs, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nb * bs, device="cuda")[:T].to(torch.int64)
    slots[5] = -1
    write_kv_cache(k, v, kc, vc, slots)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        assert torch.equal(kc[s // bs, :, s % bs], k[t]) and torch.equal(vc[s // bs, :, s % bs], v[t])
    assert int((kc != 0).any(-1).sum()) == (T - 1) * H


@pytest.mark.parametrize("S,H,D", [(5, 4, 64), (64, 16, 128)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_rope_kv_write_matches_eager_ops(dtype, S, H, D):
    """lsb_rope_kv_write == lightserve-style apply_rope (torch ops) + cache write,
    bit for bit (16-bit inputs take the vectorised kernel, fp32 the scalar one);
    a row whose block table is empty (an idle decode row) writes no cache slot."""
    from lightserve_b200.kernels.paged_attention import rope_kv_write
    from lightserve_b200.model.minimal_llama import LlamaConfig, apply_rope, precompute_rope

    torch.manual_seed(0)
    bs, mb = 16, 6
    cfg = LlamaConfig(vocab_size=8, hidden_size=H * D, intermediate_size=8, n_layers=1, n_heads=H,
                      head_dim=D, max_seq_len=96, rope_theta=10000.0, dtype=dtype)
    cos, sin = precompute_rope(cfg, "cuda")
    qkv = torch.randn(S, 3, H, D, device="cuda").to(dtype)
    pos = torch.randint(0, 96, (S,), device="cuda")
    pos[:5] = torch.tensor([0, 5, 17, 63, 95], device="cuda")
    nb = S * mb
    bt = torch.randperm(nb, device="cuda").view(S, mb).to(torch.int32)
    bt[2] = -1  # idle row
    kc = torch.zeros(nb, H, bs, D, device="cuda", dtype=dtype); vc = torch.zeros_like(kc)
    q_out = torch.empty(S, H, D, device="cuda", dtype=dtype)
    cl = torch.zeros(S, dtype=torch.int32, device="cuda")
    rope_kv_write(qkv, cos, sin, pos, bt, q_out, kc, vc, cl)

    q_ref, k_ref = apply_rope(qkv[:, 0], qkv[:, 1], cos[pos].unsqueeze(1), sin[pos].unsqueeze(1))
    kc2 = torch.zeros_like(kc); vc2 = torch.zeros_like(vc)
    slots = bt.gather(1, (pos // bs).unsqueeze(1)).squeeze(1).long() * bs + pos % bs
    slots[2] = -1
    write_kv_cache(k_ref.contiguous(), qkv[:, 2], kc2, vc2, slots)
    assert torch.equal(q_out, q_ref)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(cl, (pos + 1).to(torch.int32))
