"""Pins the CPU oracle against golden vectors produced by lightserve's own code
(tests/golden/make_golden.py: its Triton kernels under the Triton CPU
interpreter, and reference_llama_forward's greedy decode)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import attention as oa
from oracle import llama as ol
from oracle import rmsnorm as orms

ATTN_FILES = sorted(GOLDEN.glob("attn_*.npz"))
RMS_FILES = sorted(GOLDEN.glob("rmsnorm_*.npz"))


def test_golden_files_present():
    assert len(ATTN_FILES) >= 5 and len(RMS_FILES) >= 4
    assert (GOLDEN / "llama_toy.npz").exists()


@pytest.mark.parametrize("path", ATTN_FILES, ids=lambda p: p.stem)
def test_tiled_forward_matches_reference_kernels(path):
    g = np.load(path)
    o, lse = oa.flash_fwd_tiled(g["q"], g["k"], g["v"], bool(g["causal"]))
    np.testing.assert_allclose(o, g["o"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(lse, g["lse"], atol=2e-6, rtol=1e-5)
    # The LSE forward and the forward-only kernel agree (reference test :107-124).
    np.testing.assert_allclose(g["o_fwd_only"], g["o"], atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("path", ATTN_FILES, ids=lambda p: p.stem)
def test_tiled_backward_matches_reference_kernels(path):
    g = np.load(path)
    dq, dk, dv = oa.flash_bwd_tiled(g["q"], g["k"], g["v"], g["o"], g["do"], g["lse"], bool(g["causal"]))
    for a, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(a, g[name], atol=1e-5, rtol=1e-4, err_msg=name)


@pytest.mark.parametrize("path", ATTN_FILES, ids=lambda p: p.stem)
def test_dense_reference_matches_reference_kernels(path):
    g = np.load(path)
    q, k, v, do = (torch.from_numpy(g[n]) for n in ("q", "k", "v", "do"))
    o, lse = oa.attention_ref(q, k, v, bool(g["causal"]), return_lse=True)
    np.testing.assert_allclose(o.numpy(), g["o"], atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(lse.numpy(), g["lse"], atol=1e-5, rtol=1e-4)
    dq, dk, dv = oa.attention_ref_grads(q, k, v, do, bool(g["causal"]))
    for a, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(a.numpy(), g[name], atol=1e-4, rtol=1e-4, err_msg=name)


@pytest.mark.parametrize("path", RMS_FILES, ids=lambda p: p.stem)
def test_rmsnorm_oracle_matches_reference_kernel(path):
    g = np.load(path)
    out, h = orms.rmsnorm_residual(torch.from_numpy(g["x"]), torch.from_numpy(g["r"]),
                                   torch.from_numpy(g["w"]), float(g["eps"]))
    np.testing.assert_array_equal(h.numpy(), g["h"])
    np.testing.assert_allclose(out.numpy(), g["out"], atol=1e-6, rtol=1e-5)


def _toy():
    from lightserve_b200.model.minimal_llama import LlamaConfig, init_weights

    cfg = LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=688, n_layers=2, n_heads=4,
                      head_dim=64, max_seq_len=64, rope_theta=10000.0, dtype=torch.float32)
    return cfg, init_weights(cfg, device="cpu", seed=0)


def test_llama_oracle_matches_reference_logits_and_tokens():
    g = np.load(GOLDEN / "llama_toy.npz")
    cfg, w = _toy()
    prompts = [list(row[:n]) for row, n in zip(g["prompts"], g["prompt_lens"])]
    with torch.no_grad():
        logits = ol.reference_forward(w, cfg, torch.tensor([prompts[1]]))
    np.testing.assert_allclose(logits.numpy(), g["logits_prompt1"], atol=1e-5, rtol=1e-4)
    with torch.no_grad():
        for p, toks in zip(prompts, g["tokens"]):
            assert ol.greedy_full_recompute(w, cfg, p, len(toks)) == list(toks)


def test_paged_oracle_equals_last_row_of_causal_attention():
    torch.manual_seed(0)
    S, H, D, bs, L = 2, 3, 16, 4, 11
    k = torch.randn(S, H, L, D); v = torch.randn(S, H, L, D); q = torch.randn(S, H, L, D)
    nb = 16
    kc = torch.zeros(nb, H, bs, D); vc = torch.zeros(nb, H, bs, D)
    perm = torch.randperm(nb)
    bt = torch.full((S, 4), -1, dtype=torch.int32)
    for s in range(S):
        for t in range(L):
            blk = int(perm[s * 4 + t // bs]); bt[s, t // bs] = blk
            kc[blk, :, t % bs] = k[s, :, t]; vc[blk, :, t % bs] = v[s, :, t]
    out = ol.paged_decode_ref(q[:, :, -1], kc, vc, bt, torch.full((S,), L, dtype=torch.int32))
    full = oa.attention_ref(q, k, v, causal=True)[:, :, -1]
    torch.testing.assert_close(out, full, atol=1e-5, rtol=1e-5)
