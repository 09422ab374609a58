"""Greedy next-token kernel (lsb_greedy_next) against torch.argmax: ties
(first index wins), NaN (counts as the maximum), -inf rows, unaligned and
strided rows, every dtype, and the position increment."""
import pytest
import torch

from lightserve_b200.kernels import greedy_next

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("S,V", [(1, 1), (3, 7), (64, 32000), (5, 32003), (128, 4096)])
def test_matches_torch_argmax(dtype, S, V):
    g = torch.Generator(device="cuda").manual_seed(S + V)
    logits = torch.randn(S, V, device="cuda", generator=g).to(dtype)
    if V > 10:
        logits[0, 3] = logits[0, V - 2] = logits[0].max() + 1  # tie: first index
    if S > 2:
        logits[1, :] = float("-inf")
        logits[2, V // 2] = float("nan")
    pos = torch.arange(S, device="cuda", dtype=torch.int64) * 3
    tok = torch.full((S,), -5, dtype=torch.int64, device="cuda")
    greedy_next(logits, tok, pos)
    assert torch.equal(tok, logits.argmax(-1))
    assert torch.equal(pos, torch.arange(S, device="cuda", dtype=torch.int64) * 3 + 1)


def test_strided_and_unaligned_rows():
    g = torch.Generator(device="cuda").manual_seed(7)
    base = torch.randn(9, 1003, device="cuda", generator=g).to(torch.bfloat16)
    logits = base[:, 1:1001]  # row stride 1003, start not 16-byte aligned
    assert torch.equal(greedy_next(logits), logits.argmax(-1))
