"""silu_and_mul on the GPU vs lightserve's own expression
F.silu(gate) * up (model/minimal_llama.py:231-233), evaluated by PyTorch on the
same device: same roundings (silu in fp32 rounded to the dtype, then the
dtype product), so the results must be bit-identical."""
import pytest
import torch
import torch.nn.functional as F

from lightserve_b200.kernels import silu_and_mul

pytestmark = pytest.mark.gpu

SHAPES = [(1, 8), (64, 5632), (3, 13), (7, 4100), (0, 16)]


@pytest.mark.parametrize("S,I", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_matches_reference_expression(S, I, dtype):
    torch.manual_seed(0)
    gu = (3 * torch.randn(S, 2 * I, device="cuda")).to(dtype)
    got = silu_and_mul(gu)
    want = F.silu(gu[:, :I]) * gu[:, I:]
    assert got.shape == want.shape
    torch.testing.assert_close(got, want, atol=0, rtol=0)


def test_strided_rows_and_out():
    torch.manual_seed(1)
    S, I = 5, 256
    big = torch.randn(S, 2 * I + 40, device="cuda", dtype=torch.bfloat16)
    gu = big[:, : 2 * I]  # row stride 2I + 40
    out_big = torch.zeros(S, I + 24, device="cuda", dtype=torch.bfloat16)
    out = out_big[:, :I]
    silu_and_mul(gu, out=out)
    torch.testing.assert_close(out, F.silu(gu[:, :I]) * gu[:, I:], atol=0, rtol=0)
    assert torch.all(out_big[:, I:] == 0)  # nothing written past the row
