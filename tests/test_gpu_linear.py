"""Weight-streaming decode linear (lsb_linear) against an fp32 matmul of the
same bf16 operands: the decode projection shapes of config 5 (q/k/v fused,
o, gate/up fused, down, lm_head), ragged S / N / K, partial-tile stream-K
cluster splits, fp16, strided rows, determinism, and CUDA-graph replay."""
import pytest
import torch

from lightserve_b200.kernels import linear, pack_linear_weight

pytestmark = pytest.mark.gpu

DECODE_SHAPES = [(6144, 2048), (2048, 2048), (11264, 2048), (2048, 5632), (32000, 2048)]


def _check(y, x, w_t):
    ref = x.float() @ w_t.float().t()
    # One rounding to bf16/fp16 of an fp32 sum: relative 2^-8 (bf16), plus
    # the summation-order difference of the fp32 accumulation.
    tol = 8e-3 if x.dtype == torch.bfloat16 else 2e-3
    torch.testing.assert_close(y.float(), ref, atol=tol * ref.abs().max().item() + 1e-3, rtol=tol)


@pytest.mark.parametrize("S", [1, 8, 64, 100, 128])
@pytest.mark.parametrize("N,K", DECODE_SHAPES)
def test_decode_shapes(S, N, K):
    g = torch.Generator(device="cuda").manual_seed(S * 7 + N)
    x = torch.randn(S, K, device="cuda", generator=g).to(torch.bfloat16)
    w_t = (0.02 * torch.randn(N, K, device="cuda", generator=g)).to(torch.bfloat16)
    _check(linear(x, w_t), x, w_t)


@pytest.mark.parametrize("S,N,K", [(3, 1, 8), (5, 130, 72), (33, 200, 136), (64, 129, 4104),
                                   (17, 300, 64), (2, 4096, 8)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ragged(S, N, K, dtype):
    g = torch.Generator(device="cuda").manual_seed(N + K)
    x = torch.randn(S, K, device="cuda", generator=g).to(dtype)
    w_t = (0.05 * torch.randn(N, K, device="cuda", generator=g)).to(dtype)
    _check(linear(x, w_t), x, w_t)


def test_strided_rows_deterministic():
    g = torch.Generator(device="cuda").manual_seed(1)
    S, N, K = 64, 2048, 5632
    xb = torch.randn(S, K + 64, device="cuda", generator=g).to(torch.bfloat16)
    x = xb[:, :K]                      # row stride K + 64
    w_t = (0.02 * torch.randn(N, K, device="cuda", generator=g)).to(torch.bfloat16)
    outb = torch.zeros(S, N + 8, device="cuda", dtype=torch.bfloat16)
    out = outb[:, :N]
    pw = pack_linear_weight(w_t)
    ys = []
    for _ in range(3):
        linear(x, pw, out=out)
        ys.append(out.clone())
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])
    assert torch.equal(outb[:, N:], torch.zeros_like(outb[:, N:]))  # nothing past N written
    _check(ys[0], x, w_t)


def test_matches_cublas_closely():
    """Against torch's bf16 matmul (also fp32 accumulation, one rounding):
    at most a couple of bf16 ulps apart."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(64, 2048, device="cuda", generator=g).to(torch.bfloat16)
    w_t = (0.02 * torch.randn(11264, 2048, device="cuda", generator=g)).to(torch.bfloat16)
    y = linear(x, w_t).float()
    c = (x @ w_t.t()).float()
    assert ((y - c).abs() <= 2 ** -6 * c.abs() + 1e-4).float().mean() > 0.999


def test_graph_replay():
    g = torch.Generator(device="cuda").manual_seed(4)
    S, N, K = 64, 6144, 2048
    x = torch.randn(S, K, device="cuda", generator=g).to(torch.bfloat16)
    w_t = (0.02 * torch.randn(N, K, device="cuda", generator=g)).to(torch.bfloat16)
    out = torch.empty(S, N, device="cuda", dtype=torch.bfloat16)
    pw = pack_linear_weight(w_t)
    linear(x, pw, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        linear(x, pw, out=out)
    want = out.clone()
    for _ in range(3):
        out.zero_()
        x.copy_(x)  # same inputs
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    x.mul_(-1)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, -want)


def test_pack_layout():
    """Packed tile (t, k), row r, 16-byte chunk position p holds W^T row
    128 t + r, columns 64 k + 8 (p ^ (r % 8)) .. + 8; zeros past N and K."""
    g = torch.Generator(device="cuda").manual_seed(5)
    N, K = 130, 72
    w_t = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    pw = pack_linear_weight(w_t)
    tiles = pw.data.view(torch.bfloat16).view(2, 2, 128, 8, 8).cpu()  # [t][k][r][p][8]
    ref = torch.zeros(256, 128, dtype=torch.bfloat16)
    ref[:N, :K] = w_t.cpu()
    for t in range(2):
        for k in range(2):
            for r in (0, 1, 7, 8, 77, 127):
                for p_ in range(8):
                    c = p_ ^ (r % 8)
                    want = ref[128 * t + r, 64 * k + 8 * c: 64 * k + 8 * c + 8]
                    assert torch.equal(tiles[t, k, r, p_], want), (t, k, r, p_)
