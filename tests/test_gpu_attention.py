"""FlashAttention forward/backward on the GPU vs the oracle, with the shapes,
dtypes and tolerances of lightserve's kernels/tests/test_flash_attention.py and
kernels/tests/test_flash_attention_backward.py, plus golden fixtures from
lightserve's own Triton kernels and the tcgen05-path shapes."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.attention import attention_ref, attention_ref_grads
from lightserve_b200 import _lib
from lightserve_b200.kernels import flash_attention, flash_attention_forward
from lightserve_b200.kernels.flash_attention import _attn_fwd
from lightserve_b200.kernels.flash_attention_backward import (_flash_attention_backward,
                                                              _flash_attention_forward_lse)

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1, 8), (1, 1, 17, 32), (2, 2, 64, 64), (1, 4, 130, 64), (2, 8, 256, 128),
          (1, 2, 100, 96)]
# Shapes that reach the tcgen05 kernel (bf16/fp16, D in {64,128}), ragged N included.
TC_SHAPES = [(1, 2, 128, 128), (1, 1, 1, 128), (2, 3, 200, 64), (1, 2, 513, 128), (1, 4, 1024, 128),
             (2, 2, 384, 64)]


def _tol(dtype, bwd=False):
    if dtype == torch.float32:
        return 1e-3
    return 3e-2 if bwd else 2e-2


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,N,D", SHAPES)
def test_forward_matches_oracle(B, H, N, D, dtype, causal):
    torch.manual_seed(0)
    q, k, v = (torch.randn(B, H, N, D, device="cuda", dtype=dtype) for _ in range(3))
    out = flash_attention_forward(q, k, v, causal=causal)
    exp = attention_ref(q, k, v, causal)
    t = _tol(dtype)
    torch.testing.assert_close(out.float().cpu(), exp, atol=t, rtol=t)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,N,D", TC_SHAPES)
def test_tensor_core_forward_matches_oracle(B, H, N, D, dtype, causal):
    torch.manual_seed(1)
    q, k, v = (torch.randn(B, H, N, D, device="cuda", dtype=dtype) for _ in range(3))
    o, L = _flash_attention_forward_lse(q, k, v, causal)
    exp, lse = attention_ref(q, k, v, causal, return_lse=True)
    torch.testing.assert_close(o.float().cpu(), exp, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(L.cpu(), lse, atol=2e-2, rtol=1e-3)
    # The SIMT kernel of the same library agrees.
    o2 = torch.empty_like(q)
    _attn_fwd(q, k, v, o2, None, causal, impl=_lib.IMPL_SIMT)
    torch.testing.assert_close(o.float(), o2.float(), atol=2e-2, rtol=2e-2)


def test_forward_non_contiguous():
    torch.manual_seed(0)
    q = torch.randn(1, 64, 4, 32, device="cuda").transpose(1, 2)
    k = torch.randn(1, 4, 64, 32, device="cuda")
    v = torch.randn(1, 4, 64, 32, device="cuda")
    torch.testing.assert_close(flash_attention_forward(q, k, v).cpu(), attention_ref(q, k, v, False),
                               atol=1e-3, rtol=1e-3)


def test_forward_non_contiguous_bf16_tensor_core():
    torch.manual_seed(0)
    q = torch.randn(2, 256, 4, 128, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    k = torch.randn(2, 256, 4, 128, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    v = torch.randn(2, 4, 256, 128, device="cuda", dtype=torch.bfloat16)
    out = flash_attention_forward(q, k, v, causal=True)
    torch.testing.assert_close(out.float().cpu(), attention_ref(q, k, v, True), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("attn_*.npz")), ids=lambda p: p.stem)
def test_matches_reference_kernel_golden(path):
    g = np.load(path)
    q, k, v, do = (torch.from_numpy(g[n]).cuda().requires_grad_(n != "do") for n in ("q", "k", "v", "do"))
    causal = bool(g["causal"])
    o = flash_attention(q, k, v, causal=causal)
    o.backward(do)
    np.testing.assert_allclose(o.detach().cpu().numpy(), g["o"], atol=1e-4, rtol=1e-3)
    for t, n in ((q, "dq"), (k, "dk"), (v, "dv")):
        np.testing.assert_allclose(t.grad.cpu().numpy(), g[n], atol=1e-3, rtol=1e-3, err_msg=n)
    _, L = _flash_attention_forward_lse(q.detach(), k.detach(), v.detach(), causal)
    np.testing.assert_allclose(L.cpu().numpy(), g["lse"], atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,H,N,D", [(1, 1, 4, 8), (1, 2, 9, 16)])
def test_gradcheck(B, H, N, D, causal):
    torch.manual_seed(0)
    q, k, v = (torch.randn(B, H, N, D, device="cuda", requires_grad=True) for _ in range(3))
    assert torch.autograd.gradcheck(lambda a, b, c: flash_attention(a, b, c, causal=causal), (q, k, v),
                                    eps=1e-3, atol=1e-2, rtol=1e-2)


BWD_SHAPES = [(1, 1, 17, 32), (2, 2, 64, 64), (1, 4, 130, 64), (2, 8, 256, 128), (1, 2, 300, 128),
              (1, 2, 1000, 128), (2, 4, 700, 64), (1, 20, 2048, 64)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,N,D", BWD_SHAPES)
def test_backward_matches_oracle(B, H, N, D, dtype, causal):
    torch.manual_seed(0)
    q, k, v = (torch.randn(B, H, N, D, device="cuda", dtype=dtype, requires_grad=True) for _ in range(3))
    do = torch.randn(B, H, N, D, device="cuda", dtype=dtype)
    out = flash_attention(q, k, v, causal=causal)
    out.backward(do)
    eq, ek, ev = attention_ref_grads(q, k, v, do, causal)
    t = _tol(dtype, bwd=True)
    for a, e, n in ((q.grad, eq, "dq"), (k.grad, ek, "dk"), (v.grad, ev, "dv")):
        torch.testing.assert_close(a.float().cpu(), e, atol=t, rtol=t, msg=n)


@pytest.mark.parametrize("D", [64, 128])
def test_backward_simt_and_default_agree_bf16(D):
    """The tcgen05 backward (D = 64 and 128) against the SIMT kernel of the same library."""
    torch.manual_seed(3)
    B, H, N = 1, 2, 256
    q, k, v, do = (torch.randn(B, H, N, D, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    o, L = _flash_attention_forward_lse(q, k, v, True)
    a = _flash_attention_backward(do, q, k, v, o, L, True, impl=_lib.IMPL_TCGEN05)
    b = _flash_attention_backward(do, q, k, v, o, L, True, impl=_lib.IMPL_SIMT)
    for x, y in zip(a, b):
        torch.testing.assert_close(x.float(), y.float(), atol=3e-2, rtol=3e-2)


def test_forward_matches_forward_only_kernel():
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 4, 130, 64, device="cuda") for _ in range(3))
    torch.testing.assert_close(flash_attention(q, k, v, causal=True),
                               flash_attention_forward(q, k, v, causal=True), atol=1e-3, rtol=1e-3)


def test_full_size_forward_properties():
    """BASELINE config 2 (4x32x4096x128 bf16, causal): finite, sampled rows
    against the oracle, and causality (perturbing the last key leaves every
    earlier row bit-identical)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    B, H, N, D = 4, 32, 4096, 128
    q, k, v = (torch.randn(B, H, N, D, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(3))
    o = flash_attention_forward(q, k, v, causal=True)
    assert torch.isfinite(o).all()
    for b, h in ((0, 0), (3, 31), (2, 17)):
        exp = attention_ref(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1], True)
        torch.testing.assert_close(o[b:b + 1, h:h + 1].float().cpu(), exp, atol=2e-2, rtol=2e-2)
    k2 = k.clone(); k2[:, :, -1] += 1.0
    o2 = flash_attention_forward(q, k2, v, causal=True)
    assert torch.equal(o[:, :, :-1], o2[:, :, :-1])


@pytest.mark.parametrize("chunk", [1, 3, 16])
def test_forward_host_streaming_matches_device(chunk):
    """flash_attention_forward_host streams (b, h) chunks of pinned host
    tensors through the same kernel: bit-identical to the device call."""
    from lightserve_b200.kernels import flash_attention_forward_host

    torch.manual_seed(5)
    B, H, N, D = 2, 5, 300, 128
    q, k, v = (torch.randn(B, H, N, D, dtype=torch.bfloat16).pin_memory() for _ in range(3))
    got = flash_attention_forward_host(q, k, v, causal=True, chunk_slices=chunk)
    torch.cuda.synchronize()
    want = flash_attention_forward(q.cuda(), k.cuda(), v.cuda(), causal=True).cpu()
    assert got.device.type == "cpu"
    torch.testing.assert_close(got, want, atol=0, rtol=0)
