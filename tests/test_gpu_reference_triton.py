"""Same-box comparison with lightserve's own Triton kernels on the B200.

The reference modules are staged unmodified under baseline/_ref/kernels by
tests/stage_reference_kernels.py (the package never imports them). Both
implementations run on identical seeded bf16 inputs and each is held to the
reference's own tolerance against the fp32 oracle; the two are also compared
directly. Shapes: the reference's test shapes
(kernels/tests/test_flash_attention.py:24, test_flash_attention_backward.py:71,
test_fused_rmsnorm_residual.py:20) and BASELINE configs 2-4 (sampled slices
for the oracle, whole tensors for the direct comparison).
"""
import sys
from pathlib import Path

import pytest
import torch

from oracle.attention import attention_ref, attention_ref_grads
from oracle.rmsnorm import rmsnorm_residual
from lightserve_b200.kernels import flash_attention, flash_attention_forward, fused_add_rmsnorm

REF_DIR = Path(__file__).resolve().parent.parent / "baseline" / "_ref"

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not (REF_DIR / "kernels" / "flash_attention.py").exists(),
                       reason="reference kernels not staged (tests/stage_reference_kernels.py)"),
]


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, str(REF_DIR))
    try:
        from kernels import flash_attention as rfa
        from kernels import flash_attention_backward as rfb
        from kernels import fused_rmsnorm_residual as rrn
    finally:
        sys.path.remove(str(REF_DIR))
    return rfa, rfb, rrn


def _qkv(shape, seed, n=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(*shape, device="cuda", generator=g).to(torch.bfloat16) for _ in range(n)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,H,N,D", [(1, 1, 17, 32), (2, 2, 64, 64), (1, 4, 130, 64), (2, 8, 256, 128),
                                     (1, 2, 1000, 128)])
def test_forward_vs_reference_triton(ref, B, H, N, D, causal):
    rfa, _, _ = ref
    q, k, v = _qkv((B, H, N, D), 0)
    ours = flash_attention_forward(q, k, v, causal=causal)
    theirs = rfa.flash_attention_forward(q, k, v, causal=causal)
    exp = attention_ref(q, k, v, causal)
    torch.testing.assert_close(ours.float().cpu(), exp, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(theirs.float().cpu(), exp, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(ours, theirs, atol=2e-2, rtol=2e-2)


def test_config2_forward_vs_reference_triton(ref):
    rfa, _, _ = ref
    q, k, v = _qkv((4, 32, 4096, 128), 1)
    ours = flash_attention_forward(q, k, v, causal=True)
    theirs = rfa.flash_attention_forward(q, k, v, causal=True)
    d = (ours.float() - theirs.float()).abs()
    assert d.max().item() <= 2e-2, f"max-abs {d.max().item():.3g}"
    for b, h in ((0, 0), (3, 31)):
        exp = attention_ref(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1], True)
        torch.testing.assert_close(theirs[b:b + 1, h:h + 1].float().cpu(), exp, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,H,N,D", [(1, 1, 17, 32), (2, 2, 64, 64), (1, 4, 130, 64), (2, 8, 256, 128)])
def test_backward_vs_reference_triton(ref, B, H, N, D, causal):
    _, rfb, _ = ref
    q, k, v, do = _qkv((B, H, N, D), 2, n=4)
    grads = []
    for fn in (flash_attention, rfb.flash_attention):
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        fn(qq, kk, vv, causal=causal).backward(do)
        grads.append((qq.grad, kk.grad, vv.grad))
    exp = attention_ref_grads(q, k, v, do, causal)
    for i, name in enumerate(("dq", "dk", "dv")):
        for impl in (0, 1):
            torch.testing.assert_close(grads[impl][i].float().cpu(), exp[i], atol=3e-2, rtol=3e-2,
                                       msg=f"{name} impl {impl}")
        torch.testing.assert_close(grads[0][i], grads[1][i], atol=5e-2, rtol=5e-2, msg=name)


def test_config3_backward_vs_reference_triton(ref):
    _, rfb, _ = ref
    q, k, v, do = _qkv((4, 32, 2048, 128), 3, n=4)
    grads = []
    for fn in (flash_attention, rfb.flash_attention):
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        fn(qq, kk, vv, causal=True).backward(do)
        grads.append((qq.grad, kk.grad, vv.grad))
    for i, name in enumerate(("dq", "dk", "dv")):
        d = (grads[0][i].float() - grads[1][i].float()).abs().max().item()
        assert d <= 5e-2, f"{name}: ours vs reference Triton max-abs {d:.3g}"


@pytest.mark.parametrize("M,N", [(1, 1), (1, 17), (37, 300), (8, 4096), (4, 4097), (2, 8192),
                                 (16384, 4096)])
def test_rmsnorm_vs_reference_triton(ref, M, N):
    _, _, rrn = ref
    x, r = _qkv((M, N), 4, n=2)
    g = torch.Generator(device="cuda").manual_seed(5)
    w = (1 + 0.02 * torch.randn(N, device="cuda", generator=g)).to(torch.bfloat16)
    out, h = fused_add_rmsnorm(x, r, w, 1e-6)
    rout, rh = rrn.fused_add_rmsnorm(x, r, w, 1e-6)
    assert torch.equal(h, rh)
    torch.testing.assert_close(out, rout, atol=2e-2, rtol=2e-2)
    if M * N <= 1 << 16:
        eo, _ = rmsnorm_residual(x, r, w, 1e-6)
        torch.testing.assert_close(rout.cpu(), eo, atol=2e-2, rtol=2e-2)
