"""fused_add_rmsnorm on the GPU vs the oracle (shapes/dtypes/tolerances of
kernels/tests/test_fused_rmsnorm_residual.py) and vs lightserve's own kernel
outputs (golden fixtures)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.rmsnorm import rmsnorm_residual
from lightserve_b200.kernels import fused_add_rmsnorm

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1), (1, 17), (37, 300), (8, 4096), (4, 4097), (2, 8192), (3, 40000)]
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


@pytest.mark.parametrize("M,N", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
def test_matches_oracle(M, N, dtype):
    torch.manual_seed(0)
    x = torch.randn(M, N, device="cuda", dtype=dtype)
    r = torch.randn(M, N, device="cuda", dtype=dtype)
    w = torch.randn(N, device="cuda", dtype=dtype)
    out, h = fused_add_rmsnorm(x, r, w, 1e-6)
    eo, eh = rmsnorm_residual(x, r, w, 1e-6)
    torch.testing.assert_close(h.cpu(), eh, atol=0, rtol=0)  # h is an exact dtype add
    atol = 1e-5 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(out.cpu(), eo, atol=atol, rtol=atol)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("rmsnorm_*.npz")), ids=lambda p: p.stem)
def test_matches_reference_kernel_golden(path):
    g = np.load(path)
    x, r, w = (torch.from_numpy(g[n]).cuda() for n in ("x", "r", "w"))
    out, h = fused_add_rmsnorm(x, r, w, float(g["eps"]))
    np.testing.assert_array_equal(h.cpu().numpy(), g["h"])
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], atol=1e-5, rtol=1e-5)


def test_row_strided_views():
    torch.manual_seed(0)
    base = torch.randn(16, 1024, device="cuda", dtype=torch.bfloat16)
    x = base[:, :512]  # row stride 1024
    r = torch.randn(16, 512, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(512, device="cuda", dtype=torch.bfloat16)
    out, h = fused_add_rmsnorm(x, r, w)
    eo, eh = rmsnorm_residual(x, r, w, 1e-6)
    torch.testing.assert_close(out.cpu(), eo, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(h.cpu(), eh, atol=0, rtol=0)


def test_output_is_unit_rms_before_weight():
    torch.manual_seed(0)
    x = torch.randn(16, 512, device="cuda")
    r = torch.randn(16, 512, device="cuda")
    out, _ = fused_add_rmsnorm(x, r, torch.ones(512, device="cuda"), eps=1e-6)
    torch.testing.assert_close(out.pow(2).mean(-1).sqrt(), torch.ones(16, device="cuda"), atol=1e-3, rtol=1e-3)


def test_zero_row_stays_finite_via_eps():
    z = torch.zeros(4, 128, device="cuda")
    out, h = fused_add_rmsnorm(z, z.clone(), torch.randn(128, device="cuda"), eps=1e-6)
    assert torch.all(torch.isfinite(out)) and torch.all(h == 0)


def test_full_size_config_properties():
    """BASELINE config 4 (16384 x 4096 bf16): h is bit-exact x + r and a sample
    of rows matches the oracle."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(16384, 4096, device="cuda", dtype=torch.bfloat16, generator=g)
    r = torch.randn(16384, 4096, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (1 + 0.02 * torch.randn(4096, device="cuda", generator=g)).to(torch.bfloat16)
    out, h = fused_add_rmsnorm(x, r, w, 1e-6)
    assert torch.equal(h, x + r)
    rows = torch.randint(0, 16384, (64,), generator=g, device="cuda")
    eo, _ = rmsnorm_residual(x[rows], r[rows], w, 1e-6)
    torch.testing.assert_close(out[rows].cpu(), eo, atol=2e-2, rtol=2e-2)
