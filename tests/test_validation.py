"""The reference's argument checks (AssertionError before any launch), on CPU
tensors: kernels/tests/test_flash_attention.py:80-122,
kernels/tests/test_flash_attention_backward.py:127-139,
kernels/tests/test_fused_rmsnorm_residual.py:80-96."""
import pytest
import torch

from lightserve_b200.kernels import (flash_attention, flash_attention_forward, fused_add_rmsnorm,
                                     paged_decode_attention)

FNS = [flash_attention_forward, flash_attention]


@pytest.mark.parametrize("fn", FNS)
def test_rejects_shape_mismatch(fn):
    with pytest.raises(AssertionError):
        fn(torch.randn(1, 2, 16, 32), torch.randn(1, 2, 16, 32), torch.randn(1, 2, 8, 32))


@pytest.mark.parametrize("fn", FNS)
def test_rejects_dtype_mismatch(fn):
    with pytest.raises(AssertionError):
        fn(torch.randn(1, 2, 16, 32), torch.randn(1, 2, 16, 32, dtype=torch.float16), torch.randn(1, 2, 16, 32))


@pytest.mark.parametrize("fn", FNS)
def test_rejects_wrong_ndim(fn):
    with pytest.raises(AssertionError):
        fn(torch.randn(2, 16, 32), torch.randn(2, 16, 32), torch.randn(2, 16, 32))


@pytest.mark.parametrize("fn", FNS)
def test_rejects_cpu_tensor(fn):
    with pytest.raises(AssertionError):
        fn(torch.randn(1, 2, 16, 32), torch.randn(1, 2, 16, 32), torch.randn(1, 2, 16, 32))


@pytest.mark.parametrize("fn", FNS)
def test_rejects_head_dim_mismatch(fn):
    with pytest.raises(AssertionError):
        fn(torch.randn(1, 2, 16, 32), torch.randn(1, 2, 16, 32), torch.randn(1, 2, 16, 64))


def test_rmsnorm_rejects_shape_mismatch():
    with pytest.raises(AssertionError):
        fused_add_rmsnorm(torch.randn(4, 8), torch.randn(4, 9), torch.randn(8))


def test_rmsnorm_rejects_noncontiguous_input():
    with pytest.raises(AssertionError):
        fused_add_rmsnorm(torch.randn(8, 4).t(), torch.randn(4, 8), torch.randn(8))


def test_rmsnorm_rejects_cpu():
    with pytest.raises(AssertionError):
        fused_add_rmsnorm(torch.randn(4, 8), torch.randn(4, 8), torch.randn(8))


def test_paged_decode_rejects_bad_tables():
    q = torch.randn(2, 4, 64)
    kc = torch.randn(8, 4, 16, 64)
    with pytest.raises(AssertionError):
        paged_decode_attention(q, kc, kc, torch.zeros(2, 4, dtype=torch.int64), torch.ones(2, dtype=torch.int32))


def test_swiglu_rejects_bad_input():
    from lightserve_b200.kernels import silu_and_mul
    with pytest.raises(AssertionError):
        silu_and_mul(torch.zeros(4, 6))  # CPU tensor
    with pytest.raises(AssertionError):
        silu_and_mul(torch.zeros(4, 5, device="meta"))  # odd width


def test_forward_host_rejects_device_tensors():
    from lightserve_b200.kernels import flash_attention_forward_host
    q = torch.zeros(1, 1, 4, 8, device="meta")
    with pytest.raises(AssertionError):
        flash_attention_forward_host(q, q, q)


def test_varlen_rejects_bad_input():
    from lightserve_b200.kernels import flash_attention_varlen
    cu = torch.tensor([0, 16], dtype=torch.int32)
    with pytest.raises(AssertionError):  # [B, H, N, D] instead of packed [T, H, D]
        flash_attention_varlen(*(torch.randn(1, 2, 16, 64) for _ in range(3)), cu, 16)
    with pytest.raises(AssertionError):  # shape mismatch
        flash_attention_varlen(torch.randn(16, 2, 64), torch.randn(16, 2, 64), torch.randn(8, 2, 64), cu, 16)
    with pytest.raises(AssertionError):  # CPU tensors
        flash_attention_varlen(*(torch.randn(16, 2, 64, dtype=torch.bfloat16) for _ in range(3)), cu, 16)


def test_rope_kv_write_slots_rejects_bad_input():
    from lightserve_b200.kernels import rope_kv_write_slots
    qkv = torch.randn(4, 3, 2, 8)
    cache = torch.zeros(4, 2, 16, 8)
    with pytest.raises(AssertionError):  # slot mapping must be int64
        rope_kv_write_slots(qkv, torch.ones(8, 8), torch.ones(8, 8), torch.arange(4),
                            torch.arange(4, dtype=torch.int32), torch.empty(4, 2, 8), None, cache, cache.clone())
