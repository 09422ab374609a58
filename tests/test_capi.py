"""The C-ABI library loads without a GPU, exports every symbol the header
declares, and rejects bad arguments before touching the device."""
import ctypes
import re

from conftest import ROOT
from lightserve_b200 import _lib


def _declared():
    text = (ROOT / "include" / "lightserve_b200.h").read_text()
    return sorted(set(re.findall(r"LSB_API\s+[\w\s\*]+?\b(lsb_\w+)\s*\(", text)))


def test_header_declares_all_bound_symbols():
    assert _declared() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.lsb_version()


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.lsb_attn_bwd_workspace_size(4, 32, 2048, 128) == 4 * 4 * 32 * 2048 + 4 * 4 * 32 * 2048 * 128 + 256
    assert lib.lsb_attn_bwd_workspace_size(0, 1, 1, 1) == 0
    # A context that fits one 512-token partition needs no scratch.
    assert lib.lsb_paged_decode_workspace_size(64, 16, 128, 32, 16) == 0
    parts = -(-(264 * 16) // 512)
    assert lib.lsb_paged_decode_workspace_size(64, 16, 128, 264, 16) == 4 * 64 * 16 * parts * 130


def test_invalid_arguments_rejected_without_launch():
    lib = _lib.load()
    rc = lib.lsb_rmsnorm_residual(None, None, None, None, None, -1, 4, 4, 4, 4, 4, 1e-6, 1, None)
    assert rc == _lib.LSB_ERR_INVALID and "negative" in _lib.last_error()
    rc = lib.lsb_rmsnorm_residual(None, None, None, None, None, 4, 4, 4, 4, 4, 4, 1e-6, 9, None)
    assert rc == _lib.LSB_ERR_INVALID
    s = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    rc = lib.lsb_attn_fwd(None, None, None, None, None, 1, 1, 8, 0, s, s, s, s, 1.0, 0, 1, 0, None)
    assert rc == _lib.LSB_ERR_INVALID
    rc = lib.lsb_paged_decode(None, None, None, None, None, None, 1, 1, 128, 4, 12, 8, 0, 0, 0, 0,
                              1.0, 1, None, 0, None)
    assert rc == _lib.LSB_ERR_INVALID and "power of two" in _lib.last_error()
    # Empty problems are a successful no-op (no device access).
    assert lib.lsb_attn_fwd(None, None, None, None, None, 0, 1, 8, 64, s, s, s, s, 1.0, 0, 1, 0, None) == 0
