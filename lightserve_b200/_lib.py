"""ctypes binding of liblightserve_b200.so (declared in include/lightserve_b200.h).

The shared library is the only compute path of this package: if it cannot be
found or built, importing any operator raises. There is no PyTorch, Triton or
CPU fallback behind these functions.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "liblightserve_b200.so"
_lock = threading.Lock()
_lib = None

LSB_OK = 0
LSB_ERR_INVALID = 1
LSB_ERR_UNSUPPORTED = 2
LSB_ERR_CUDA = 3

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

IMPL_AUTO = 0
IMPL_SIMT = 1
IMPL_TCGEN05 = 2

_DTYPE_CODES = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}

# Every symbol include/lightserve_b200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_I64P = ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    "lsb_last_error": (ctypes.c_char_p, []),
    "lsb_version": (ctypes.c_char_p, []),
    "lsb_device_error": (_I, []),
    "lsb_device_error_reset": (_I, []),
    "lsb_set_programmatic_launch": (_I, [_I]),
    "lsb_selftest_bounded_wait": (_I, [_P, _P]),
    "lsb_rmsnorm_residual": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _F, _I, _P]),
    "lsb_attn_fwd": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64P, _I64P, _I64P, _I64P,
                          _F, _I, _I, _I, _P]),
    "lsb_attn_fwd_varlen": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                 _I64P, _I64P, _I64P, _I64P, _F, _I, _I, _P]),
    "lsb_attn_bwd_workspace_size": (_I64, [_I64, _I64, _I64, _I64]),
    "lsb_attn_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                          _I64P, _I64P, _I64P, _I64P, _I64P, _I64P, _I64P, _I64P,
                          _F, _I, _I, _I, _P, _I64, _P]),
    "lsb_kv_cache_write": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                _I64, _I64, _I64, _I64, _I, _P]),
    "lsb_paged_decode_workspace_size": (_I64, [_I64, _I64, _I64, _I64, _I64]),
    "lsb_paged_decode": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                              _I64, _I64, _I64, _I64, _F, _I, _P, _I64, _P]),
    "lsb_rope_kv_write": (_I, [_P, _I64, _I64, _I64, _P, _P, _I64, _P, _P, _I64, _P, _P, _P, _P,
                               _I64, _I64, _I64, _I64, _I64, _I, _P]),
    "lsb_rope_kv_write_slots": (_I, [_P, _I64, _I64, _I64, _P, _P, _I64, _P, _P, _P, _P, _P, _P,
                                     _I64, _I64, _I64, _I64, _I64, _I, _P]),
    "lsb_swiglu": (_I, [_P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "lsb_greedy_next": (_I, [_P, _I64, _I64, _I64, _I, _P, _P, _P]),
    "lsb_linear_packed_bytes": (_I64, [_I64, _I64]),
    "lsb_linear_pack": (_I, [_P, _I64, _I64, _I64, _I, _P, _I64, _P]),
    "lsb_linear": (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _P]),
    "lsb_paged_decode_static_scratch_capacity": (_I64, []),
    "lsb_paged_decode_static_scratch": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                             _I64, _I64, _I64, _I64, _I64, _F, _I, _P]),
}


def library_path() -> Path:
    return _LIB_PATH


def load(build_if_missing: bool = True):
    """Returns the loaded ctypes library, building it first if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            if not build_if_missing or os.environ.get("LSB_NO_BUILD"):
                raise RuntimeError(
                    f"{_LIB_PATH} is missing: run `python -m lightserve_b200.build` "
                    "(the CUDA extension is the only implementation of these operators)"
                )
            from . import build as _build

            _build.build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().lsb_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != LSB_OK:
        kind = {LSB_ERR_INVALID: "invalid argument", LSB_ERR_UNSUPPORTED: "unsupported",
                LSB_ERR_CUDA: "CUDA error"}.get(rc, f"status {rc}")
        raise RuntimeError(f"{what} failed ({kind}): {last_error()}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[t]
    except KeyError:
        raise AssertionError(f"unsupported dtype {t}; expected float32, bfloat16 or float16")


def strides4(t: torch.Tensor):
    return (ctypes.c_int64 * 4)(*t.stride())


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


_NULL = contextlib.nullcontext()


def device_guard(device: torch.device):
    """Makes `device` current for the launch; free when it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return _NULL
    return torch.cuda.device(device)


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class DeviceWaitError(RuntimeError):
    """A kernel of the library gave up on a bounded on-chip wait; the outputs
    of the launches since the last check are not trustworthy."""

    def __init__(self, code: int):
        self.code = code
        what = ("the device error words could not be read: " + last_error()
                if code == LSB_DEVICE_ERR_QUERY else f"a bounded wait gave up (code {code:#x})")
        super().__init__(f"lightserve_b200 device error: {what}")


LSB_DEVICE_ERR_QUERY = 0xCDA


def check_device_errors(reset: bool = True) -> None:
    """Raises DeviceWaitError if any kernel of the library timed out on an
    on-chip wait since the last reset (by default the error words are cleared
    when read, so each error is reported once). Synchronises the current
    device: call it at step or test boundaries, not between launches."""
    lib = load()
    code = lib.lsb_device_error_reset() if reset else lib.lsb_device_error()
    if code != 0:
        raise DeviceWaitError(int(code))
