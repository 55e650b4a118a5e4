"""B200-native (sm_100a) FlashAttention-2 hot path of CUDA_Transformer.

The product is the shared library ``lib/libct_b200.so`` (CUDA kernels behind
the C ABI in ``include/ct_b200.h``); ``cuda_transformer`` and
``cuda_autograd_fns`` at the repository root are the drop-in PyTorch front end
over it.  This module locates and loads the library with ctypes for callers
that use the C ABI directly (tests, benchmarks, non-torch hosts).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libct_b200.so"
HEADER_PATH = PKG_DIR.parent / "include" / "ct_b200.h"

# status codes / precision modes (include/ct_b200.h)
CT_OK = 0
CT_ERR_INVALID_ARGUMENT = 1
CT_ERR_UNSUPPORTED_HEAD_DIM = 2
CT_ERR_UNSUPPORTED_LAYOUT = 3
CT_ERR_LAUNCH_FAILED = 4
CT_ERR_DEVICE_TIMEOUT = 5
CT_ERR_CUDA = 6
CT_ERR_UNSUPPORTED_DEVICE = 7
CT_ERR_WORKSPACE_TOO_SMALL = 8
PRECISION_3XTF32 = 0
PRECISION_TF32 = 1
PRECISION_FP32 = 2
EPILOGUE_NONE = 0
EPILOGUE_GELU = 1
EPILOGUE_GELU_GRAD = 2
CT_FA2_BWD_NOALLOC_MAX_ROWS = 2097152  # batch * heads * seq_len limit of ct_fa2_bwd_noalloc
CT_DEVSTAT_TIMEOUT = 1  # watchdog word bit: a bounded device-side wait ran out
CT_WAIT_LIMIT_MIN_NS = 100000
CT_WAIT_LIMIT_MAX_NS = 60000000000

_i64p = ctypes.POINTER(ctypes.c_int64)
_fp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t

# argtypes of every exported entry point (restype int unless noted)
SIGNATURES = {
    "ct_status_string": ([_int], ctypes.c_char_p),
    "ct_version": ([], _int),
    "ct_device_status": ([_int, _int, ctypes.POINTER(ctypes.c_uint)], _int),
    "ct_fa2_fwd": ([_fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _fp, _i64, _i64, _i64, _i64, _int,
                    _int, _fp], _int),
    "ct_fa2_bwd_delta": ([_fp, _i64p, _fp, _i64p, _fp, _i64, _i64, _i64, _i64, _fp], _int),
    "ct_fa2_bwd_dq": ([_fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _fp, _i64,
                       _i64, _i64, _i64, _int, _int, _fp], _int),
    "ct_fa2_bwd_dkdv": ([_fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _fp,
                         _fp, _i64, _i64, _i64, _i64, _int, _int, _fp], _int),
    "ct_fa2_bwd_workspace_size": ([_i64, _i64, _i64, _i64], _sz),
    "ct_fa2_bwd": ([_fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp,
                    _fp, _fp, _fp, _sz, _i64, _i64, _i64, _i64, _int, _int, _fp], _int),
    "ct_fa2_bwd_fused": ([_fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p,
                          _fp, _fp, _fp, _fp, _sz, _i64, _i64, _i64, _i64, _int, _int, _fp], _int),
    "ct_fa2_bwd_noalloc": ([_fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp, _i64p, _fp,
                            _i64p, _fp, _fp, _fp, _i64, _i64, _i64, _i64, _int, _int, _fp], _int),
    "ct_linear_fwd": ([_fp, _i64p, _fp, _i64p, _fp, _i64, _fp, _i64, _i64, _i64, _i64, _i64, _int,
                       _fp], _int),
    "ct_linear_workspace_size": ([_i64, _i64, _i64, _i64], _sz),
    "ct_linear_fwd_ex": ([_fp, _i64p, _fp, _i64p, _fp, _i64, _fp, _i64, _i64, _i64, _i64, _i64,
                          _int, _int, _fp, _fp, _fp, _int, _fp, _sz, _fp], _int),
    "ct_linear_fwd_ws": ([_fp, _i64p, _fp, _i64p, _fp, _i64, _fp, _i64, _i64, _i64, _i64, _i64,
                          _int, _fp, _sz, _fp], _int),
    "ct_bias_grad_workspace_size": ([_i64, _i64, _i64], _sz),
    "ct_bias_grad": ([_fp, _i64p, _fp, _i64, _i64, _i64, _fp, _sz, _fp], _int),
    "ct_softmax_fwd": ([_fp, _fp, _i64, _i64, _fp], _int),
    "ct_softmax_bwd": ([_fp, _fp, _fp, _i64, _i64, _fp], _int),
    "ct_gelu_fwd": ([_fp, _fp, _i64, _fp], _int),
    "ct_gelu_bwd": ([_fp, _fp, _fp, _i64, _fp], _int),
    "ct_layernorm_fwd": ([_fp, _fp, _fp, _fp, _fp, _fp, _i64, _i64, ctypes.c_float, _fp], _int),
    "ct_layernorm_bwd_workspace_size": ([_i64, _i64], _sz),
    "ct_layernorm_bwd": ([_fp, _fp, _fp, _fp, _fp, _fp, _fp, _fp, _i64, _i64, _fp, _sz, _fp],
                         _int),
    "ct_cross_entropy_fwd_bwd": ([_fp, _i64, _i64, _i64, _fp, _i64, _fp, _fp], _int),
    "ct_set_wait_limit_ns": ([_int, ctypes.c_ulonglong], _int),
    "ct_get_wait_limit_ns": ([_int, ctypes.POINTER(ctypes.c_ulonglong)], _int),
    "ct_watchdog_selftest": ([_fp], _int),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Loads libct_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m cuda_transformer_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        _lib = handle
    return _lib


def strides(t) -> ctypes.Array:
    """int64[] of a tensor's element strides, for the C ABI."""
    return (ctypes.c_int64 * t.dim())(*t.stride())


def status_string(rc: int) -> str:
    return lib().ct_status_string(rc).decode()


def check(rc: int, what: str = "ct call") -> None:
    if rc != CT_OK:
        raise RuntimeError(f"{what}: {status_string(rc)} (status {rc})")


def set_wait_limit_ns(device: int, limit_ns: int) -> None:
    """Limit of every bounded device-side wait on `device` (default 2 s)."""
    check(lib().ct_set_wait_limit_ns(device, limit_ns), "ct_set_wait_limit_ns")


def wait_limit_ns(device: int = 0) -> int:
    v = ctypes.c_ulonglong(0)
    check(lib().ct_get_wait_limit_ns(device, ctypes.byref(v)), "ct_get_wait_limit_ns")
    return int(v.value)


def device_status(device: int = 0, clear: bool = False) -> int:
    """Watchdog word of a device (0 = no device-side wait has expired)."""
    v = ctypes.c_uint(0)
    check(lib().ct_device_status(device, 1 if clear else 0, ctypes.byref(v)), "ct_device_status")
    return int(v.value)
