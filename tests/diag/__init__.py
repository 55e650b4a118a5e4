"""Loader of the TEST-ONLY diagnostics library tests/diag/libct_diag.so
(built by ``python -m cuda_transformer_b200.build``; declared in ct_diag.h)."""
from __future__ import annotations

import ctypes
from pathlib import Path

DIAG_DIR = Path(__file__).resolve().parent
LIB_PATH = DIAG_DIR / "libct_diag.so"
HEADER_PATH = DIAG_DIR / "ct_diag.h"

_fp = ctypes.c_void_p
_int = ctypes.c_int
SIGNATURES = {
    "ct_diag_umma_tf32": [_int, _fp, _fp, _fp, _int, _fp],
    "ct_diag_umma_m64": [_int, _fp, _fp, _fp, _int, _fp],
    "ct_diag_umma_pair": [_int, _fp, _fp, _fp, _int, _fp],
    "ct_diag_mma_rate": [_int, _int, _int, _int, _fp, _fp],
    "ct_diag_status": [ctypes.POINTER(ctypes.c_uint)],
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m cuda_transformer_b200.build`")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(h, name)
            fn.argtypes = args
            fn.restype = _int
        _lib = h
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what}: status {rc}")


def status() -> int:
    v = ctypes.c_uint(0)
    check(lib().ct_diag_status(ctypes.byref(v)), "ct_diag_status")
    return int(v.value)
