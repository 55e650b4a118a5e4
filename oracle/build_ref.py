"""Builds oracle/_ref/libref_fa2.so -- TEST INFRASTRUCTURE.

Compiles the reference's FlashAttention-2 kernels from the reference checkout
(``Transformer_kernels/flash_attention.cuh``, included where it lies) together
with ``oracle/ref_fa2_shim.cu`` for sm_100a.  The library is git-ignored; the
GPU tests use it as a second parity reference and time it beside the product
kernels ("reference kernels rebuilt for sm_100").  Nothing in the product links
or loads it.

Usage: python oracle/build_ref.py [--reference-root DIR]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libref_fa2.so"
DEFAULT_REF = Path(os.environ.get("CT_REFERENCE_ROOT", "/root/reference"))
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")


def build_if_available(reference_root: Path = DEFAULT_REF, force: bool = False) -> Path | None:
    header = reference_root / "Transformer_kernels" / "flash_attention.cuh"
    if not header.exists():
        return OUT if OUT.exists() else None
    src = HERE / "ref_fa2_shim.cu"
    if OUT.exists() and not force and OUT.stat().st_mtime > max(src.stat().st_mtime,
                                                               header.stat().st_mtime):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cmd = [NVCC, "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
           "-I", str(reference_root), str(src), "-o", str(OUT)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("building the reference FA2 kernels failed")
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", type=Path, default=DEFAULT_REF)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_if_available(a.reference_root, a.force))


if __name__ == "__main__":
    main()
