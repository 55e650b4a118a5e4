"""Builds the reference-side test infrastructure under oracle/_ref/ -- TEST
INFRASTRUCTURE, git-ignored, carried to the GPU box with the snapshot.

* ``oracle/_ref/libref_fa2.so``: the reference's FlashAttention-2 kernels
  compiled from the reference checkout (``Transformer_kernels/flash_attention.cuh``,
  included where it lies) together with ``oracle/ref_fa2_shim.cu`` for sm_100a.
  The GPU tests use it as a second parity reference and time it beside the
  product kernels ("reference kernels rebuilt for sm_100").
* ``oracle/_ref/reference_tests/``: the reference's own test suite
  (``test/*.py``), copied byte for byte, so ``tests/test_gpu_reference_suite.py``
  can run it unchanged against this repository's drop-in packages on a machine
  that has no reference checkout.  ``MANIFEST.json`` records each file's
  SHA-256.

Nothing in the product links, loads or imports any of it.

The reference checkout is found from ``--reference-root``, else the
``CT_REFERENCE_ROOT`` environment variable, else the ``reference_path`` field
of the repository's ``BASELINE.json``; without one, the existing outputs are
kept.

Usage: python oracle/build_ref.py [--reference-root DIR] [--force]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
OUT_DIR = HERE / "_ref"
OUT = OUT_DIR / "libref_fa2.so"
TESTS_OUT = OUT_DIR / "reference_tests"
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
# the reference suite's files (test/), run unchanged
REFERENCE_TEST_FILES = ("conftest.py", "test_flash_attention.py", "test_linear.py",
                        "test_softmax.py", "test_gelu.py", "test_causal_self_attn.py")


def default_reference_root() -> Path | None:
    env = os.environ.get("CT_REFERENCE_ROOT")
    if env:
        return Path(env)
    baseline = REPO / "BASELINE.json"
    if baseline.exists():
        path = json.loads(baseline.read_text()).get("reference_path")
        if path:
            return Path(path)
    return None


def _build_kernels(reference_root: Path, force: bool) -> Path | None:
    header = reference_root / "Transformer_kernels" / "flash_attention.cuh"
    if not header.exists():
        return OUT if OUT.exists() else None
    src = HERE / "ref_fa2_shim.cu"
    if OUT.exists() and not force and OUT.stat().st_mtime > max(src.stat().st_mtime,
                                                               header.stat().st_mtime):
        return OUT
    OUT_DIR.mkdir(exist_ok=True)
    cmd = [NVCC, "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
           "-I", str(reference_root), str(src), "-o", str(OUT)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("building the reference FA2 kernels failed")
    return OUT


def _copy_reference_tests(reference_root: Path) -> Path | None:
    src_dir = reference_root / "test"
    if not src_dir.is_dir():
        return TESTS_OUT if TESTS_OUT.exists() else None
    TESTS_OUT.mkdir(parents=True, exist_ok=True)
    manifest = {}
    for name in REFERENCE_TEST_FILES:
        src = src_dir / name
        if not src.exists():
            continue
        data = src.read_bytes()
        (TESTS_OUT / name).write_bytes(data)
        manifest[name] = hashlib.sha256(data).hexdigest()
    (TESTS_OUT / "MANIFEST.json").write_text(json.dumps(
        {"source": "test/ of the reference checkout, copied unchanged", "sha256": manifest},
        indent=1))
    return TESTS_OUT


def build_if_available(reference_root: Path | None = None, force: bool = False) -> Path | None:
    root = reference_root or default_reference_root()
    if root is None or not root.exists():
        return OUT if OUT.exists() else None
    _copy_reference_tests(root)
    return _build_kernels(root, force)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", type=Path, default=None)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_if_available(a.reference_root, a.force))
    print(TESTS_OUT if TESTS_OUT.exists() else "reference tests: no checkout found")


if __name__ == "__main__":
    main()
