"""In-tree build of the native libraries.

* ``cuda_transformer_b200/lib/libct_b200.so`` -- every CUDA kernel plus the
  C ABI declared in ``include/ct_b200.h``; compiled by nvcc for sm_100a only,
  CUDA runtime linked statically, no torch dependency.
* ``cuda_transformer/_C<ext>`` -- the PyTorch operator registrations
  (``torch.ops.cuda_transformer.*``); a thin C++ shim over the C ABI.
* ``tests/diag/libct_diag.so`` -- TEST-ONLY diagnostics (operand-layout checks
  and a tensor-pipe throughput probe, ``tests/diag/ct_diag.h``); not linked
  into or loaded by the product.

Objects go to ``cuda_transformer_b200/_build``; a translation unit is rebuilt
when it, or any header next to it, is newer than its object.

Usage: ``python -m cuda_transformer_b200.build [--force] [--jobs N]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "lib" / "libct_b200.so"
INCLUDE = ROOT / "include"
TORCH_EXT_SRC = CSRC / "torch_ext" / "ops.cpp"
TORCH_EXT_OUT = ROOT / "cuda_transformer" / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))
DIAG_DIR = ROOT / "tests" / "diag"
DIAG_SRC = DIAG_DIR / "ct_diag.cu"
DIAG_LIB = DIAG_DIR / "libct_diag.so"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills",
    *ARCH, "-I", str(INCLUDE), "-I", str(CSRC),
]


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")
    # keep ptxas spill warnings visible
    for line in (res.stdout + res.stderr).splitlines():
        if "spill" in line.lower() and "0 bytes spill" not in line:
            sys.stderr.write(line + "\n")


def build_core(force: bool = False, jobs: int | None = None) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    work = []
    for src in sources:
        obj = OBJ / (src.stem + ".o")
        if force or _stale(obj, [src, *headers]):
            work.append([NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if work:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(_run, work))
    objs = [OBJ / (s.stem + ".o") for s in sources]
    if force or _stale(LIB, objs):
        _run([NVCC, "-shared", *ARCH, "-cudart", "static", "-o", str(LIB), *map(str, objs)])
    return LIB


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension

    inc = [f"-I{p}" for p in cpp_extension.include_paths()]
    inc += [f"-I{sysconfig.get_paths()['include']}", f"-I{CUDA_HOME}/include", f"-I{INCLUDE}"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = ["-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths()]
    libs = libdirs + ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
                      f"-L{LIB.parent}", "-lct_b200",
                      "-Wl,-rpath,$ORIGIN/../cuda_transformer_b200/lib",
                      *[f"-Wl,-rpath,{p}" for p in cpp_extension.library_paths()]]
    return inc + defs, libs


def build_torch_ext(force: bool = False) -> Path:
    deps = [TORCH_EXT_SRC, LIB, *INCLUDE.glob("*.h")]
    if not (force or _stale(TORCH_EXT_OUT, deps)):
        return TORCH_EXT_OUT
    cflags, libs = _torch_flags()
    _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", *cflags, str(TORCH_EXT_SRC),
          "-o", str(TORCH_EXT_OUT), *libs])
    return TORCH_EXT_OUT


def build_diag(force: bool = False) -> Path | None:
    """Test-only diagnostics library (absent from a product-only checkout)."""
    if not DIAG_SRC.exists():
        return None
    deps = [DIAG_SRC, DIAG_DIR / "ct_diag.h", *_headers()]
    if force or _stale(DIAG_LIB, deps):
        _run([NVCC, *NVCC_FLAGS, "-I", str(DIAG_DIR), "-shared", "-cudart", "static",
              str(DIAG_SRC), "-o", str(DIAG_LIB)])
    return DIAG_LIB


def build_all(force: bool = False, jobs: int | None = None) -> None:
    build_core(force, jobs)
    build_torch_ext(force)
    build_diag(force)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args()
    build_all(a.force, a.jobs)
    print(LIB)
    print(TORCH_EXT_OUT)


if __name__ == "__main__":
    main()
