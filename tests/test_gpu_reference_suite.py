"""The reference's own test suite (test/test_flash_attention.py,
test_linear.py, test_softmax.py, test_gelu.py, test_causal_self_attn.py and
its conftest.py), run UNCHANGED against this repository's drop-in packages
``cuda_transformer`` and ``cuda_autograd_fns``.

oracle/build_ref.py copies the files byte for byte (SHA-256 in MANIFEST.json)
into the git-ignored oracle/_ref/reference_tests/, which travels with the
snapshot.  Each file imports ``cuda_transformer.ops``; a child pytest process
runs them with this repository first on PYTHONPATH, so those imports bind to
this repository's operators (the test checks which module was loaded).  The
reference tests draw unseeded random inputs, so the suite runs three times.
The default precision (3xTF32) is the one the reference's FP32 tolerances
apply to."""
import hashlib
import json
import os
import subprocess
import sys

import pytest

from .conftest import ROOT

SUITE = ROOT / "oracle" / "_ref" / "reference_tests"
FILES = ["test_flash_attention.py", "test_linear.py", "test_softmax.py", "test_gelu.py",
         "test_causal_self_attn.py"]
REPEATS = 3


def _env():
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT) + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
    env.pop("CUDA_TRANSFORMER_PRECISION", None)  # the default, FP32-accurate mode
    return env


@pytest.fixture(scope="module")
def suite():
    if not (SUITE / "MANIFEST.json").exists():
        pytest.skip("reference test suite not copied: oracle/build_ref.py needs the reference "
                    "checkout on the build machine")
    manifest = json.loads((SUITE / "MANIFEST.json").read_text())["sha256"]
    for name, digest in manifest.items():
        assert hashlib.sha256((SUITE / name).read_bytes()).hexdigest() == digest, name
    assert set(FILES) <= set(manifest)
    return SUITE


@pytest.mark.gpu
def test_reference_suite_binds_to_this_repository(suite):
    out = subprocess.run(
        [sys.executable, "-c",
         "import cuda_transformer, cuda_autograd_fns, cuda_transformer.ops as o;"
         "print(cuda_transformer.__file__); print(cuda_autograd_fns.__file__);"
         "print(o.flash_attention_fwd.__module__)"],
        cwd=suite, env=_env(), capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.split()
    assert lines[0].startswith(str(ROOT / "cuda_transformer")), lines
    assert lines[1].startswith(str(ROOT / "cuda_autograd_fns")), lines


@pytest.mark.gpu
@pytest.mark.parametrize("run", range(REPEATS))
def test_reference_suite_unchanged(suite, run):
    res = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "--rootdir", str(suite),
         *FILES],
        cwd=suite, env=_env(), capture_output=True, text=True, timeout=1200)
    tail = "\n".join(res.stdout.splitlines()[-15:])
    print(tail)
    assert res.returncode == 0, tail + res.stderr[-2000:]
    assert " passed" in tail and "failed" not in tail and "error" not in tail.lower(), tail
