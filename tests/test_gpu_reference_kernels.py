"""Parity against the reference's own FlashAttention-2 kernels
(Transformer_kernels/flash_attention.cuh) rebuilt for sm_100a by
oracle/build_ref.py: same inputs through both, on the reference test grid and
BASELINE config 1.  Both approximate the exact math; their outputs must agree
within the FP32-mode tolerance (1e-4 relative)."""
import ctypes
from pathlib import Path

import pytest
import torch

from . import ct_helpers as H
from .conftest import ROOT

REF_LIB = ROOT / "oracle" / "_ref" / "libref_fa2.so"
GRID = [(1, 1, 64, 128, False), (1, 1, 64, 128, True), (1, 1, 65, 64, True),
        (2, 4, 128, 32, False), (2, 4, 128, 64, True), (2, 4, 257, 64, True),
        (1, 2, 512, 128, True), (2, 4, 256, 64, True), (2, 4, 256, 64, False)]


@pytest.fixture(scope="module")
def ref():
    if not REF_LIB.exists():
        pytest.skip("reference kernels not built (oracle/build_ref.py needs the reference checkout)")
    lib = ctypes.CDLL(str(REF_LIB))
    vp, i = ctypes.c_void_p, ctypes.c_int
    lib.ref_fa2_fwd.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, i, vp]
    lib.ref_fa2_bwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, i, vp]
    return lib


def _ref_run(lib, q, k, v, do, causal):
    B, Hh, T, D = q.shape
    P = H._p
    o, dq, dk, dv = (torch.empty_like(q) for _ in range(4))
    lse = torch.empty(B, Hh, T, device=q.device)
    delta = torch.empty(B, Hh, T, device=q.device)
    assert lib.ref_fa2_fwd(P(q), P(k), P(v), P(o), P(lse), B, Hh, T, D, int(causal), H._stream()) == 0
    assert lib.ref_fa2_bwd(P(q), P(k), P(v), P(o), P(do), P(lse), P(dq), P(dk), P(dv), P(delta),
                           B, Hh, T, D, int(causal), H._stream()) == 0
    torch.cuda.synchronize()
    return o, lse, dq, dk, dv


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hh,T,D,causal", GRID)
def test_matches_reference_kernels(cuda_device, ref, B, Hh, T, D, causal):
    g = torch.Generator().manual_seed(T * 3 + D)
    q, k, v = (torch.randn(B, Hh, T, D, generator=g).to(cuda_device) for _ in range(3))
    do = torch.rand(B, Hh, T, D, generator=g).to(cuda_device)
    r_o, r_l, r_dq, r_dk, r_dv = _ref_run(ref, q, k, v, do, causal)
    o, lse = H.fa2_fwd(q, k, v, causal)
    dq, dk, dv = H.fa2_bwd(q, k, v, o, do, lse, causal)
    for name, a, b in (("O", o, r_o), ("L", lse, r_l), ("dQ", dq, r_dq), ("dK", dk, r_dk),
                       ("dV", dv, r_dv)):
        assert H.rel_err(a, b) < 1e-4, (name, H.rel_err(a, b))
    H.assert_device_clean()


@pytest.mark.gpu
def test_timing_against_reference_kernels_config2(cuda_device, ref, record_property):
    """BASELINE config 2 (B=4, H=32, N=4096, D=64, causal): fwd+bwd time of the
    reference kernels rebuilt for sm_100a vs this implementation (3xTF32) on
    the same B200, CUDA events, one warm-up each."""
    B, Hh, T, D = 4, 32, 4096, 64
    g = torch.Generator(device=cuda_device).manual_seed(0)
    q, k, v, do = (torch.randn(B, Hh, T, D, device=cuda_device, generator=g) for _ in range(4))

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    def ours():
        o, lse = H.fa2_fwd(q, k, v, True)
        H.fa2_bwd(q, k, v, o, do, lse, True)

    t_ref = timed(lambda: _ref_run(ref, q, k, v, do, True), 1)
    t_ours = timed(ours, 5)
    flops = 3.5 * 4.0 * B * Hh * T * T * D * 0.5
    msg = (f"config2 fwd+bwd: reference kernels {t_ref:.1f} ms ({flops / t_ref / 1e9:.2f} TFLOPS), "
           f"this implementation {t_ours:.2f} ms ({flops / t_ours / 1e9:.1f} TFLOPS), "
           f"speed-up {t_ref / t_ours:.1f}x")
    print(msg)
    record_property("config2_timing", msg)
    assert t_ours < t_ref
    H.assert_device_clean()
