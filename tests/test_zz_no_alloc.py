"""ct_fa2_bwd_noalloc: the FlashAttention-2 backward for callers that cannot
allocate device memory (a plugin handed only tensor pointers by a host whose
allocator it cannot reach, a service with no cudaMalloc after start-up).  It
keeps the delta temporary in a fixed array inside the library instead of a
caller workspace.

The GPU tests call it through the C ABI on two problems in a row (so a stale
array left by the first call would show up in the second) and check it
  * bit for bit against the per-kernel entry points (ct_fa2_bwd_delta,
    ct_fa2_bwd_dq, ct_fa2_bwd_dkdv), which run the same deterministic
    kernels with caller-owned delta,
  * bit for bit against ct_fa2_bwd, which runs the same kernels with a
    caller workspace, and
  * against the FP64 oracle within the precision mode's tolerance,
for every backward path it can reach: the tensor-core kernels (3xTF32 and
TF32, head dim 64 and 128, including the two-pass head-dim-128 dK/dV) and
the CUDA-core kernels (FP32 mode).  The CPU tests check that oversized and
overflowing shapes are rejected during validation, before any CUDA call.
Collected last on purpose: a run that stops at the first failure has run
every other test by then."""
import ctypes

import pytest
import torch

import cuda_transformer_b200 as cb
from oracle import fa2 as orc

from . import ct_helpers as H

TOL = {cb.PRECISION_3XTF32: 1e-4, cb.PRECISION_TF32: 2e-3, cb.PRECISION_FP32: 1e-5}


def _noalloc(q, k, v, o, do, lse, causal, prec):
    B, Hh, T, D = q.shape
    dq, dk, dv = (torch.empty(B, Hh, T, D, device=q.device) for _ in range(3))
    rc = cb.lib().ct_fa2_bwd_noalloc(H._p(q), cb.strides(q), H._p(k), cb.strides(k), H._p(v),
                                     cb.strides(v), H._p(o), cb.strides(o), H._p(do),
                                     cb.strides(do), H._p(lse), cb.strides(lse), H._p(dq),
                                     H._p(dk), H._p(dv), B, Hh, T, D, int(causal), prec,
                                     H._stream())
    cb.check(rc, "ct_fa2_bwd_noalloc")
    return dq, dk, dv


# (precision, head dim): every backward path the entry point dispatches to
PATHS = [(cb.PRECISION_3XTF32, 64), (cb.PRECISION_TF32, 64), (cb.PRECISION_TF32, 128),
         (cb.PRECISION_3XTF32, 128), (cb.PRECISION_FP32, 64), (cb.PRECISION_FP32, 128)]


@pytest.mark.gpu
@pytest.mark.parametrize("prec,D", PATHS)
def test_noalloc_matches_workspace_entry_point_and_oracle(cuda_device, prec, D):
    # two calls in a row; the second problem has fewer rows than the first
    for i, (B, Hh, T, causal) in enumerate([(2, 4, 256, True), (1, 3, 200, False)]):
        g = torch.Generator().manual_seed(500 + i)
        q, k, v, do = (torch.randn(B, Hh, T, D, generator=g).to(cuda_device) for _ in range(4))
        o, lse = H.fa2_fwd(q, k, v, causal, prec)
        ref = H.fa2_bwd_split(q, k, v, o, do, lse, causal, prec)
        ws_ref = H.fa2_bwd(q, k, v, o, do, lse, causal, prec)
        got = _noalloc(q, k, v, o, do, lse, causal, prec)
        torch.cuda.synchronize()
        for name, a, b, c in zip(("dQ", "dK", "dV"), got, ref, ws_ref):
            assert torch.equal(a, b), (i, name, H.rel_err(a, b))
            assert torch.equal(a, c), (i, name, H.rel_err(a, c))
        qn, kn, vn, dn = (t.cpu().double().numpy() for t in (q, k, v, do))
        o_ref, l_ref = orc.attention_fwd(qn, kn, vn, causal)
        grads = orc.attention_bwd(qn, kn, vn, o_ref, dn, l_ref, causal)
        for name, a, r in zip(("dQ", "dK", "dV"), got, grads):
            assert H.rel_err(a, r) < TOL[prec], (i, name, H.rel_err(a, r))
    H.assert_device_clean()


def _call_with_shape(B, Hh, T, D):
    """Calls the entry point with dummy (never dereferenced) pointers."""
    p = ctypes.c_void_p(256)
    s4 = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    s3 = (ctypes.c_int64 * 3)(1, 1, 1)
    return cb.lib().ct_fa2_bwd_noalloc(p, s4, p, s4, p, s4, p, s4, p, s4, p, s3, p, p, p, B, Hh,
                                       T, D, 1, cb.PRECISION_3XTF32, None)


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    rows = cb.CT_FA2_BWD_NOALLOC_MAX_ROWS + 1  # rejected during validation, nothing launched
    assert _call_with_shape(1, 1, rows, 64) == cb.CT_ERR_WORKSPACE_TOO_SMALL
    assert _call_with_shape(4, 32, 16385, 64) == cb.CT_ERR_WORKSPACE_TOO_SMALL


@pytest.mark.parametrize("B,Hh,T", [
    (2 ** 62 + 1, 4, 1),       # B*H*T would wrap to 4
    (2 ** 62, 4, 1),           # B*H*T would wrap to 0
    (2 ** 40, 2 ** 40, 1),     # B*H overflows int64
    (1, 1, 2 ** 31),           # T beyond the kernels' 32-bit index range
    (2 ** 31, 1, 1),           # B*H beyond 2^31
    (-1, 4, 4),
])
def test_noalloc_rejects_overflowing_shapes(B, Hh, T):
    assert _call_with_shape(B, Hh, T, 64) == cb.CT_ERR_INVALID_ARGUMENT


def test_noalloc_rejects_bad_head_dim_and_precision():
    assert _call_with_shape(1, 1, 16, 48) == cb.CT_ERR_UNSUPPORTED_HEAD_DIM
    p = ctypes.c_void_p(256)
    s4 = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    s3 = (ctypes.c_int64 * 3)(1, 1, 1)
    rc = cb.lib().ct_fa2_bwd_noalloc(p, s4, p, s4, p, s4, p, s4, p, s4, p, s3, p, p, p, 1, 1, 16,
                                     64, 1, 7, None)
    assert rc == cb.CT_ERR_INVALID_ARGUMENT
