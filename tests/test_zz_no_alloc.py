"""ct_fa2_bwd_noalloc: the FlashAttention-2 backward for callers that cannot
allocate device memory (a plugin handed only tensor pointers, a service with
no cudaMalloc after start-up).  It keeps the delta temporary in a fixed array
inside the library instead of a caller workspace.  These tests call it
through the C ABI and compare it with ct_fa2_bwd (which takes a workspace) on
two calls in a row with different problems, so a stale array from the first
call would show up in the second.  Collected last on purpose."""
import ctypes

import pytest
import torch

import cuda_transformer_b200 as cb

from . import ct_helpers as H


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


@pytest.mark.gpu
@pytest.mark.parametrize("prec", [cb.PRECISION_3XTF32, cb.PRECISION_TF32])
def test_noalloc_matches_workspace_entry_point(cuda_device, prec):
    tol = 1e-4 if prec == cb.PRECISION_3XTF32 else 2e-3
    for i, (B, Hh, T, D, causal) in enumerate([(2, 4, 256, 64, True), (1, 3, 200, 64, False)]):
        g = torch.Generator().manual_seed(500 + i)
        q, k, v, do = (torch.randn(B, Hh, T, D, generator=g).to(cuda_device) for _ in range(4))
        o, lse = H.fa2_fwd(q, k, v, causal, prec)
        ref = H.fa2_bwd(q, k, v, o, do, lse, causal, prec)
        got = _noalloc(q, k, v, o, do, lse, causal, prec)
        torch.cuda.synchronize()
        for name, a, b in zip(("dQ", "dK", "dV"), got, ref):
            assert H.rel_err(a, b) < tol, (i, name, H.rel_err(a, b))
    H.assert_device_clean()


@pytest.mark.gpu
def test_noalloc_rejects_problems_beyond_the_fixed_scratch(cuda_device):
    x = torch.zeros(16, device=cuda_device)
    s4 = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    s3 = (ctypes.c_int64 * 3)(1, 1, 1)
    rows = cb.CT_FA2_BWD_NOALLOC_MAX_ROWS + 1  # rejected during validation, nothing launched
    rc = cb.lib().ct_fa2_bwd_noalloc(H._p(x), s4, H._p(x), s4, H._p(x), s4, H._p(x), s4,
                                     H._p(x), s4, H._p(x), s3, H._p(x), H._p(x), H._p(x), 1, 1,
                                     rows, 64, 1, cb.PRECISION_3XTF32, H._stream())
    assert rc == cb.CT_ERR_WORKSPACE_TOO_SMALL
