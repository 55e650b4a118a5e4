"""Failure detection on the device, exercised without a fault: the device
wait limit is lowered to 1 ms, ct_watchdog_selftest launches one CTA whose
waits on a barrier phase that nothing completes run out, and the CTA takes
the attention kernels' abort teardown (MMA commit + bounded drain, TMEM
release).  The test checks that the call returns promptly, that
ct_device_status reports CT_DEVSTAT_TIMEOUT, and that after the word is
cleared (and the limit restored) a normal FlashAttention-2 forward + backward
runs and matches the oracle."""
import time

import pytest
import torch

import cuda_transformer_b200 as cb
from oracle import fa2 as orc

from . import ct_helpers as H


@pytest.mark.gpu
def test_short_wait_limit_expires_and_device_stays_usable(cuda_device):
    idx = cuda_device.index or 0
    H.assert_device_clean(idx)
    default = cb.wait_limit_ns(idx)
    assert default == 2_000_000_000
    try:
        cb.set_wait_limit_ns(idx, 1_000_000)  # 1 ms
        assert cb.wait_limit_ns(idx) == 1_000_000
        t0 = time.perf_counter()
        cb.check(cb.lib().ct_watchdog_selftest(H._stream()), "ct_watchdog_selftest")
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert elapsed < 1.0, elapsed  # the waits gave up after ~1-2 ms
        assert cb.device_status(idx, clear=True) == cb.CT_DEVSTAT_TIMEOUT
        assert cb.device_status(idx) == 0
    finally:
        cb.set_wait_limit_ns(idx, default)
        cb.device_status(idx, clear=True)
    assert cb.wait_limit_ns(idx) == default
    # the context is intact: a normal attention call succeeds afterwards
    g = torch.Generator().manual_seed(7)
    q, k, v, do = (torch.randn(1, 2, 192, 64, generator=g).to(cuda_device) for _ in range(4))
    o, lse = H.fa2_fwd(q, k, v, True)
    dq, dk, dv = H.fa2_bwd(q, k, v, o, do, lse, True)
    torch.cuda.synchronize()
    qn, kn, vn, dn = (t.cpu().double().numpy() for t in (q, k, v, do))
    o_ref, l_ref = orc.attention_fwd(qn, kn, vn, True)
    refs = orc.attention_bwd(qn, kn, vn, o_ref, dn, l_ref, True)
    assert H.rel_err(o, o_ref) < 1e-4 and H.rel_err(lse, l_ref) < 1e-4
    for got, ref in zip((dq, dk, dv), refs):
        assert H.rel_err(got, ref) < 1e-4
    H.assert_device_clean(idx)


def test_wait_limit_range_checked_before_any_device_call():
    assert cb.lib().ct_set_wait_limit_ns(0, cb.CT_WAIT_LIMIT_MIN_NS - 1) == cb.CT_ERR_INVALID_ARGUMENT
    assert cb.lib().ct_set_wait_limit_ns(0, cb.CT_WAIT_LIMIT_MAX_NS + 1) == cb.CT_ERR_INVALID_ARGUMENT
    assert cb.lib().ct_get_wait_limit_ns(0, None) == cb.CT_ERR_INVALID_ARGUMENT
