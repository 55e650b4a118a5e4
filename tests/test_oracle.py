"""CPU tests: the NumPy oracle against the reference tests' own math (torch,
float64) and against the committed golden vectors.  This pins the oracle
before any GPU result is compared with it."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import fa2 as orc
from oracle.torch_ref import sdpa_reference

from .conftest import ROOT

GOLDEN = ROOT / "tests" / "golden"

# the reference FA2 test grid (test/test_flash_attention.py:52-60)
REF_GRID = [
    (1, 1, 64, 128, False), (1, 1, 64, 128, True), (1, 1, 65, 64, True),
    (2, 4, 128, 32, False), (2, 4, 128, 64, True), (2, 4, 257, 64, True),
    (1, 2, 512, 128, True),
]


def _inputs(B, H, T, D, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, T, D, generator=g, dtype=torch.float64) for _ in range(4)]


@pytest.mark.parametrize("B,H,T,D,causal", REF_GRID)
def test_oracle_matches_reference_test_math(B, H, T, D, causal):
    q, k, v, do = _inputs(B, H, T, D, seed=T * 7 + D)
    o_ref, l_ref, dq_ref, dk_ref, dv_ref = sdpa_reference(q, k, v, do, causal)
    o, lse = orc.attention_fwd(q.numpy(), k.numpy(), v.numpy(), causal)
    np.testing.assert_allclose(o, o_ref.numpy(), rtol=0, atol=1e-12)
    np.testing.assert_allclose(lse, l_ref.numpy(), rtol=0, atol=1e-12)
    dq, dk, dv = orc.attention_bwd(q.numpy(), k.numpy(), v.numpy(), o, do.numpy(), lse, causal)
    for got, ref in ((dq, dq_ref), (dk, dk_ref), (dv, dv_ref)):
        np.testing.assert_allclose(got, ref.numpy(), rtol=0, atol=1e-11)


@pytest.mark.parametrize("T,causal,br,bc", [(65, True, 16, 16), (100, False, 16, 16),
                                            (257, True, 128, 64), (130, True, 128, 128)])
def test_tiled_online_softmax_equals_direct(T, causal, br, bc):
    q, k, v, _ = _inputs(1, 2, T, 32, seed=T)
    o1, l1 = orc.attention_fwd(q.numpy(), k.numpy(), v.numpy(), causal)
    o2, l2 = orc.attention_fwd_tiled(q.numpy(), k.numpy(), v.numpy(), causal, br, bc)
    np.testing.assert_allclose(o2, o1, atol=1e-12)
    np.testing.assert_allclose(l2, l1, atol=1e-12)


def test_delta_matches_definition():
    q, k, v, do = _inputs(1, 2, 40, 64, seed=3)
    o, _ = orc.attention_fwd(q.numpy(), k.numpy(), v.numpy(), True)
    delta = orc.attention_bwd_delta(o, do.numpy())
    np.testing.assert_allclose(delta, (o * do.numpy()).sum(-1), atol=1e-12)


def test_fa2_golden_vectors():
    z = np.load(GOLDEN / "fa2_golden.npz")
    names = sorted({k.split("/")[0] for k in z.files})
    assert len(names) == 5
    for n in names:
        causal = bool(z[f"{n}/causal"])
        q, k, v, do = (z[f"{n}/{x}"] for x in ("q", "k", "v", "do"))
        o, lse = orc.attention_fwd(q, k, v, causal)
        np.testing.assert_allclose(o, z[f"{n}/o"], atol=2e-6, err_msg=n)
        np.testing.assert_allclose(lse, z[f"{n}/lse"], atol=4e-6, err_msg=n)
        dq, dk, dv = orc.attention_bwd(q, k, v, o, do, lse, causal)
        for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
            np.testing.assert_allclose(got, z[f"{n}/{name}"], atol=4e-6, err_msg=f"{n}/{name}")


def test_rowops_golden_vectors():
    z = np.load(GOLDEN / "rowops_golden.npz")
    np.testing.assert_allclose(orc.softmax_fwd(z["softmax/x"]), z["softmax/p"], atol=1e-12)
    np.testing.assert_allclose(orc.softmax_bwd(z["softmax/p"], z["softmax/dp"]), z["softmax/dx"],
                               atol=1e-12)
    np.testing.assert_allclose(orc.gelu_fwd(z["gelu/x"]), z["gelu/y"], atol=1e-12)
    np.testing.assert_allclose(orc.gelu_bwd(z["gelu/x"], z["gelu/dy"]), z["gelu/dx"], atol=1e-12)
    y, _, _ = orc.layernorm_fwd(z["ln/x"], z["ln/gamma"], z["ln/beta"])
    np.testing.assert_allclose(y, z["ln/y"], atol=1e-12)
    dx, dg, db = orc.layernorm_bwd(z["ln/x"], z["ln/gamma"], z["ln/dy"])
    np.testing.assert_allclose(dx, z["ln/dx"], atol=1e-11)
    np.testing.assert_allclose(dg, z["ln/dgamma"], atol=1e-11)
    np.testing.assert_allclose(db, z["ln/dbeta"], atol=1e-11)
    np.testing.assert_allclose(orc.linear_fwd(z["linear/x"], z["linear/w"], z["linear/b"]),
                               z["linear/y"], atol=1e-12)
    np.testing.assert_allclose(orc.bias_grad(z["linear/dy"]), z["linear/db"], atol=1e-12)


def test_flop_convention():
    # 962.07 GFLOP for fwd+bwd, causal
    assert math.isclose(orc.fa2_flops(4, 32, 4096, 64, True), 962.072674304e9, rel_tol=1e-12)
    assert math.isclose(orc.fa2_flops(4, 32, 1024, 64, False), 120.259084288e9, rel_tol=1e-12)


def test_gelu_is_erf_form():
    x = np.linspace(-4, 4, 41)
    ref = F.gelu(torch.tensor(x), approximate="none").numpy()
    np.testing.assert_allclose(orc.gelu_fwd(x), ref, atol=1e-12)


@pytest.mark.parametrize("causal", [True, False])
def test_chunked_oracle_matches_closed_form(causal):
    """The row-chunked evaluation used for long-sequence GPU parity equals the
    closed form (chunks smaller than T, ragged last chunk)."""
    q, k, v, do = (t.numpy() for t in _inputs(2, 2, 300, 32, seed=91))
    o, lse = orc.attention_fwd(q, k, v, causal)
    grads = orc.attention_bwd(q, k, v, o, do, lse, causal)
    got = orc.attention_fwd_bwd_chunked(q, k, v, do, causal, chunk=128)
    for a, b in zip(got, (o, lse, *grads)):
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-11)
