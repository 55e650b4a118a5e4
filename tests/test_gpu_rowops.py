"""GPU parity of the row-wise kernels and the linear layer through the C ABI,
against the oracle on the reference tests' grids, golden vectors, and the
BASELINE config-4 shapes (compared with float64 PyTorch on the device)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import cuda_transformer_b200 as cb
from oracle import fa2 as orc

from . import ct_helpers as H
from .conftest import ROOT

ROW_GRID = [(1, 64, 32), (1, 65, 32), (2, 32, 64), (4, 128, 64), (1, 70, 120)]  # test_softmax/gelu
LIN_GRID = [(1, 32, 64, 32), (1, 32, 65, 32), (2, 64, 32, 64), (2, 128, 32, 64), (1, 512, 70, 120)]


def _r(shape, seed, dev, kind="rand"):
    g = torch.Generator().manual_seed(seed)
    t = torch.rand(*shape, generator=g) if kind == "rand" else torch.randn(*shape, generator=g)
    return t.to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("b,m,n", ROW_GRID + [(1, 3, 4096), (2, 2, 5000), (1, 2, 20000)])
def test_softmax(cuda_device, b, m, n):
    x = _r((b, m, n), n, cuda_device, "randn")
    dp = _r((b, m, n), n + 1, cuda_device)
    p = H.softmax_fwd(x)
    ref = orc.softmax_fwd(x.cpu().numpy())
    assert np.abs(p.cpu().double().numpy() - ref).max() < 1e-6
    dx = H.softmax_bwd(p, dp)
    refb = orc.softmax_bwd(p.cpu().double().numpy(), dp.cpu().numpy())
    assert np.abs(dx.cpu().double().numpy() - refb).max() < 1e-6
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("b,m,n", ROW_GRID + [(1, 7, 33)])
def test_gelu(cuda_device, b, m, n):
    x = _r((b, m, n), 3 * n, cuda_device, "randn")
    dy = _r((b, m, n), 3 * n + 1, cuda_device)
    y = H.gelu_fwd(x)
    assert np.abs(y.cpu().double().numpy() - orc.gelu_fwd(x.cpu().numpy())).max() < 1e-6
    dx = H.gelu_bwd(x, dy)
    assert np.abs(dx.cpu().double().numpy() - orc.gelu_bwd(x.cpu().numpy(), dy.cpu().numpy())).max() < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("rows,n", [(5, 384), (37, 512), (16384, 384), (3, 100), (9, 1024),
                                    (7, 1536), (5, 3001), (700, 2048), (2, 4100), (3, 8192)])
def test_layernorm(cuda_device, rows, n):
    x = _r((rows, n), n, cuda_device, "randn")
    g = 1.0 + 0.1 * _r((n,), n + 1, cuda_device, "randn")
    b = 0.1 * _r((n,), n + 2, cuda_device, "randn")
    dy = _r((rows, n), n + 3, cuda_device, "randn")
    y, mean, rstd = H.layernorm_fwd(x, g, b)
    xd = x.double().requires_grad_(True)
    gd, bd = g.double().requires_grad_(True), b.double().requires_grad_(True)
    var = torch.var(xd, dim=-1, keepdim=True, unbiased=False)
    yr = (xd - xd.mean(-1, keepdim=True)) / torch.sqrt(var + 1e-5) * gd + bd  # gpt/gpt.py:55-58
    yr.backward(dy.double())
    assert (y.double() - yr).abs().max().item() < 1e-5
    dx, dg, db = H.layernorm_bwd(x, g, mean, rstd, dy)
    assert H.rel_err(dx, xd.grad) < 1e-5
    assert H.rel_err(dg, gd.grad) < 1e-5
    assert H.rel_err(db, bd.grad) < 1e-5
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("prec", [cb.PRECISION_3XTF32, cb.PRECISION_FP32])
@pytest.mark.parametrize("B,T,fin,fout", LIN_GRID + [(1, 16384, 384, 1536), (1, 16384, 1536, 384)])
def test_linear(cuda_device, prec, B, T, fin, fout):
    x = _r((B, T, fin), fin, cuda_device)
    w = 0.02 * _r((fin, fout), fout, cuda_device, "randn")
    b = 0.02 * _r((fout,), fout + 1, cuda_device, "randn")
    dy = _r((B, T, fout), fout + 2, cuda_device)
    out = H.linear_fwd(x, w, b, prec)
    ref = x.double() @ w.double() + b.double()
    assert (out.double() - ref).abs().max().item() < 1e-4 * max(1.0, ref.abs().max().item())
    # the autograd backward's three calls (cuda_autograd_fns/cuda_linear_layer.py)
    zero_in = torch.zeros(fin, device=cuda_device)
    dx = H.linear_fwd(dy, w.unsqueeze(0).transpose(1, 2), zero_in, prec)
    assert H.rel_err(dx, dy.double() @ w.double().t()) < 1e-5
    rows = B * T
    dw = H.linear_fwd(x.reshape(1, rows, fin).transpose(1, 2), dy.reshape(1, rows, fout),
                      torch.zeros(fout, device=cuda_device), prec)[0]
    # all-positive inputs over up to 16384 rows: the tensor core's
    # round-toward-zero accumulator leaves ~1e-5 relative in 3xTF32
    assert H.rel_err(dw, x.reshape(rows, fin).double().t() @ dy.reshape(rows, fout).double()) < 2e-5
    db = H.bias_grad(dy)
    assert H.rel_err(db, dy.double().sum((0, 1))) < 1e-5
    H.assert_device_clean()


@pytest.mark.gpu
def test_bias_grad_strided(cuda_device):
    dy = _r((3, 50, 40), 5, cuda_device).transpose(1, 2)  # (3, 40, 50) non-contiguous
    assert H.rel_err(H.bias_grad(dy), dy.double().sum((0, 1))) < 1e-6


@pytest.mark.gpu
def test_rowops_golden_vectors(cuda_device):
    z = np.load(ROOT / "tests" / "golden" / "rowops_golden.npz")
    t = lambda k: torch.from_numpy(z[k]).float().to(cuda_device)  # noqa: E731
    p = H.softmax_fwd(t("softmax/x"))
    assert np.abs(p.cpu().double().numpy() - z["softmax/p"]).max() < 1e-6
    assert np.abs(H.softmax_bwd(t("softmax/p"), t("softmax/dp")).cpu().double().numpy() - z["softmax/dx"]).max() < 1e-6
    assert np.abs(H.gelu_fwd(t("gelu/x")).cpu().double().numpy() - z["gelu/y"]).max() < 1e-6
    assert np.abs(H.gelu_bwd(t("gelu/x"), t("gelu/dy")).cpu().double().numpy() - z["gelu/dx"]).max() < 1e-6
    y, mean, rstd = H.layernorm_fwd(t("ln/x"), t("ln/gamma"), t("ln/beta"))
    assert np.abs(y.cpu().double().numpy() - z["ln/y"]).max() < 1e-5
    dx, dg, db = H.layernorm_bwd(t("ln/x"), t("ln/gamma"), mean, rstd, t("ln/dy"))
    assert H.rel_err(dx, z["ln/dx"]) < 1e-5 and H.rel_err(dg, z["ln/dgamma"]) < 1e-5
    assert H.rel_err(db, z["ln/dbeta"]) < 1e-5
    out = H.linear_fwd(t("linear/x"), t("linear/w"), t("linear/b"))
    assert np.abs(out.cpu().double().numpy() - z["linear/y"]).max() < 1e-5


@pytest.mark.gpu
def test_gelu_wide_range(cuda_device):
    """Exact GELU over [-12, 12] (both tails) against the FP64 oracle: error
    within a few FP32 ulps of max(1, |value|)."""
    x = torch.linspace(-12.0, 12.0, 200001, dtype=torch.float32)
    dy = torch.ones_like(x)
    xd = x.to(cuda_device)
    y = H.gelu_fwd(xd).cpu().double().numpy()
    dx = H.gelu_bwd(xd, dy.to(cuda_device)).cpu().double().numpy()
    ry, rdx = orc.gelu_fwd(x.numpy()), orc.gelu_bwd(x.numpy(), dy.numpy())
    assert (np.abs(y - ry) / np.maximum(1.0, np.abs(ry))).max() < 5e-7
    assert (np.abs(dx - rdx) / np.maximum(1.0, np.abs(rdx))).max() < 5e-7
