"""GPU parity of the linear layer's fused neighbours and of the fused
lm_head + cross entropy, against FP64 torch:

* GELU epilogue (fc1 + activation, gpt/gpt.py:134-135): out = x W + b and
  act = gelu(out) from one GEMM;
* GELU-gradient epilogue: (dy W^T) * gelu'(h);
* the bias gradient formed inside the weight-gradient GEMM (db = colsum(dy)
  with dW = x^T dy), split-K and accumulate included
  (cuda_autograd_fns/cuda_linear_layer.py:25-27, warp_sum_kernel.cuh:13-51);
* the cross-entropy row kernel (loss and softmax - onehot in place);
* CudaMLP and CudaLinearCrossEntropy end to end.
Tensor-core paths (3xTF32 1e-4, TF32 2e-3) and the CUDA-core fallback (FP32
mode, unaligned shapes) are covered."""
import pytest
import torch
import torch.nn.functional as F

from cuda_transformer import ops

from . import ct_helpers as H

TOL = {0: 1e-4, 1: 2e-3, 2: 1e-5}


def _r(shape, seed, dev, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("prec", [0, 1, 2])
@pytest.mark.parametrize("m,k,n", [(300, 384, 1536), (256, 1536, 384), (130, 64, 65),
                                   (70, 65, 120)])
def test_gelu_epilogue(cuda_device, prec, m, k, n):
    x = _r((2, m, k), 1, cuda_device)
    w = _r((k, n), 2, cuda_device, 0.05)
    b = _r((n,), 3, cuda_device, 0.1)
    out, act, cs = ops.linear_fused(x, w, b, prec, ops.EPILOGUE_GELU, None, False)
    ref = x.double() @ w.double() + b.double()
    assert cs.numel() == 0
    assert H.rel_err(out, ref) < TOL[prec]
    assert H.rel_err(act, F.gelu(ref)) < TOL[prec]
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("prec", [0, 1, 2])
@pytest.mark.parametrize("m,k,n", [(300, 384, 1536), (130, 1536, 68), (70, 65, 120)])
def test_gelu_grad_epilogue(cuda_device, prec, m, k, n):
    dy = _r((1, m, k), 4, cuda_device)
    wt = _r((k, n), 5, cuda_device, 0.05)
    h = _r((1, m, n), 6, cuda_device)
    zero = torch.zeros(n, device=cuda_device)
    out, _, _ = ops.linear_fused(dy, wt, zero, prec, ops.EPILOGUE_GELU_GRAD, h, False)
    hd = h.double().requires_grad_()
    F.gelu(hd).backward(torch.ones_like(hd))
    ref = (dy.double() @ wt.double()) * hd.grad
    assert H.rel_err(out, ref) < TOL[prec]
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("prec", [0, 1, 2])
@pytest.mark.parametrize("rows,k,n", [(16384, 384, 1536), (16384, 1536, 384), (1000, 384, 1536),
                                      (257, 64, 65), (512, 70, 120)])
def test_weight_grad_with_fused_bias_grad(cuda_device, prec, rows, k, n):
    """dW = x^T dy and db = colsum(dy) from one GEMM (16384 rows: split-K
    slices add dW and db in slice order)."""
    x = _r((1, rows, k), 7, cuda_device)
    dy = _r((1, rows, n), 8, cuda_device)
    zero = torch.zeros(n, device=cuda_device)
    dw, _, db = ops.linear_fused(x.transpose(1, 2), dy, zero, prec, 0, None, True)
    assert H.rel_err(dw[0], x[0].double().t() @ dy[0].double()) < TOL[prec]
    assert H.rel_err(db, dy[0].double().sum(0)) < max(TOL[prec], 1e-5)
    # deterministic: bit-identical on a second call
    dw2, _, db2 = ops.linear_fused(x.transpose(1, 2), dy, zero, prec, 0, None, True)
    assert torch.equal(dw, dw2) and torch.equal(db, db2)
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("prec", [0, 1, 2])
def test_linear_accumulate(cuda_device, prec):
    x = _r((1, 4096, 384), 9, cuda_device)
    dy = _r((1, 4096, 1024), 10, cuda_device)
    zero = torch.zeros(1024, device=cuda_device)
    acc = _r((1, 384, 1024), 11, cuda_device)
    cs = _r((1024,), 12, cuda_device)
    acc0, cs0 = acc.clone(), cs.clone()
    ops.linear_accumulate_(acc, cs, x.transpose(1, 2), dy, zero, prec)
    assert H.rel_err(acc, acc0.double() + x[0].double().t() @ dy[0].double()) < TOL[prec]
    assert H.rel_err(cs, cs0.double() + dy[0].double().sum(0)) < max(TOL[prec], 1e-5)
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,vocab", [(300, 65), (64, 100256), (33, 4100), (5, 2048)])
def test_cross_entropy_rows(cuda_device, rows, vocab):
    logits = _r((rows, vocab), 13, cuda_device, 3.0)
    g = torch.Generator().manual_seed(14)
    t = torch.randint(0, vocab, (rows,), generator=g)
    t[1] = -100  # ignored row
    t = t.to(cuda_device)
    ld = logits.double().requires_grad_()
    ref_rows = F.cross_entropy(ld, t, reduction="none", ignore_index=-100)
    ref_rows.sum().backward()
    work = logits.clone()
    loss = ops.cross_entropy_fwd_bwd_(work, t, -100)
    assert H.rel_err(loss, ref_rows) < 1e-5
    assert H.rel_err(work, ld.grad) < 1e-5
    assert float(loss[1]) == 0.0 and bool((work[1] == 0).all())
    bad = t.clone()
    bad[0] = vocab  # out of range: that row alone is NaN
    work = logits.clone()
    loss = ops.cross_entropy_fwd_bwd_(work, bad, -100)
    assert torch.isnan(loss[0]) and torch.isnan(work[0]).all()
    assert torch.isfinite(loss[2:]).all() and torch.isfinite(work[2:]).all()
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("d", [384, 512])
def test_fused_mlp_matches_composition(cuda_device, d):
    from cuda_autograd_fns import CudaMLP

    x = _r((2, 256, d), 15, cuda_device).requires_grad_()
    w1 = _r((d, 4 * d), 16, cuda_device, 0.02).requires_grad_()
    b1 = _r((4 * d,), 17, cuda_device, 0.02).requires_grad_()
    w2 = _r((4 * d, d), 18, cuda_device, 0.02).requires_grad_()
    b2 = _r((d,), 19, cuda_device, 0.02).requires_grad_()
    dy = _r((2, 256, d), 20, cuda_device)
    y = CudaMLP.apply(x, w1, b1, w2, b2)
    y.backward(dy)
    ps = [t.detach().double().requires_grad_() for t in (x, w1, b1, w2, b2)]
    yr = F.gelu(ps[0] @ ps[1] + ps[2]) @ ps[3] + ps[4]
    yr.backward(dy.double())
    assert H.rel_err(y, yr) < 1e-4
    for got, ref in zip((x, w1, b1, w2, b2), ps):
        assert H.rel_err(got.grad, ref.grad) < 1e-4
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("vocab,chunk", [(100256, 96), (65, None), (4100, 7)])
def test_fused_linear_cross_entropy(cuda_device, vocab, chunk):
    from cuda_autograd_fns import CudaLinearCrossEntropy

    d = 512
    x = _r((2, 128, d), 21, cuda_device).requires_grad_()
    w = _r((d, vocab), 22, cuda_device, 0.02).requires_grad_()
    b = _r((vocab,), 23, cuda_device, 0.02).requires_grad_()
    g = torch.Generator().manual_seed(24)
    t = torch.randint(0, vocab, (2, 128), generator=g)
    t[0, :3] = -100
    t = t.to(cuda_device)
    loss = CudaLinearCrossEntropy.apply(x, w, b, t, -100, chunk)
    (loss * 2.5).backward()
    ps = [v.detach().double().requires_grad_() for v in (x, w, b)]
    lr = F.cross_entropy((ps[0] @ ps[1] + ps[2]).reshape(-1, vocab), t.reshape(-1), ignore_index=-100)
    (lr * 2.5).backward()
    assert abs(loss.item() - lr.item()) < 1e-5 * abs(lr.item())
    for got, ref in zip((x, w, b), ps):
        assert H.rel_err(got.grad, ref.grad) < 1e-4
    H.assert_device_clean()
