"""The drop-in PyTorch surface on the GPU: the reference test-suite's cases
(grids, input distributions and tolerances of test/test_flash_attention.py,
test/test_linear.py, test/test_softmax.py, test/test_gelu.py and
test/test_causal_self_attn.py) rewritten against ``cuda_transformer.ops``
with fixed seeds, plus an end-to-end decoder block through the autograd
functions as gpt/gpt.py uses them."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ct_helpers as H


@pytest.fixture(scope="module")
def ops():
    from cuda_transformer import ops as o
    return o


FA_GRID = [(1, 1, 64, 128, False), (1, 1, 64, 128, True), (1, 1, 65, 64, True),
           (2, 4, 128, 32, False), (2, 4, 128, 64, True), (2, 4, 257, 64, True),
           (1, 2, 512, 128, True)]


@pytest.mark.gpu
@pytest.mark.parametrize("B,nh,T,hs,causal", FA_GRID)
def test_flash_attention_reference_case(cuda_device, ops, B, nh, T, hs, causal):
    torch.manual_seed(T * 131 + hs)
    q = torch.randn(B, nh, T, hs, device=cuda_device, requires_grad=True)
    k = torch.randn(B, nh, T, hs, device=cuda_device, requires_grad=True)
    v = torch.randn(B, nh, T, hs, device=cuda_device, requires_grad=True)
    out = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=hs ** -0.5)
    s = (q @ k.transpose(-2, -1)) * hs ** -0.5
    if causal:
        s = s.masked_fill(torch.tril(torch.ones(T, T, device=cuda_device)) == 0, float("-inf"))
    L = torch.logsumexp(s, dim=-1)
    o, l = ops.flash_attention_fwd(q.detach(), k.detach(), v.detach(), causal)
    assert torch.allclose(o, out, atol=1e-5)
    assert torch.allclose(L, l, atol=1e-5)
    dO = torch.rand_like(out)
    out.backward(dO)
    dq, dk, dv = ops.flash_attention_bwd(q.detach(), k.detach(), v.detach(), o, dO, L.detach(), causal)
    assert torch.allclose(dq, q.grad, atol=1e-4)
    assert torch.allclose(dk, k.grad, atol=1e-4)
    assert torch.allclose(dv, v.grad, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,fin,fout", [(1, 32, 64, 32), (1, 32, 65, 32), (2, 64, 32, 64),
                                          (2, 128, 32, 64), (1, 512, 70, 120)])
def test_linear_reference_case(cuda_device, ops, B, T, fin, fout):
    torch.manual_seed(fin * 7 + fout)
    x = torch.rand(B, T, fin, device=cuda_device, requires_grad=True)
    lin = nn.Linear(fin, fout, device=cuda_device)
    w_t = lin.weight.detach().t()
    out = ops.cuda_fma(x.detach(), w_t, lin.bias.detach())
    ref = lin(x)
    assert torch.allclose(out, ref, atol=1e-5)
    dy = torch.rand_like(ref)
    dx, dw, db = torch.autograd.grad(ref, [x, lin.weight, lin.bias], dy)
    w = w_t.unsqueeze(0).transpose(1, 2)
    dx_c = ops.cuda_fma(dy, w, torch.zeros(fin, device=cuda_device))
    dw_c = torch.sum(ops.cuda_fma(dy.transpose(1, 2), x.detach(), torch.zeros(fin, device=cuda_device)), 0)
    db_c = ops.db_calculation(dy)
    assert torch.allclose(dx, dx_c, atol=1e-5)
    assert torch.allclose(dw, dw_c, atol=1e-5)
    assert torch.allclose(db, db_c, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("b,m,n", [(1, 64, 32), (1, 65, 32), (2, 32, 64), (4, 128, 64), (1, 70, 120)])
def test_softmax_gelu_reference_cases(cuda_device, ops, b, m, n):
    torch.manual_seed(m * n)
    x = torch.rand(b, m, n, device=cuda_device, requires_grad=True)
    p = F.softmax(x, dim=-1)
    assert torch.allclose(ops.cuda_softmax(x.detach()), p, atol=1e-5)
    dp = torch.rand_like(p)
    p.backward(dp)
    assert torch.allclose(ops.cuda_softmax_bwd(p.detach(), dp), x.grad, atol=1e-5)
    x2 = torch.rand(b, m, n, device=cuda_device, requires_grad=True)
    y = F.gelu(x2)
    assert torch.allclose(ops.gelu_activation(x2.detach()), y, atol=1e-5)
    dy = torch.rand_like(x2)
    y.backward(dy)
    assert torch.allclose(ops.gelu_activation_bwd(x2.detach(), dy), x2.grad, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,nh,hs,causal", [(1, 64, 1, 32, False), (1, 65, 1, 32, True),
                                              (2, 128, 4, 64, True), (1, 512, 2, 128, True)])
def test_materialised_attention_reference_case(cuda_device, ops, B, T, nh, hs, causal):
    torch.manual_seed(T + hs)
    C = nh * hs
    qkv = torch.rand(B, T, 3 * C, device=cuda_device, requires_grad=True)
    q, k, v = (t.reshape(B, T, nh, hs).transpose(1, 2) for t in (qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]))
    s = (q @ k.transpose(-2, -1)) * hs ** -0.5
    if causal:
        s = s.masked_fill(torch.tril(torch.ones(T, T, device=cuda_device)) == 0, float("-inf"))
    probs = F.softmax(s, dim=-1)
    ref = (probs @ v).transpose(1, 2).reshape(B, T, C)
    out, cprobs = ops.causal_self_attention_fwd(qkv.detach(), nh, causal)
    assert torch.allclose(out, ref, atol=1e-5)
    dO = torch.rand_like(ref)
    ref.backward(dO)
    dq, dk, dv = (g.reshape(B, T, nh, hs).transpose(1, 2).reshape(B * nh, T, hs) for g in qkv.grad.chunk(3, -1))
    heads = lambda t: t.reshape(B, T, nh, hs).transpose(1, 2).reshape(B * nh, T, hs)  # noqa: E731
    qc, kc, vc = (heads(t) for t in qkv.detach().chunk(3, -1))
    dqc, dkc, dvc = ops.causal_self_attention_bwd(qc, kc, vc, cprobs.reshape(B * nh, T, T), heads(dO))
    assert torch.allclose(dqc / hs ** 0.5, dq, atol=1e-4)
    assert torch.allclose(dkc / hs ** 0.5, dk, atol=1e-4)
    assert torch.allclose(dvc, dv, atol=1e-4)


@pytest.mark.gpu
def test_decoder_block_matches_torch(cuda_device):
    """One pre-LN decoder block (gpt/gpt.py:122-152 structure, flash attention)
    through the autograd functions vs. the same block in float64 torch."""
    from cuda_autograd_fns import (CudaFlashAttention, CudaGeluLayer, CudaLayerNorm,
                                   CudaLinearLayer)
    torch.manual_seed(5)
    B, T, C, nh = 2, 256, 384, 6
    hs = C // nh
    shapes = dict(wqkv=(C, 3 * C), bqkv=(3 * C,), wo=(C, C), bo=(C,), w1=(C, 4 * C),
                  b1=(4 * C,), w2=(4 * C, C), b2=(C,))
    p = {n: (0.02 * torch.randn(*s, device=cuda_device)).requires_grad_(True)
         for n, s in shapes.items()}
    p["g"] = torch.ones(C, device=cuda_device, requires_grad=True)
    p["beta"] = torch.zeros(C, device=cuda_device, requires_grad=True)
    x = torch.randn(B, T, C, device=cuda_device, requires_grad=True)

    def block(x, p, lin, ln, attn, gelu):
        h = ln(x, p["g"], p["beta"])
        qkv = lin(h, p["wqkv"], p["bqkv"])
        q, k, v = (t.reshape(B, T, nh, hs).transpose(1, 2) for t in qkv.chunk(3, dim=-1))
        a = attn(q, k, v).transpose(1, 2).reshape(B, T, C)
        x = x + lin(a, p["wo"], p["bo"])
        h = ln(x, p["g"], p["beta"])
        return x + lin(gelu(lin(h, p["w1"], p["b1"])), p["w2"], p["b2"])

    def ln_ref(t, g, b):
        var = torch.var(t, dim=-1, keepdim=True, unbiased=False)
        return (t - t.mean(-1, keepdim=True)) / torch.sqrt(var + 1e-5) * g + b

    y = block(x, p, CudaLinearLayer.apply, lambda t, g, b: CudaLayerNorm.apply(t, g, b, 1e-5),
              lambda q, k, v: CudaFlashAttention.apply(q, k, v, True)[0], CudaGeluLayer.apply)
    dy = torch.randn_like(y)
    grads = torch.autograd.grad(y, [x, *p.values()], dy)

    pr = {n: t.detach().double().requires_grad_(True) for n, t in p.items()}
    xr = x.detach().double().requires_grad_(True)
    yr = block(xr, pr, lambda t, w, b: t @ w + b, ln_ref,
               lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True), F.gelu)
    gref = torch.autograd.grad(yr, [xr, *pr.values()], dy.double())
    assert H.rel_err(y, yr) < 1e-4
    for name, got, ref in zip(["x", *p.keys()], grads, gref):
        assert H.rel_err(got, ref) < 1e-4, name
