"""Calls into the C ABI (libct_b200.so) on torch CUDA tensors, for the GPU
parity tests.  Every helper allocates dense outputs with torch, passes raw
pointers / strides / sizes and the current stream, and raises on a non-zero
status."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

import cuda_transformer_b200 as cb


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def fa2_fwd(q, k, v, causal, precision=cb.PRECISION_3XTF32):
    B, H, T, D = q.shape
    o = torch.empty(B, H, T, D, device=q.device, dtype=torch.float32)
    lse = torch.empty(B, H, T, device=q.device, dtype=torch.float32)
    rc = cb.lib().ct_fa2_fwd(_p(q), cb.strides(q), _p(k), cb.strides(k), _p(v), cb.strides(v),
                             _p(o), _p(lse), B, H, T, D, int(causal), precision, _stream())
    cb.check(rc, "ct_fa2_fwd")
    return o, lse


def fa2_bwd(q, k, v, o, do, lse, causal, precision=cb.PRECISION_3XTF32):
    B, H, T, D = q.shape
    dq, dk, dv = (torch.empty(B, H, T, D, device=q.device, dtype=torch.float32) for _ in range(3))
    ws_bytes = cb.lib().ct_fa2_bwd_workspace_size(B, H, T, D)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
    rc = cb.lib().ct_fa2_bwd(_p(q), cb.strides(q), _p(k), cb.strides(k), _p(v), cb.strides(v),
                             _p(o), cb.strides(o), _p(do), cb.strides(do), _p(lse),
                             cb.strides(lse), _p(dq), _p(dk), _p(dv), _p(ws), ws_bytes, B, H, T,
                             D, int(causal), precision, _stream())
    cb.check(rc, "ct_fa2_bwd")
    return dq, dk, dv


def fa2_bwd_fused(q, k, v, o, do, lse, causal, precision=cb.PRECISION_TF32):
    """ct_fa2_bwd_fused: the one-kernel backward (TF32, head dim 64)."""
    B, H, T, D = q.shape
    dq, dk, dv = (torch.empty(B, H, T, D, device=q.device, dtype=torch.float32) for _ in range(3))
    ws_bytes = cb.lib().ct_fa2_bwd_workspace_size(B, H, T, D)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
    rc = cb.lib().ct_fa2_bwd_fused(_p(q), cb.strides(q), _p(k), cb.strides(k), _p(v),
                                   cb.strides(v), _p(o), cb.strides(o), _p(do), cb.strides(do),
                                   _p(lse), cb.strides(lse), _p(dq), _p(dk), _p(dv), _p(ws),
                                   ws_bytes, B, H, T, D, int(causal), precision, _stream())
    cb.check(rc, "ct_fa2_bwd_fused")
    return dq, dk, dv


def fa2_bwd_split(q, k, v, o, do, lse, causal, precision=cb.PRECISION_3XTF32):
    """The backward through its per-kernel entry points (delta, then the
    query-stationary dQ kernel and the key/value-stationary dK/dV kernel),
    never the one-kernel path ct_fa2_bwd may take."""
    B, H, T, D = q.shape
    dq, dk, dv = (torch.empty(B, H, T, D, device=q.device, dtype=torch.float32) for _ in range(3))
    delta = fa2_delta(o, do)
    cb.check(cb.lib().ct_fa2_bwd_dq(_p(q), cb.strides(q), _p(k), cb.strides(k), _p(v),
                                    cb.strides(v), _p(do), cb.strides(do), _p(lse),
                                    cb.strides(lse), _p(delta), _p(dq), B, H, T, D, int(causal),
                                    precision, _stream()), "ct_fa2_bwd_dq")
    cb.check(cb.lib().ct_fa2_bwd_dkdv(_p(q), cb.strides(q), _p(k), cb.strides(k), _p(v),
                                      cb.strides(v), _p(do), cb.strides(do), _p(lse),
                                      cb.strides(lse), _p(delta), _p(dk), _p(dv), B, H, T, D,
                                      int(causal), precision, _stream()), "ct_fa2_bwd_dkdv")
    return dq, dk, dv


def fa2_delta(o, do):
    B, H, T, D = o.shape
    delta = torch.empty(B, H, T, device=o.device, dtype=torch.float32)
    cb.check(cb.lib().ct_fa2_bwd_delta(_p(o), cb.strides(o), _p(do), cb.strides(do), _p(delta),
                                       B, H, T, D, _stream()), "ct_fa2_bwd_delta")
    return delta


def linear_fwd(x, w, b, precision=cb.PRECISION_3XTF32, workspace=False):
    """ct_linear_fwd, or ct_linear_fwd_ws with a workspace (split-K allowed)."""
    w3 = w if w.dim() == 3 else w.unsqueeze(0)
    batch, m, k = x.shape
    n = w3.shape[2]
    out = torch.empty(batch, m, n, device=x.device, dtype=torch.float32)
    if workspace:
        wsb = cb.lib().ct_linear_workspace_size(batch, m, k, n)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=x.device)
        rc = cb.lib().ct_linear_fwd_ws(_p(x), cb.strides(x), _p(w3), cb.strides(w3), _p(b),
                                       b.stride(0), _p(out), batch, m, k, n, w3.shape[0],
                                       precision, _p(ws), wsb, _stream())
    else:
        rc = cb.lib().ct_linear_fwd(_p(x), cb.strides(x), _p(w3), cb.strides(w3), _p(b),
                                    b.stride(0), _p(out), batch, m, k, n, w3.shape[0], precision,
                                    _stream())
    cb.check(rc, "ct_linear_fwd")
    return out


def bias_grad(dy):
    batch, m, n = dy.shape
    db = torch.empty(n, device=dy.device, dtype=torch.float32)
    wsb = cb.lib().ct_bias_grad_workspace_size(batch, m, n)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dy.device)
    cb.check(cb.lib().ct_bias_grad(_p(dy), cb.strides(dy), _p(db), batch, m, n, _p(ws), wsb,
                                   _stream()), "ct_bias_grad")
    return db


def softmax_fwd(x):
    y = torch.empty_like(x)
    cb.check(cb.lib().ct_softmax_fwd(_p(x), _p(y), x.numel() // x.shape[-1], x.shape[-1],
                                     _stream()), "ct_softmax_fwd")
    return y


def softmax_bwd(p, dp):
    dx = torch.empty_like(p)
    cb.check(cb.lib().ct_softmax_bwd(_p(p), _p(dp), _p(dx), p.numel() // p.shape[-1],
                                     p.shape[-1], _stream()), "ct_softmax_bwd")
    return dx


def gelu_fwd(x):
    y = torch.empty_like(x)
    cb.check(cb.lib().ct_gelu_fwd(_p(x), _p(y), x.numel(), _stream()), "ct_gelu_fwd")
    return y


def gelu_bwd(x, dy):
    dx = torch.empty_like(x)
    cb.check(cb.lib().ct_gelu_bwd(_p(x), _p(dy), _p(dx), x.numel(), _stream()), "ct_gelu_bwd")
    return dx


def layernorm_fwd(x, g, b, eps=1e-5):
    n = x.shape[-1]
    rows = x.numel() // n
    y = torch.empty_like(x)
    mean = torch.empty(rows, device=x.device)
    rstd = torch.empty(rows, device=x.device)
    cb.check(cb.lib().ct_layernorm_fwd(_p(x), _p(g), _p(b), _p(y), _p(mean), _p(rstd), rows, n,
                                       ctypes.c_float(eps), _stream()), "ct_layernorm_fwd")
    return y, mean, rstd


def layernorm_bwd(x, g, mean, rstd, dy):
    n = x.shape[-1]
    rows = x.numel() // n
    dx = torch.empty_like(x)
    dg = torch.empty(n, device=x.device)
    db = torch.empty(n, device=x.device)
    wsb = cb.lib().ct_layernorm_bwd_workspace_size(rows, n)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=x.device)
    cb.check(cb.lib().ct_layernorm_bwd(_p(x), _p(g), _p(mean), _p(rstd), _p(dy), _p(dx), _p(dg),
                                       _p(db), rows, n, _p(ws), wsb, _stream()),
             "ct_layernorm_bwd")
    return dx, dg, db


def diag_umma(mode, a, b, n):
    """One TF32 tensor-core product through the test-only diagnostics library."""
    from tests import diag

    d = torch.empty(128, n, device=a.device, dtype=torch.float32)
    diag.check(diag.lib().ct_diag_umma_tf32(mode, _p(a), _p(b), _p(d), n, _stream()),
               "ct_diag_umma")
    torch.cuda.synchronize()
    assert diag.status() == 0, "diagnostic kernel's bounded wait ran out"
    return d


def rel_err(x, ref) -> float:
    """max |x - ref| / max |ref| (the north-star tolerance metric)."""
    x = x.detach().double().cpu() if torch.is_tensor(x) else torch.as_tensor(np.asarray(x, np.float64))
    ref = ref.detach().double().cpu() if torch.is_tensor(ref) else torch.as_tensor(np.asarray(ref, np.float64))
    denom = ref.abs().max().item()
    return (x - ref).abs().max().item() / (denom if denom > 0 else 1.0)


def assert_device_clean(device_index: int = 0) -> None:
    """No device-side bounded wait has expired (and clear the word)."""
    torch.cuda.synchronize()
    v = cb.device_status(device_index, clear=True)
    assert v == 0, f"device watchdog raised: {v:#x}"
