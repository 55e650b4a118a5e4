"""NumPy FP64 restatement of the reference's hot-path math (test infrastructure).

Every function cites the reference lines it restates
(AnshSachinkumarArora/CUDA_Transformer).  Tensors are NumPy arrays; attention
tensors are [B, H, T, D].
"""
from __future__ import annotations

import math

import numpy as np


def _mask(T: int, causal: bool) -> np.ndarray:
    """Keep-mask of the score tile: (!causal || q >= k) && q < T && k < T
    (Transformer_kernels/flash_attention.cuh:117, :318, :452)."""
    keep = np.ones((T, T), dtype=bool)
    if causal:
        keep = np.tril(keep)
    return keep


def attention_fwd(q, k, v, causal: bool):
    """O and L of flash_attention_fwd_kernel (flash_attention.cuh:27-170) in
    closed form: S = Q K^T / sqrt(D) (:115-116, the launcher passes
    sm_scale = sqrt(hs) and the kernel inverts it, :45), masked to -inf (:117),
    P = softmax(S), O = P V, L = rowmax + ln(rowsum) (:167)."""
    q, k, v = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    D = q.shape[-1]
    s = np.einsum("bhqd,bhkd->bhqk", q, k) / math.sqrt(D)
    s = np.where(_mask(q.shape[2], causal), s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhqk,bhkd->bhqd", p / l, v)
    lse = (m + np.log(l))[..., 0]
    return o, lse


def attention_fwd_tiled(q, k, v, causal: bool, br: int = 16, bc: int = 16):
    """The same forward in the reference kernel's loop order
    (flash_attention.cuh:86-167): per br-row block, stream bc-column K/V
    blocks up to qEnd (:84), keep running m and l, rescale O by
    alpha = exp(m_old - m_new) (:126, :150) and finish with O / l, m + ln l."""
    q, k, v = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    B, H, T, D = q.shape
    scale = 1.0 / math.sqrt(D)
    o = np.zeros((B, H, T, D))
    lse = np.zeros((B, H, T))
    for r0 in range(0, T, br):
        rows = np.arange(r0, min(r0 + br, T))
        q_end = min(r0 + br, T) if causal else T
        m = np.full((B, H, len(rows), 1), -np.inf)
        l = np.zeros((B, H, len(rows), 1))
        acc = np.zeros((B, H, len(rows), D))
        for c0 in range(0, q_end, bc):
            cols = np.arange(c0, min(c0 + bc, T))
            s = np.einsum("bhqd,bhkd->bhqk", q[:, :, rows], k[:, :, cols]) * scale
            keep = (rows[:, None] >= cols[None, :]) if causal else np.ones((len(rows), len(cols)), bool)
            s = np.where(keep, s, -np.inf)
            m_new = np.maximum(m, s.max(axis=-1, keepdims=True))
            alpha = np.exp(m - m_new)
            p = np.exp(s - m_new)
            l = alpha * l + p.sum(axis=-1, keepdims=True)
            acc = acc * alpha + np.einsum("bhqk,bhkd->bhqd", p, v[:, :, cols])
            m = m_new
        o[:, :, rows] = acc / l
        lse[:, :, rows] = (m + np.log(l))[..., 0]
    return o, lse


def attention_bwd_delta(o, do):
    """delta = rowsum(O * dO) (flash_attention_bwd_delta, flash_attention.cuh:175-213)."""
    return np.einsum("bhtd,bhtd->bht", np.asarray(o, np.float64), np.asarray(do, np.float64))


def attention_bwd(q, k, v, o, do, lse, causal: bool):
    """dQ, dK, dV of flash_attention_bwd_dq / _dk_dv (flash_attention.cuh:216-504):
    P = exp(S - L) with S scaled by 1/sqrt(D) and masked (:318-323, :452-457);
    dP = dO V^T (:312-318); dS = P * (dP - delta) (:326, :476);
    dQ = dS K / sqrt(D) (:337); dV = P^T dO (:462); dK = dS^T Q / sqrt(D) (:486)."""
    q, k, v, o, do, lse = (np.asarray(t, dtype=np.float64) for t in (q, k, v, o, do, lse))
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    keep = _mask(q.shape[2], causal)
    p = np.where(keep, np.exp(np.where(keep, s, 0.0) - lse[..., None]), 0.0)
    dp = np.einsum("bhqd,bhkd->bhqk", do, v)
    delta = attention_bwd_delta(o, do)
    ds = p * (dp - delta[..., None])
    dq = np.einsum("bhqk,bhkd->bhqd", ds, k) * scale
    dk = np.einsum("bhqk,bhqd->bhkd", ds, q) * scale
    dv = np.einsum("bhqk,bhqd->bhkd", p, do)
    return dq, dk, dv


def attention_fwd_bwd_chunked(q, k, v, do, causal: bool, chunk: int = 1024):
    """The closed forms of attention_fwd and attention_bwd (same reference
    lines) evaluated for one (b,h) pair at a time over `chunk` query rows at a
    time, so host memory stays O(chunk * T) at long sequence lengths: per chunk
    S = Q_c K^T / sqrt(D) (masked), L = rowmax + ln(rowsum), O_c = P V,
    delta_c = rowsum(O_c * dO_c), dS = P * (dO_c V^T - delta_c),
    dQ_c = dS K / sqrt(D); dK += dS^T Q_c / sqrt(D), dV += P^T dO_c.
    Returns O, LSE, dQ, dK, dV in float64."""
    q, k, v, do = (np.asarray(t, dtype=np.float64) for t in (q, k, v, do))
    B, H, T, D = q.shape
    scale = 1.0 / math.sqrt(D)
    o = np.empty_like(q)
    lse = np.empty((B, H, T))
    dq, dk, dv = np.empty_like(q), np.zeros_like(q), np.zeros_like(q)
    cols = np.arange(T)
    for b in range(B):
        for h in range(H):
            kk, vv = k[b, h], v[b, h]
            for r0 in range(0, T, chunk):
                r1 = min(r0 + chunk, T)
                qc, dc = q[b, h, r0:r1], do[b, h, r0:r1]
                s = (qc @ kk.T) * scale
                if causal:
                    s = np.where(cols[None, :] <= np.arange(r0, r1)[:, None], s, -np.inf)
                m = s.max(axis=1, keepdims=True)
                e = np.exp(s - m)
                l = e.sum(axis=1, keepdims=True)
                p = e / l
                oc = p @ vv
                o[b, h, r0:r1] = oc
                lse[b, h, r0:r1] = (m + np.log(l))[:, 0]
                delta = (oc * dc).sum(axis=1, keepdims=True)
                ds = p * (dc @ vv.T - delta)
                dq[b, h, r0:r1] = (ds @ kk) * scale
                dk[b, h] += (ds.T @ qc) * scale
                dv[b, h] += p.T @ dc
    return o, lse, dq, dk, dv


# ------------------------------------------------------------- row kernels
def softmax_fwd(x):
    """naive_softmax (Transformer_kernels/softmax.cuh:25-106): exp(x - max) / sum."""
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def softmax_bwd(p, dp):
    """naive_softmax_bwd (softmax.cuh:108-159): p * (dp - sum(p * dp))."""
    p, dp = np.asarray(p, np.float64), np.asarray(dp, np.float64)
    return p * (dp - (p * dp).sum(axis=-1, keepdims=True))


def _phi(x):
    return np.exp(-0.5 * x * x) / math.sqrt(2.0 * math.pi)


def _Phi(x):
    from math import erf
    return 0.5 * (1.0 + np.vectorize(erf)(x / math.sqrt(2.0)))


def gelu_fwd(x):
    """gelu (Transformer_kernels/GeLU.cuh:7-16): x * Phi(x) (erf form)."""
    x = np.asarray(x, np.float64)
    return x * _Phi(x)


def gelu_bwd(x, dy):
    """gelu_bwd (GeLU.cuh:19-29): dy * (Phi(x) + x * phi(x))."""
    x, dy = np.asarray(x, np.float64), np.asarray(dy, np.float64)
    return dy * (_Phi(x) + x * _phi(x))


def layernorm_fwd(x, gamma, beta, eps=1e-5):
    """gpt/gpt.py:55-58: (x - mean) / sqrt(var_biased + eps) * alpha + beta."""
    x = np.asarray(x, np.float64)
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(var + eps)
    return (x - mean) * rstd * gamma + beta, mean[..., 0], rstd[..., 0]


def layernorm_bwd(x, gamma, dy, eps=1e-5):
    """Gradients of gpt/gpt.py:55-58 w.r.t. x, alpha and beta."""
    x, gamma, dy = (np.asarray(t, np.float64) for t in (x, gamma, dy))
    mean = x.mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(((x - mean) ** 2).mean(axis=-1, keepdims=True) + eps)
    xhat = (x - mean) * rstd
    g = dy * gamma
    dx = rstd * (g - g.mean(axis=-1, keepdims=True) - xhat * (g * xhat).mean(axis=-1, keepdims=True))
    red = tuple(range(x.ndim - 1))
    return dx, (dy * xhat).sum(axis=red), dy.sum(axis=red)


def linear_fwd(x, w, b):
    """fused_multiply_add (Transformer_kernels/fused_multiply_add.cuh:10-93):
    out[b] = x[b] @ W[b or 0] + bias."""
    x, w, b = (np.asarray(t, np.float64) for t in (x, w, b))
    if w.ndim == 2:
        w = w[None]
    return np.matmul(x, w) + b


def bias_grad(dy):
    """warp_sum_kernel (Transformer_kernels/warp_sum_kernel.cuh:13-51): column sums."""
    dy = np.asarray(dy, np.float64)
    return dy.reshape(-1, dy.shape[-1]).sum(axis=0)


def fa2_flops(B: int, H: int, N: int, D: int, causal: bool, mode: str = "fwd+bwd") -> float:
    """FLOP convention of benchmark/cuda_bench.py:63-69: fwd = 4 B H N^2 D,
    halved when causal; bwd = 2.5 x fwd."""
    fwd = 4.0 * B * H * N * N * D * (0.5 if causal else 1.0)
    return {"fwd": fwd, "bwd": 2.5 * fwd, "fwd+bwd": 3.5 * fwd}[mode]
