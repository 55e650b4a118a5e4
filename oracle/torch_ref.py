"""The reference test-suite's own math path in PyTorch (test infrastructure).

``sdpa_reference`` restates test/test_flash_attention.py:10-49: O from
F.scaled_dot_product_attention with scale 1/sqrt(hs), L from logsumexp of the
masked scaled logits, and dQ/dK/dV from autograd.  Run on the CPU (any dtype)
it pins the NumPy oracle; ``cpu_flash_fwd_bwd`` is the same computation through
torch's fused CPU attention kernel (which returns the log-sum-exp directly) and
is what the benchmark times as the reference's FP32 math on the host cores.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def logsumexp_reference(q, k, causal: bool):
    """test/test_flash_attention.py:10-21."""
    sm_scale = k.shape[-1] ** (-0.5)
    s = (q @ k.transpose(-2, -1)) * sm_scale
    if causal:
        T = q.size(-2)
        mask = torch.tril(torch.ones(T, T, device=q.device, dtype=torch.bool))
        s = s.masked_fill(~mask, float("-inf"))
    return torch.logsumexp(s, dim=-1)


def sdpa_reference(q, k, v, do, causal: bool):
    """O, L, dQ, dK, dV exactly as the reference test computes its expectation
    (test/test_flash_attention.py:23-49)."""
    q = q.detach().clone().requires_grad_(True)
    k = k.detach().clone().requires_grad_(True)
    v = v.detach().clone().requires_grad_(True)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=k.shape[-1] ** (-0.5))
    lse = logsumexp_reference(q.detach(), k.detach(), causal)
    o.backward(do)
    return o.detach(), lse, q.grad, k.grad, v.grad


def cpu_flash_fwd_bwd(q, k, v, do, causal: bool):
    """Forward (with log-sum-exp) and backward on the host through torch's
    fused CPU attention kernel; q, k, v must require grad."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    out = torch.ops.aten._scaled_dot_product_flash_attention_for_cpu(
        q, k, v, 0.0, causal, attn_mask=None, scale=scale)
    o, lse = out[0], out[1]
    o.backward(do)
    return o, lse
