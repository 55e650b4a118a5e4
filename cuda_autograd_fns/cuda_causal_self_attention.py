"""Materialised causal attention autograd function (reference:
cuda_autograd_fns/cuda_causal_self_attention.py).  Off the hot path.  The
backward follows the math of test/test_causal_self_attn.py:60-67: the operator
returns dq and dk multiplied by sqrt(hs), so both are divided by sqrt(hs) here
(the reference divides dk and dv)."""
import torch
from cuda_transformer.ops import causal_self_attention_fwd, causal_self_attention_bwd


class CudaCausalSelfAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, nh, causal):
        out, probs = causal_self_attention_fwd(qkv, nh, causal)
        ctx.save_for_backward(qkv, probs)
        ctx.nh = nh
        return out

    @staticmethod
    def backward(ctx, grad_output):
        qkv, probs = ctx.saved_tensors
        nh = ctx.nh
        q, k, v = qkv.chunk(3, dim=-1)
        B, T, C = q.shape
        hs = C // nh
        scale = hs ** 0.5

        def heads(t):
            return t.reshape(B, T, nh, hs).transpose(1, 2).reshape(B * nh, T, hs)

        dO = heads(grad_output.contiguous())
        dq, dk, dv = causal_self_attention_bwd(heads(q), heads(k), heads(v),
                                               probs.reshape(B * nh, T, T), dO)

        def merge(t):
            return t.reshape(B, nh, T, hs).transpose(1, 2).reshape(B, T, C)

        return torch.concat([merge(dq) / scale, merge(dk) / scale, merge(dv)], dim=-1), None, None
