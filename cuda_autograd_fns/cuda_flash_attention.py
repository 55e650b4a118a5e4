"""FlashAttention-2 autograd function (reference: cuda_autograd_fns/cuda_flash_attention.py:4-17).

Saves q, k, v, o and the log-sum-exp, recomputes the probabilities in the
backward, and ignores the gradient flowing into the log-sum-exp output."""
import torch
from cuda_transformer.ops import flash_attention_fwd, flash_attention_bwd


class CudaFlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal):
        o, l = flash_attention_fwd(q, k, v, causal)
        ctx.save_for_backward(q, k, v, o, l)
        ctx.causal = causal
        return o, l

    @staticmethod
    def backward(ctx, grad_output, grad_l=None):
        q, k, v, o, l = ctx.saved_tensors
        dq, dk, dv = flash_attention_bwd(q, k, v, o, grad_output, l, ctx.causal)
        return dq, dk, dv, None
