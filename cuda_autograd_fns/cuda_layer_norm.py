"""LayerNorm autograd function over the CUDA LayerNorm kernels.

The reference computes LayerNorm with torch operations in gpt/gpt.py:47-59
((x - mean) / sqrt(var_biased + eps) * alpha + beta); this function gives the
same result from one forward and one backward kernel."""
import torch
from cuda_transformer.ops import layernorm_fwd, layernorm_bwd


class CudaLayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, beta, eps=1e-5):
        xc = x.contiguous()
        y, mean, rstd = layernorm_fwd(xc, gamma.contiguous(), beta.contiguous(), float(eps))
        ctx.save_for_backward(xc, gamma, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, grad_output):
        x, gamma, mean, rstd = ctx.saved_tensors
        dx, dg, db = layernorm_bwd(x, gamma.contiguous(), mean, rstd, grad_output.contiguous())
        return dx, dg, db, None
