"""The transformer MLP (gpt/gpt.py:134-136: fc1 -> GELU -> fc2) as one
autograd function whose GELU runs in the linear layers' epilogues.

Forward: fc1's GEMM writes both its pre-activation h = x W1 + b1 and
a = gelu(h) (no separate activation pass over h); y = a W2 + b2.
Backward: fc2's input-gradient GEMM multiplies by gelu'(h) in its epilogue,
giving dh = (dy W2^T) * gelu'(h) directly (no separate activation-gradient
pass); dW2, db2 and dW1, db1 each come from one GEMM (db formed from the dy
tiles that GEMM stages); dx = dh W1^T.  Same results as CudaLinearLayer,
CudaGeluLayer, CudaLinearLayer applied in sequence (the reference's
composition).

FUSE_FORWARD / FUSE_BACKWARD choose per direction between the epilogue and a
separate element-wise GELU kernel.  What pays depends on the shapes: the
epilogue adds its activation work (erf, and exp in the backward) to the GEMM's
four epilogue warps, the separate kernel adds one pass over h.  Measured on a
B200 for [16384 x 384] x [384 x 1536] (the benchmark GPT's fc1): forward
153.7 us fused vs 155.6 us separate in 3xTF32 and 108.6 vs 94.8 us in TF32;
backward 202 vs 167 us (3xTF32) and 156 vs 109 us (TF32) -- so both default to
the separate kernel, and the fused epilogues stay available."""
import torch
from cuda_transformer.ops import (EPILOGUE_GELU, EPILOGUE_GELU_GRAD, cuda_fma, gelu_activation,
                                  gelu_activation_bwd, linear_fused)

from .cuda_linear_layer import _precision, _zeros, weight_and_bias_grad


FUSE_FORWARD = False
FUSE_BACKWARD = False


class CudaMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2):
        if FUSE_FORWARD:
            h, a, _ = linear_fused(x, w1, b1, _precision(), EPILOGUE_GELU, None, False)
        else:
            h = cuda_fma(x, w1, b1)
            a = gelu_activation(h)
        y = cuda_fma(a, w2, b2)
        ctx.save_for_backward(x, w1, w2, h, a)
        return y

    @staticmethod
    def backward(ctx, grad_output):
        x, w1, w2, h, a = ctx.saved_tensors
        dy = grad_output.contiguous()
        if FUSE_BACKWARD:
            dh, _, _ = linear_fused(dy, w2.t().unsqueeze(0), _zeros(w2.shape[0], dy.device),
                                    _precision(), EPILOGUE_GELU_GRAD, h, False)
        else:
            dh = gelu_activation_bwd(h, cuda_fma(dy, w2.t().unsqueeze(0),
                                                  _zeros(w2.shape[0], dy.device)))
        dw2, db2 = weight_and_bias_grad(a, dy)
        dw1, db1 = weight_and_bias_grad(x, dh)
        dx = cuda_fma(dh, w1.t().unsqueeze(0), _zeros(x.shape[-1], x.device))
        return dx, dw1, db1, dw2, db2
