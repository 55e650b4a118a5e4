"""The transformer MLP (gpt/gpt.py:134-136: fc1 -> GELU -> fc2) as one
autograd function whose GELU runs in the linear layers' epilogues.

Forward: fc1's GEMM writes both its pre-activation h = x W1 + b1 and
a = gelu(h) (no separate activation pass over h); y = a W2 + b2.
Backward: fc2's input-gradient GEMM multiplies by gelu'(h) in its epilogue,
giving dh = (dy W2^T) * gelu'(h) directly (no separate activation-gradient
pass); dW2, db2 and dW1, db1 each come from one GEMM (db formed from the dy
tiles that GEMM stages); dx = dh W1^T.  Same results as CudaLinearLayer,
CudaGeluLayer, CudaLinearLayer applied in sequence (the reference's
composition)."""
import torch
from cuda_transformer.ops import EPILOGUE_GELU, EPILOGUE_GELU_GRAD, cuda_fma, linear_fused

from .cuda_linear_layer import _precision, _zeros, weight_and_bias_grad


class CudaMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2):
        h, a, _ = linear_fused(x, w1, b1, _precision(), EPILOGUE_GELU, None, False)
        y = cuda_fma(a, w2, b2)
        ctx.save_for_backward(x, w1, w2, h, a)
        return y

    @staticmethod
    def backward(ctx, grad_output):
        x, w1, w2, h, a = ctx.saved_tensors
        dy = grad_output.contiguous()
        dh, _, _ = linear_fused(dy, w2.t().unsqueeze(0), _zeros(w2.shape[0], dy.device),
                                _precision(), EPILOGUE_GELU_GRAD, h, False)
        dw2, db2 = weight_and_bias_grad(a, dy)
        dw1, db1 = weight_and_bias_grad(x, dh)
        dx = cuda_fma(dh, w1.t().unsqueeze(0), _zeros(x.shape[-1], x.device))
        return dx, dw1, db1, dw2, db2
