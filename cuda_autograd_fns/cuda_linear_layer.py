"""Linear layer autograd function (reference: cuda_autograd_fns/cuda_linear_layer.py:4-28).

Forward: out = x @ W + b with W stored (in, out).  Backward: dx = dy @ W^T;
dW is one GEMM with the (batch, seq) dimensions folded into the reduction
(x^T @ dy over batch*seq rows) instead of a per-batch product followed by a
torch sum, and db -- the column sums of dy -- is formed inside that same GEMM
from the dy tiles it stages (no separate pass over dy).  The zero biases of
the two backward products are cached per device and length (the operator only
reads them)."""
import functools
import os

import torch
from cuda_transformer.ops import cuda_fma, db_calculation, linear_fused

_ZEROS = {}


def _zeros(n, device):
    """A cached all-zero bias of length n (the operator only reads it)."""
    key = (device, n)
    z = _ZEROS.get(key)
    if z is None:
        z = _ZEROS[key] = torch.zeros(n, dtype=torch.float32, device=device)
    return z


@functools.lru_cache(maxsize=1)
def _precision():
    """The operators' default precision (CUDA_TRANSFORMER_PRECISION, read once
    like the operator library does)."""
    return {"tf32": 1, "fp32": 2, "simt": 2}.get(os.environ.get("CUDA_TRANSFORMER_PRECISION", ""), 0)


def weight_and_bias_grad(x, dy, precision=None):
    """dW = x^T dy and db = colsum(dy) over all leading dimensions, in one GEMM
    (x (..., k), dy (..., n))."""
    rows = x.numel() // x.shape[-1]
    x2 = x.reshape(1, rows, x.shape[-1])
    dy2 = dy.reshape(1, rows, dy.shape[-1])
    dw, _, db = linear_fused(x2.transpose(1, 2), dy2, _zeros(dy.shape[-1], dy.device),
                             _precision() if precision is None else precision, 0, None, True)
    return dw[0], db


class CudaLinearLayer(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, bias):
        out = cuda_fma(x, weights, bias)
        ctx.save_for_backward(x, weights, bias)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        x, weights, _ = ctx.saved_tensors
        dy = grad_output
        w = weights.unsqueeze(0) if weights.dim() == 2 else weights
        dx = cuda_fma(dy, w.transpose(1, 2), _zeros(x.shape[-1], x.device))
        if weights.dim() == 2:
            dw, db = weight_and_bias_grad(x, dy)
        else:
            dw = cuda_fma(x.transpose(1, 2), dy, _zeros(dy.shape[-1], dy.device))
            db = db_calculation(dy)
        return dx, dw, db
