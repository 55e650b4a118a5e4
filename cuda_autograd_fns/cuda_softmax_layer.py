"""Row-softmax autograd function (reference: cuda_autograd_fns/cuda_softmax_layer.py:4-15)."""
import torch
from cuda_transformer.ops import cuda_softmax, cuda_softmax_bwd


class CudaSoftmaxLayer(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        out = cuda_softmax(x)
        ctx.save_for_backward(out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        out, = ctx.saved_tensors
        return cuda_softmax_bwd(out, grad_output.contiguous())
