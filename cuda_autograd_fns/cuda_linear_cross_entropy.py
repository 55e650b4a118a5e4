"""lm_head + cross entropy (gpt/gpt.py:167-175) without materialising the
logits of every row.

logits = x W + b feeds F.cross_entropy (mean over the counted rows) in the
reference; with its vocabulary of 100256 the logits are the largest
activation of the model.  Here the rows go through in chunks: each chunk's
logits come from the linear-layer GEMM, one kernel turns them in place into
the per-row loss and the unscaled gradient softmax - onehot(target), and the
chunk's input gradient (dlogits W^T), weight gradient and bias gradient (one
accumulating GEMM, db formed from the dlogits tiles it stages) are formed at
once.  Only one chunk of logits is ever alive; the backward scales the saved
gradients by grad_output / (counted rows)."""
import torch
from cuda_transformer.ops import cross_entropy_fwd_bwd_, cuda_fma_ex, linear_accumulate_

from .cuda_linear_layer import _precision, _zeros

CHUNK_BYTES = 256 << 20  # logits held at once


class CudaLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, bias, targets, ignore_index=-100, chunk_rows=None):
        d, vocab = weights.shape
        x2 = x.reshape(-1, d)
        t = targets.reshape(-1)
        rows = x2.shape[0]
        prec = _precision()
        step = chunk_rows or max(1, min(rows, CHUNK_BYTES // (4 * vocab)))
        loss_rows = torch.empty(rows, device=x.device, dtype=torch.float32)
        dx = torch.empty(rows, d, device=x.device, dtype=torch.float32)
        dw = torch.zeros(d, vocab, device=x.device, dtype=torch.float32)
        db = torch.zeros(vocab, device=x.device, dtype=torch.float32)
        w_t = weights.t().unsqueeze(0)
        zero_d, zero_v = _zeros(d, x.device), _zeros(vocab, x.device)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            xc = x2[r0:r1].unsqueeze(0)
            logits = cuda_fma_ex(xc, weights, bias, prec)[0]            # (c, vocab)
            loss_rows[r0:r1] = cross_entropy_fwd_bwd_(logits, t[r0:r1], ignore_index)
            g = logits.unsqueeze(0)                                       # softmax - onehot
            dx[r0:r1] = cuda_fma_ex(g, w_t, zero_d, prec)[0]
            linear_accumulate_(dw.unsqueeze(0), db, xc.transpose(1, 2), g, zero_v, prec)
        counted = (t != ignore_index).sum().clamp_min(1).to(torch.float32)
        ctx.save_for_backward(dx, dw, db, counted)
        ctx.x_shape = x.shape
        return loss_rows.sum() / counted

    @staticmethod
    def backward(ctx, grad_output):
        dx, dw, db, counted = ctx.saved_tensors
        s = grad_output / counted
        return (dx * s).reshape(ctx.x_shape), dw * s, db * s, None, None, None
