"""Data-parallel GPT training step built from the cuda_transformer operators.

The model follows the reference GPT (gpt/gpt.py:47-175): token + position
embedding, pre-LayerNorm decoder blocks (x + attn(ln1(x)), x + mlp(ln2(x))),
causal FlashAttention-2 on the (B, nh, T, hs) views of the fused QKV
projection, an exact-GELU 4x MLP, a final LayerNorm and the lm_head, with the
cross-entropy loss.  Every linear layer, LayerNorm, GELU, attention and the
large-vocabulary loss run on this package's kernels (CudaLinearLayer,
CudaLayerNorm, CudaFlashAttention, CudaMLP; the weight gradients form the bias
gradients in the same GEMM; with a vocabulary of FUSED_CE_MIN_VOCAB or more,
CudaLinearCrossEntropy runs the lm_head and the loss chunk by chunk so the
logits of every row are never held at once); the embeddings, AdamW and the
small-vocabulary loss are torch's.

Default shape (the data-parallel benchmark configuration): 6 blocks,
d_model 384, 6 heads of 64, context 256, vocabulary 65 with the lm_head tied to
the token embedding, 64 sequences per GPU, AdamW lr 3e-4, weights
N(0, 0.02).  gpt/gpt.py's own shape: --layers 1 --d 512 --heads 4 --vocab 100256
--untied.  Tokens are uniform in [0, vocab), seeded per rank, staged in
pinned host memory and copied to the GPU inside every timed step (as the
reference's Generate_Batch does, gpt/gpt.py:39-45).

One process per GPU (torchrun); with more than one, gradients are averaged by
torch DistributedDataParallel over NCCL: bucketed all-reduces that start
while the backward is still running.  The step time is the maximum over ranks
of the CUDA-event time of the timed steps.  With N > 1 the line also reports
the communication the step exposes: the same steps timed again with DDP's
gradient synchronisation switched off (``no_sync``: compute only), the
difference to the synchronised step, and one stand-alone all-reduce of all
gradients (a bound on the communication if none of it overlapped).

  python -m cuda_transformer_b200.gpt_case [--steps 20 --warmup 5]
  torchrun --nproc-per-node N -m cuda_transformer_b200.gpt_case --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.nn as nn

import torch.nn.functional as F

from cuda_autograd_fns import (CudaFlashAttention, CudaLayerNorm, CudaLinearCrossEntropy,
                               CudaLinearLayer, CudaMLP)

# The fused lm_head + loss pays where the logits are large (gpt/gpt.py's
# 100256-token vocabulary); for 65 characters torch's loss on the full logits
# is cheaper than chunking.
FUSED_CE_MIN_VOCAB = 4096


class LayerNorm(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.alpha = nn.Parameter(torch.ones(d))
        self.beta = nn.Parameter(torch.zeros(d))

    def forward(self, x):
        return CudaLayerNorm.apply(x, self.alpha, self.beta, 1e-5)


class Attention(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.heads, self.hs = heads, d // heads
        self.qkv_weight = nn.Parameter(torch.empty(d, 3 * d).normal_(0.0, 0.02))
        self.qkv_bias = nn.Parameter(torch.zeros(3 * d))
        self.out_weight = nn.Parameter(torch.empty(d, d).normal_(0.0, 0.02))
        self.out_bias = nn.Parameter(torch.zeros(d))

    def forward(self, x):
        B, T, C = x.shape
        qkv = CudaLinearLayer.apply(x, self.qkv_weight, self.qkv_bias)
        # strided (B, nh, T, hs) views: the attention kernels read them in place
        q, k, v = (t.reshape(B, T, self.heads, self.hs).transpose(1, 2) for t in qkv.chunk(3, dim=-1))
        o, _ = CudaFlashAttention.apply(q, k, v, True)
        o = o.transpose(1, 2).reshape(B, T, C)
        return CudaLinearLayer.apply(o, self.out_weight, self.out_bias)


class MLP(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.fc1_weights = nn.Parameter(torch.empty(d, 4 * d).normal_(0.0, 0.02))
        self.fc1_bias = nn.Parameter(torch.zeros(4 * d))
        self.fc2_weights = nn.Parameter(torch.empty(4 * d, d).normal_(0.0, 0.02))
        self.fc2_bias = nn.Parameter(torch.zeros(d))

    def forward(self, x):  # fc1 -> GELU -> fc2
        return CudaMLP.apply(x, self.fc1_weights, self.fc1_bias, self.fc2_weights, self.fc2_bias)


class Block(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.ln1, self.attn, self.ln2, self.mlp = LayerNorm(d), Attention(d, heads), LayerNorm(d), MLP(d)

    def forward(self, x):
        x = x + self.attn(self.ln1(x))
        return x + self.mlp(self.ln2(x))


class GPT(nn.Module):
    def __init__(self, layers=6, d=384, heads=6, ctx=256, vocab=65, tied=True):
        super().__init__()
        self.tok = nn.Embedding(vocab, d)
        self.pos = nn.Embedding(ctx, d)
        nn.init.normal_(self.tok.weight, 0.0, 0.02)
        nn.init.normal_(self.pos.weight, 0.0, 0.02)
        self.blocks = nn.ModuleList([Block(d, heads) for _ in range(layers)])
        self.ln = LayerNorm(d)
        self.tied = tied
        if not tied:
            self.lm_head_weights = nn.Parameter(torch.empty(d, vocab).normal_(0.0, 0.02))
        self.lm_head_bias = nn.Parameter(torch.zeros(vocab))

    def forward(self, idx, targets=None):
        """(logits, None) without targets; with them the mean cross-entropy
        loss, as (None, loss) when the lm_head and the loss run fused (large
        vocabularies), else (logits, loss)."""
        T = idx.shape[1]
        x = self.tok(idx) + self.pos(torch.arange(T, device=idx.device))
        for blk in self.blocks:
            x = blk(x)
        x = self.ln(x)
        w = self.tok.weight.t() if self.tied else self.lm_head_weights
        if targets is not None and w.shape[1] >= FUSED_CE_MIN_VOCAB:
            return None, CudaLinearCrossEntropy.apply(x, w, self.lm_head_bias, targets)
        logits = CudaLinearLayer.apply(x, w, self.lm_head_bias)
        if targets is None:
            return logits, None
        return logits, F.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))


def n_params(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def matmul_params(model: "GPT") -> int:
    """Parameters that enter a matrix product: all but the position table and,
    when the lm_head has its own weights, the token table (a lookup)."""
    skip = model.pos.weight.numel() + (0 if model.tied else model.tok.weight.numel())
    return n_params(model) - skip


def step_flops(params: int, layers: int, d: int, ctx: int, tokens: int) -> float:
    """Training FLOPs of one step: 6 * params * tokens for the dense layers
    (params: matmul_params),
    plus causal attention (2 * 2 * T * d per token per layer forward, half of
    it masked, x3 for forward + backward)."""
    return 6.0 * params * tokens + 3.0 * 2.0 * layers * ctx * d * tokens


def rank_batches(seed: int, n: int, batch: int, ctx: int, vocab: int) -> list:
    """n (input, target) token batches in pinned host memory, seeded per rank."""
    g = torch.Generator().manual_seed(seed)
    pin = torch.cuda.is_available()
    out = []
    for _ in range(n):
        t = torch.randint(0, vocab, (batch, ctx + 1), generator=g, dtype=torch.int64)
        x, y = t[:, :-1].contiguous(), t[:, 1:].contiguous()
        out.append((x.pin_memory(), y.pin_memory()) if pin else (x, y))
    return out


def max_over_ranks(ms: float, dist, world: int, device) -> float:
    """The job's time: the maximum over ranks of a per-rank time."""
    if world == 1:
        return ms
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def tokens_per_step(world: int, batch_per_gpu: int, ctx: int) -> int:
    """Weak scaling: every rank trains batch_per_gpu sequences of ctx tokens."""
    return world * batch_per_gpu * ctx


def timed_ms(fn, steps: int) -> float:
    """CUDA-event time of `steps` calls of fn() on the current stream."""
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--d", type=int, default=384)
    ap.add_argument("--heads", type=int, default=6)
    ap.add_argument("--ctx", type=int, default=256)
    ap.add_argument("--vocab", type=int, default=65)
    ap.add_argument("--batch", type=int, default=64, help="sequences per GPU")
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--gpus", type=int, default=None,
                    help="expected number of ranks (launch N > 1 with torchrun)")
    ap.add_argument("--untied", action="store_true",
                    help="separate lm_head weights and bias, as gpt/gpt.py has them")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.gpus is not None and a.gpus != world:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}: launch one process per GPU "
                         "with torchrun --nproc-per-node N")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    torch.manual_seed(1234)  # identical initial weights on every rank
    model = GPT(a.layers, a.d, a.heads, a.ctx, a.vocab, tied=not a.untied).to(dev)
    params = n_params(model)
    net = model
    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP
        net = DDP(model, device_ids=[local], gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=a.lr, fused=True)
    batches = rank_batches(1000 + rank, 8, a.batch, a.ctx, a.vocab)

    losses = []

    def step(i):
        x, y = batches[i % len(batches)]
        x = x.to(dev, non_blocking=True)
        y = y.to(dev, non_blocking=True)
        _, loss = net(x, y)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for i in range(a.warmup):
        losses.append(step(i).item())
    if world > 1:
        dist.barrier()
    last = [None]

    def timed_step(i):
        last[0] = step(a.warmup + i)

    ms = timed_ms(timed_step, a.steps)
    losses.append(last[0].item())
    ms = max_over_ranks(ms, dist, world, dev)
    comm = None
    if world > 1:
        # the same steps without DDP's gradient all-reduces (compute only), and
        # one stand-alone all-reduce of every gradient (fp32, flattened)
        dist.barrier()

        def unsynced(i):
            with net.no_sync():
                step(a.warmup + a.steps + i)

        ms_nosync = max_over_ranks(timed_ms(unsynced, a.steps), dist, world, dev)
        flat = torch.zeros(params, device=dev)
        dist.all_reduce(flat)  # warm-up
        dist.barrier()
        ar_ms = max_over_ranks(timed_ms(lambda i: dist.all_reduce(flat), 5) / 5, dist, world, dev)
        dist.barrier()
        step_ms, comp_ms = ms / a.steps, ms_nosync / a.steps
        comm = {"allreduce_bytes": params * 4, "allreduce_ms_standalone": ar_ms,
                "allreduce_share_if_unoverlapped": ar_ms / step_ms,
                "step_ms_without_sync": comp_ms,
                "exposed_comm_ms": step_ms - comp_ms,
                "exposed_comm_share": (step_ms - comp_ms) / step_ms,
                "allreduce_busbw_gbs": 2.0 * (world - 1) / world * params * 4 / (ar_ms * 1e-3) / 1e9}
    tokens = tokens_per_step(world, a.batch, a.ctx)
    if rank == 0:
        flops = step_flops(matmul_params(model), a.layers, a.d, a.ctx, tokens)
        print(json.dumps({
            "metric": "GPT DP training tokens/s", "value": tokens * a.steps / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "ms_per_step": ms / a.steps, "steps": a.steps,
            "warmup": a.warmup, "tflops": flops * a.steps / (ms * 1e-3) / 1e12,
            "scaling": "weak", "params": params, "loss_first": losses[0], "loss_last": losses[-1],
            "loss_uniform": math.log(a.vocab), "communication": comm,
            "config": {"layers": a.layers, "d_model": a.d, "heads": a.heads, "ctx": a.ctx,
                       "vocab": a.vocab, "batch_per_gpu": a.batch, "global_batch": a.batch * world,
                       "tied": not a.untied, "optimizer": "AdamW(fused) lr %g" % a.lr,
                       "grad_sync": "DDP bucketed NCCL all-reduce" if world > 1 else "none"},
            "data": "synthetic uniform tokens, pinned host -> device each step"}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
