"""Python wrappers over ``torch.ops.cuda_transformer`` with fake (meta)
implementations -- the same ten functions, names and argument meaning as the
reference's ``cuda_transformer/ops.py:4-139``, plus this implementation's
LayerNorm and precision-explicit variants.

``precision`` (the ``*_ex`` functions): 0 = 3xTF32 (FP32-accurate, the default
of the plain functions), 1 = TF32, 2 = FP32 on the CUDA cores.  The plain
functions follow the ``CUDA_TRANSFORMER_PRECISION`` environment variable.
"""
import torch
from torch import Tensor

__all__ = [
    "cuda_fma", "db_calculation",
    "cuda_softmax", "cuda_softmax_bwd",
    "gelu_activation", "gelu_activation_bwd",
    "causal_self_attention_fwd", "causal_self_attention_bwd",
    "flash_attention_fwd", "flash_attention_bwd",
    "flash_attention_fwd_ex", "flash_attention_bwd_ex", "cuda_fma_ex",
    "layernorm_fwd", "layernorm_bwd",
    "linear_fused", "linear_accumulate_", "cross_entropy_fwd_bwd_",
]

PRECISION_3XTF32 = 0
PRECISION_TF32 = 1
PRECISION_FP32 = 2
EPILOGUE_NONE = 0
EPILOGUE_GELU = 1
EPILOGUE_GELU_GRAD = 2


def _f32(*ts):
    for t in ts:
        torch._check(t.dtype == torch.float32)


def _same_device(*ts):
    torch._check(all(t.device == ts[0].device for t in ts))


# ---------------------------------------------------------------- linear layer
def cuda_fma(x: Tensor, weights: Tensor, bias: Tensor) -> Tensor:
    """out[b] = x[b] @ weights[b or 0] + bias (weights pre-transposed, (k, n))."""
    return torch.ops.cuda_transformer.cuda_fma.default(x, weights, bias)


def cuda_fma_ex(x: Tensor, weights: Tensor, bias: Tensor, precision: int) -> Tensor:
    """cuda_fma with an explicit precision mode."""
    return torch.ops.cuda_transformer.cuda_fma_ex.default(x, weights, bias, precision)


def _fma_meta(x, weights, bias):
    _f32(x, weights, bias)
    _same_device(x, weights, bias)
    w = weights if weights.dim() == 3 else weights.unsqueeze(0)
    return torch.empty(x.size(0), x.size(1), w.size(2), dtype=x.dtype, device=x.device)


@torch.library.register_fake("cuda_transformer::cuda_fma")
def _(x, weights, bias):
    return _fma_meta(x, weights, bias)


@torch.library.register_fake("cuda_transformer::cuda_fma_ex")
def _(x, weights, bias, precision):
    return _fma_meta(x, weights, bias)


def db_calculation(dy: Tensor) -> Tensor:
    """Bias gradient: column sum of dy over (batch, m)."""
    return torch.ops.cuda_transformer.db_calculation.default(dy)


@torch.library.register_fake("cuda_transformer::db_calculation")
def _(dy):
    _f32(dy)
    return torch.empty(dy.size(-1), dtype=dy.dtype, device=dy.device)


# --------------------------------------------------------------------- softmax
def cuda_softmax(x: Tensor) -> Tensor:
    """Row softmax over the last dimension of a contiguous 3-D tensor."""
    return torch.ops.cuda_transformer.cuda_softmax.default(x)


@torch.library.register_fake("cuda_transformer::cuda_softmax")
def _(x):
    _f32(x)
    return torch.empty_like(x)


def cuda_softmax_bwd(probs: Tensor, dp: Tensor) -> Tensor:
    """Softmax backward: probs * (dp - sum(probs * dp))."""
    return torch.ops.cuda_transformer.cuda_softmax_bwd.default(probs, dp)


@torch.library.register_fake("cuda_transformer::cuda_softmax_bwd")
def _(probs, dp):
    _f32(probs, dp)
    _same_device(probs, dp)
    return torch.empty_like(probs)


# ------------------------------------------------------------------------ GELU
def gelu_activation(x: Tensor) -> Tensor:
    """Exact (erf) GELU."""
    return torch.ops.cuda_transformer.gelu_activation.default(x)


@torch.library.register_fake("cuda_transformer::gelu_activation")
def _(x):
    _f32(x)
    return torch.empty_like(x)


def gelu_activation_bwd(x: Tensor, dy: Tensor) -> Tensor:
    """GELU backward."""
    return torch.ops.cuda_transformer.gelu_activation_bwd.default(x, dy)


@torch.library.register_fake("cuda_transformer::gelu_activation_bwd")
def _(x, dy):
    _f32(x, dy)
    _same_device(x, dy)
    return torch.empty_like(x)


# ------------------------------------------------- materialised attention
def causal_self_attention_fwd(qkv: Tensor, nh: int, causal: bool) -> tuple[Tensor, Tensor]:
    """Attention with the full probability matrix (not the hot path)."""
    return torch.ops.cuda_transformer.causal_self_attention_fwd.default(qkv, nh, causal)


@torch.library.register_fake("cuda_transformer::causal_self_attention_fwd")
def _(qkv, nh, causal):
    _f32(qkv)
    b, t, three_c = qkv.shape
    c = three_c // 3
    out = torch.empty((b, t, c), dtype=qkv.dtype, device=qkv.device)
    probs = torch.empty((b, nh, t, t), dtype=qkv.dtype, device=qkv.device)
    return out, probs


def causal_self_attention_bwd(Q: Tensor, K: Tensor, V: Tensor, probs: Tensor,
                              dO: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Backward of causal_self_attention_fwd (dq, dk returned times sqrt(hs))."""
    return torch.ops.cuda_transformer.causal_self_attention_bwd.default(Q, K, V, probs, dO)


@torch.library.register_fake("cuda_transformer::causal_self_attention_bwd")
def _(Q, K, V, probs, dO):
    _f32(Q, K, V, probs, dO)
    _same_device(Q, K, V, probs, dO)
    return torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)


# ------------------------------------------------------------ FlashAttention-2
def flash_attention_fwd(Q: Tensor, K: Tensor, V: Tensor, causal: bool) -> tuple[Tensor, Tensor]:
    """FlashAttention-2 forward: returns O [B,nh,T,hs] and L = logsumexp [B,nh,T]."""
    return torch.ops.cuda_transformer.flash_attention_fwd.default(Q, K, V, causal)


def flash_attention_fwd_ex(Q: Tensor, K: Tensor, V: Tensor, causal: bool,
                           precision: int) -> tuple[Tensor, Tensor]:
    """flash_attention_fwd with an explicit precision mode."""
    return torch.ops.cuda_transformer.flash_attention_fwd_ex.default(Q, K, V, causal, precision)


def _fa_fwd_meta(Q, K, V):
    _f32(Q, K, V)
    _same_device(Q, K, V)
    O = torch.empty((Q.size(0), Q.size(1), Q.size(2), Q.size(3)), dtype=Q.dtype, device=Q.device)
    L = torch.empty((Q.size(0), Q.size(1), Q.size(2)), dtype=Q.dtype, device=Q.device)
    return O, L


@torch.library.register_fake("cuda_transformer::flash_attention_fwd")
def _(Q, K, V, causal):
    return _fa_fwd_meta(Q, K, V)


@torch.library.register_fake("cuda_transformer::flash_attention_fwd_ex")
def _(Q, K, V, causal, precision):
    return _fa_fwd_meta(Q, K, V)


def flash_attention_bwd(Q: Tensor, K: Tensor, V: Tensor, O: Tensor, dO: Tensor, L: Tensor,
                        causal: bool):
    """FlashAttention-2 backward: returns dQ, dK, dV."""
    return torch.ops.cuda_transformer.flash_attention_bwd.default(Q, K, V, O, dO, L, causal)


def flash_attention_bwd_ex(Q: Tensor, K: Tensor, V: Tensor, O: Tensor, dO: Tensor, L: Tensor,
                           causal: bool, precision: int):
    """flash_attention_bwd with an explicit precision mode."""
    return torch.ops.cuda_transformer.flash_attention_bwd_ex.default(Q, K, V, O, dO, L, causal,
                                                                     precision)


def _fa_bwd_meta(Q, K, V, O, dO, L):
    _f32(Q, K, V, O, dO, L)
    _same_device(Q, K, V, O, dO, L)
    return (torch.empty(Q.shape, dtype=Q.dtype, device=Q.device),
            torch.empty(K.shape, dtype=K.dtype, device=K.device),
            torch.empty(V.shape, dtype=V.dtype, device=V.device))


@torch.library.register_fake("cuda_transformer::flash_attention_bwd")
def _(Q, K, V, O, dO, L, causal):
    return _fa_bwd_meta(Q, K, V, O, dO, L)


@torch.library.register_fake("cuda_transformer::flash_attention_bwd_ex")
def _(Q, K, V, O, dO, L, causal, precision):
    return _fa_bwd_meta(Q, K, V, O, dO, L)


# ------------------------------------------------------------------- LayerNorm
def layernorm_fwd(x: Tensor, gamma: Tensor, beta: Tensor, eps: float = 1e-5):
    """LayerNorm over the last dim (biased variance); returns y, mean, rstd."""
    return torch.ops.cuda_transformer.layernorm_fwd.default(x, gamma, beta, eps)


@torch.library.register_fake("cuda_transformer::layernorm_fwd")
def _(x, gamma, beta, eps):
    _f32(x, gamma, beta)
    rows = x.numel() // x.size(-1)
    return (torch.empty_like(x), torch.empty(rows, dtype=x.dtype, device=x.device),
            torch.empty(rows, dtype=x.dtype, device=x.device))


def layernorm_bwd(x: Tensor, gamma: Tensor, mean: Tensor, rstd: Tensor, dy: Tensor):
    """LayerNorm backward; returns dx, dgamma, dbeta."""
    return torch.ops.cuda_transformer.layernorm_bwd.default(x, gamma, mean, rstd, dy)


@torch.library.register_fake("cuda_transformer::layernorm_bwd")
def _(x, gamma, mean, rstd, dy):
    _f32(x, gamma, mean, rstd, dy)
    return torch.empty_like(x), torch.empty_like(gamma), torch.empty_like(gamma)


# ------------------------------------------------- linear layer, fused options
def linear_fused(x: Tensor, weights: Tensor, bias: Tensor, precision: int = PRECISION_3XTF32,
                 epilogue: int = EPILOGUE_NONE, act_in: Tensor | None = None,
                 want_colsum: bool = False):
    """out = x @ weights + bias with GELU (EPILOGUE_GELU: also returns
    gelu(out)) or the GELU gradient (EPILOGUE_GELU_GRAD: out * gelu'(act_in))
    applied in the GEMM's epilogue, and optionally the column sums of
    `weights` over its reduction index (the bias gradient when weights is dY,
    batch 1).  Returns (out, act, colsum); unused ones are empty."""
    return torch.ops.cuda_transformer.linear_fused.default(x, weights, bias, precision, epilogue,
                                                           act_in, want_colsum)


@torch.library.register_fake("cuda_transformer::linear_fused")
def _(x, weights, bias, precision, epilogue, act_in, want_colsum):
    out = _fma_meta(x, weights, bias)
    act = torch.empty_like(out) if epilogue == EPILOGUE_GELU else out.new_empty(0)
    cs = out.new_empty(out.size(2)) if want_colsum else out.new_empty(0)
    return out, act, cs


def linear_accumulate_(out: Tensor, colsum: Tensor | None, x: Tensor, weights: Tensor,
                       bias: Tensor, precision: int = PRECISION_3XTF32) -> None:
    """out += x @ weights + bias, and colsum += the column sums of weights."""
    torch.ops.cuda_transformer.linear_accumulate_.default(out, colsum, x, weights, bias, precision)


@torch.library.register_fake("cuda_transformer::linear_accumulate_")
def _(out, colsum, x, weights, bias, precision):
    return None


def cross_entropy_fwd_bwd_(logits: Tensor, targets: Tensor, ignore_index: int = -100) -> Tensor:
    """Per-row cross entropy of (rows, vocab) logits; the logits are
    overwritten with softmax - onehot(targets) (unscaled gradient)."""
    return torch.ops.cuda_transformer.cross_entropy_fwd_bwd_.default(logits, targets, ignore_index)


@torch.library.register_fake("cuda_transformer::cross_entropy_fwd_bwd_")
def _(logits, targets, ignore_index):
    return logits.new_empty(logits.size(0))
