"""The data-parallel GPT step's model (cuda_transformer_b200/gpt_case.py), built
from this package's operators, against the same network written with torch
operations in FP64 (the structure of gpt/gpt.py:47-175: pre-LN blocks, causal
attention on the fused QKV projection, exact GELU, tied lm_head): loss and
every parameter gradient after one backward."""
import pytest
import torch
import torch.nn.functional as F

from . import ct_helpers as H


def _ln(x, a, b):
    var = torch.var(x, dim=-1, keepdim=True, unbiased=False)
    return (x - x.mean(-1, keepdim=True)) / torch.sqrt(var + 1e-5) * a + b  # gpt/gpt.py:55-58


def reference_loss(p, idx, tgt, layers, heads, tied=True):
    B, T = idx.shape
    x = p["tok.weight"][idx] + p["pos.weight"][:T]
    C = x.shape[-1]
    for l in range(layers):
        q_ = f"blocks.{l}."
        h = _ln(x, p[q_ + "ln1.alpha"], p[q_ + "ln1.beta"])
        qkv = h @ p[q_ + "attn.qkv_weight"] + p[q_ + "attn.qkv_bias"]
        q, k, v = (t.reshape(B, T, heads, C // heads).transpose(1, 2) for t in qkv.chunk(3, -1))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, T, C)
        x = x + o @ p[q_ + "attn.out_weight"] + p[q_ + "attn.out_bias"]
        h = _ln(x, p[q_ + "ln2.alpha"], p[q_ + "ln2.beta"])
        h = F.gelu(h @ p[q_ + "mlp.fc1_weights"] + p[q_ + "mlp.fc1_bias"])
        x = x + h @ p[q_ + "mlp.fc2_weights"] + p[q_ + "mlp.fc2_bias"]
    x = _ln(x, p["ln.alpha"], p["ln.beta"])
    w = p["tok.weight"].t() if tied else p["lm_head_weights"]
    logits = x @ w + p["lm_head_bias"]
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1))


@pytest.mark.gpu
@pytest.mark.parametrize("layers,d,heads,ctx,batch", [(2, 128, 2, 128, 2), (1, 384, 6, 256, 2)])
def test_gpt_step_matches_fp64_torch(cuda_device, layers, d, heads, ctx, batch):
    from cuda_transformer_b200.gpt_case import GPT

    torch.manual_seed(0)
    model = GPT(layers, d, heads, ctx, 65).to(cuda_device)
    g = torch.Generator().manual_seed(1)
    t = torch.randint(0, 65, (batch, ctx + 1), generator=g).to(cuda_device)
    idx, tgt = t[:, :-1], t[:, 1:]
    _, loss = model(idx, tgt)
    loss.backward()
    ref_p = {k: v.detach().double().requires_grad_() for k, v in model.named_parameters()}
    ref = reference_loss(ref_p, idx, tgt, layers, heads)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-5 * abs(ref.item())
    for name, prm in model.named_parameters():
        assert H.rel_err(prm.grad, ref_p[name].grad) < 1e-4, name
    H.assert_device_clean()


@pytest.mark.gpu
def test_gpt_at_reference_model_shape(cuda_device):
    """gpt/gpt.py's own model shape (:16-22, :149-175): one block, d_model 512,
    4 heads of 128 -- the head size the reference launcher special-cases
    (flash_attn_launcher.cu:123-133) -- context 256, vocabulary 100256 with an
    untied lm_head and bias, here at 2 sequences, in the default
    (FP32-accurate) precision, against the same network in FP64 torch."""
    from cuda_transformer_b200.gpt_case import GPT

    layers, d, heads, ctx, vocab, batch = 1, 512, 4, 256, 100256, 2
    torch.manual_seed(117)
    model = GPT(layers, d, heads, ctx, vocab, tied=False).to(cuda_device)
    g = torch.Generator().manual_seed(3)
    t = torch.randint(0, vocab, (batch, ctx + 1), generator=g).to(cuda_device)
    idx, tgt = t[:, :-1], t[:, 1:]
    _, loss = model(idx, tgt)
    loss.backward()
    ref_p = {k: v.detach().double().requires_grad_() for k, v in model.named_parameters()}
    ref = reference_loss(ref_p, idx, tgt, layers, heads, tied=False)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-5 * abs(ref.item())
    for name, prm in model.named_parameters():
        assert H.rel_err(prm.grad, ref_p[name].grad) < 1e-4, name
    H.assert_device_clean()
