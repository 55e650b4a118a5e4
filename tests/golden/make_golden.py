"""Generates the committed golden vectors in this directory.

The expected values come from the reference test-suite's own math
(test/test_flash_attention.py:10-49, test/test_softmax.py, test/test_gelu.py,
test/test_linear.py, gpt/gpt.py:55-58) evaluated by PyTorch on the CPU in
float64 -- ``oracle.torch_ref.sdpa_reference`` for attention -- on inputs drawn
with fixed seeds.  Inputs and expectations are stored as float32 (the
expectations rounded once from float64).

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from oracle.torch_ref import sdpa_reference  # noqa: E402

# (name, B, H, T, D, causal); cfg1* are the per-head shape of BASELINE config 1
FA2_CASES = [
    ("cfg1_causal", 1, 1, 256, 64, True),
    ("cfg1_full", 1, 1, 256, 64, False),
    ("ragged65_causal", 1, 1, 65, 64, True),
    ("ragged129_d32", 2, 1, 129, 32, False),
    ("d128_causal", 1, 1, 64, 128, True),
]


def fa2_golden() -> dict:
    out = {}
    for i, (name, B, H, T, D, causal) in enumerate(FA2_CASES):
        g = torch.Generator().manual_seed(1000 + i)
        q, k, v, do = (torch.randn(B, H, T, D, generator=g, dtype=torch.float32) for _ in range(4))
        o, lse, dq, dk, dv = sdpa_reference(q.double(), k.double(), v.double(), do.double(), causal)
        for key, val in dict(q=q, k=k, v=v, do=do).items():
            out[f"{name}/{key}"] = val.numpy()
        for key, val in dict(o=o, lse=lse, dq=dq, dk=dk, dv=dv).items():
            out[f"{name}/{key}"] = val.numpy().astype(np.float32)
        out[f"{name}/causal"] = np.array(causal)
    return out


def rowops_golden() -> dict:
    g = torch.Generator().manual_seed(7)
    out = {}
    x = torch.randn(2, 33, 70, generator=g)
    dp = torch.rand(2, 33, 70, generator=g)
    xd = x.double().requires_grad_(True)
    p = F.softmax(xd, dim=-1)
    p.backward(dp.double())
    out.update({"softmax/x": x.numpy(), "softmax/dp": dp.numpy(),
                "softmax/p": p.detach().numpy(), "softmax/dx": xd.grad.numpy()})
    xg = torch.randn(3, 17, 50, generator=g)
    dy = torch.rand(3, 17, 50, generator=g)
    xd = xg.double().requires_grad_(True)
    y = F.gelu(xd)
    y.backward(dy.double())
    out.update({"gelu/x": xg.numpy(), "gelu/dy": dy.numpy(), "gelu/y": y.detach().numpy(),
                "gelu/dx": xd.grad.numpy()})
    xl = torch.randn(5, 384, generator=g)
    gam = 1.0 + 0.1 * torch.randn(384, generator=g)
    bet = 0.1 * torch.randn(384, generator=g)
    dyl = torch.randn(5, 384, generator=g)
    xd, gd, bd = (t.double().requires_grad_(True) for t in (xl, gam, bet))
    var = torch.var(xd, dim=-1, keepdim=True, unbiased=False)
    mean = torch.mean(xd, dim=-1, keepdim=True)
    yl = (xd - mean) / torch.sqrt(var + 1e-5) * gd + bd
    yl.backward(dyl.double())
    out.update({"ln/x": xl.numpy(), "ln/gamma": gam.numpy(), "ln/beta": bet.numpy(),
                "ln/dy": dyl.numpy(), "ln/y": yl.detach().numpy(), "ln/dx": xd.grad.numpy(),
                "ln/dgamma": gd.grad.numpy(), "ln/dbeta": bd.grad.numpy()})
    xf = torch.rand(1, 32, 65, generator=g)
    w = torch.randn(65, 32, generator=g) * 0.1
    b = torch.randn(32, generator=g) * 0.1
    dyf = torch.rand(1, 32, 32, generator=g)
    xd, wd, bd = (t.double().requires_grad_(True) for t in (xf, w, b))
    yf = xd @ wd + bd
    yf.backward(dyf.double())
    out.update({"linear/x": xf.numpy(), "linear/w": w.numpy(), "linear/b": b.numpy(),
                "linear/dy": dyf.numpy(), "linear/y": yf.detach().numpy(),
                "linear/dx": xd.grad.numpy(), "linear/dw": wd.grad.numpy(),
                "linear/db": bd.grad.numpy()})
    return out


def main() -> None:
    np.savez_compressed(HERE / "fa2_golden.npz", **fa2_golden())
    np.savez_compressed(HERE / "rowops_golden.npz", **rowops_golden())
    print("wrote", HERE / "fa2_golden.npz", HERE / "rowops_golden.npz")


if __name__ == "__main__":
    main()
