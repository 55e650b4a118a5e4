"""Times the linear layer and the row-wise kernels through the C ABI at the
measurement shapes and prints one JSON line per kernel with its roofline:

  linear  x[16384,384] @ W[384,1536] + b  and  x[16384,1536] @ W[1536,384] + b,
          plus the backward's dx = dy W^T and dW = x^T dy (2 M N K FLOP each)
  softmax [16384,4096]  fwd (read x, write y), bwd (read p, dp, write dx)
  layernorm [16384,384] fwd (read x, write y), bwd (read x, dy, write dx);
            --ln-cols sets the row width (above 1024: the one-CTA-per-row kernels)
  gelu    [16384,1536]  fwd (read x, write y), bwd (read x, dy, write dx)
  bias grad of dy[16384,1536] (read dy)

The linear layer runs through ct_linear_fwd_ws with its workspace, as the
cuda_fma operator calls it.  Each launch is timed alone with CUDA events on
the current stream after a read of a 256 MiB buffer, so every launch starts
with a cold L2.
Peaks come from MEASURED_PEAKS.json at the repository root (dense TF32 is
half the measured dense BF16 rate).

  python -m cuda_transformer_b200.ops_case [--iters 20] [--only linear,softmax,...]
"""
from __future__ import annotations

import argparse
import ctypes
import json
from pathlib import Path

import torch

from . import PRECISION_3XTF32, PRECISION_FP32, PRECISION_TF32, check, device_status, lib

ROOT = Path(__file__).resolve().parent.parent
PREC = {"3xtf32": PRECISION_3XTF32, "tf32": PRECISION_TF32, "fp32": PRECISION_FP32}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return {"hbm_gbs": float(j.get("hbm_gbs", 6650.0)),
                "bf16_tflops": float(j.get("bf16_tflops", 1590.0)), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Timer:
    """Cold-L2 timing: before each launch a 256 MiB buffer is read, so L2
    holds only clean, unrelated lines (a write flush would leave dirty lines
    whose write-back the timed kernel would pay for)."""

    def __init__(self, dev):
        self.flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def __call__(self, fn, iters: int, warmup: int = 3) -> float:
        for _ in range(warmup):
            fn()
        total = 0.0
        for _ in range(iters):
            self.flush.max()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            total += a.elapsed_time(b)
        return total / iters


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _st():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _s3(t):
    return (ctypes.c_int64 * 3)(*t.stride())


def linear_cases(dev, timer, iters, pk, precisions):
    L = lib()
    tf32_peak = pk["bf16_tflops"] / 2.0
    out = []
    g = torch.Generator(device=dev).manual_seed(0)
    for (m, k, n) in [(16384, 384, 1536), (16384, 1536, 384)]:
        x = torch.randn(1, m, k, device=dev, generator=g)
        w = 0.02 * torch.randn(1, k, n, device=dev, generator=g)
        b = 0.02 * torch.randn(n, device=dev, generator=g)
        dy = torch.randn(1, m, n, device=dev, generator=g)
        y = torch.empty(1, m, n, device=dev)
        dx = torch.empty(1, m, k, device=dev)
        dw = torch.empty(1, k, n, device=dev)
        zk, zn = torch.zeros(k, device=dev), torch.zeros(n, device=dev)
        wt = w.transpose(1, 2)        # dx = dy @ W^T  (W^T K-major)
        xt = x.transpose(1, 2)        # dW = x^T @ dy  (x^T MN-major)
        calls = {
            "fwd": (x, w, b, y, m, k, n),
            "bwd_dx": (dy, wt, zk, dx, m, n, k),
            "bwd_dw": (xt, dy, zn, dw, k, m, n),
        }
        for name, (A, W, bias, o, mm, kk, nn) in calls.items():
            for pname in precisions:
                prec = PREC[pname]

                wsb = L.ct_linear_workspace_size(1, mm, kk, nn)
                ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)

                def run(A=A, W=W, bias=bias, o=o, mm=mm, kk=kk, nn=nn, prec=prec, ws=ws, wsb=wsb):
                    check(L.ct_linear_fwd_ws(_p(A), _s3(A), _p(W), _s3(W), _p(bias),
                                             bias.stride(0), _p(o), 1, mm, kk, nn, 1, prec,
                                             _p(ws), wsb, _st()), "ct_linear_fwd_ws")

                ms = timer(run, iters)
                flop = 2.0 * mm * nn * kk
                ach = flop / (ms * 1e-3) / 1e12
                mult = 3.0 if pname == "3xtf32" else 1.0
                rec = {"kernel": f"linear_{name}", "shape": f"[{mm},{kk}]x[{kk},{nn}]",
                       "precision": pname, "ms": ms, "achieved": ach, "unit": "TFLOP/s",
                       "algorithmic_flop": flop}
                if pname != "fp32":
                    rec.update(bound="tensor", peak=tf32_peak, frac=ach / tf32_peak,
                               frac_of_issued_mma=ach * mult / tf32_peak,
                               peak_source=f"{pk['source']} bf16 {pk['bf16_tflops']} / 2")
                out.append(rec)
    return out


def hbm_record(name, shape, ms, nbytes, pk):
    ach = nbytes / (ms * 1e-3) / 1e9
    return {"kernel": name, "shape": shape, "ms": ms, "achieved": ach, "unit": "GB/s",
            "bound": "hbm", "peak": pk["hbm_gbs"], "frac": ach / pk["hbm_gbs"],
            "algorithmic_bytes": nbytes, "peak_source": pk["source"] + " copy bandwidth"}


def row_cases(dev, timer, iters, pk, only, ln_n=384):
    L = lib()
    g = torch.Generator(device=dev).manual_seed(1)
    out = []
    if "softmax" in only:
        rows, n = 16384, 4096
        x = torch.randn(rows, n, device=dev, generator=g)
        y, dx = torch.empty_like(x), torch.empty_like(x)
        dp = torch.randn(rows, n, device=dev, generator=g)
        ms = timer(lambda: check(L.ct_softmax_fwd(_p(x), _p(y), rows, n, _st())), iters)
        out.append(hbm_record("softmax_fwd", f"[{rows},{n}]", ms, 2 * rows * n * 4, pk))
        ms = timer(lambda: check(L.ct_softmax_bwd(_p(y), _p(dp), _p(dx), rows, n, _st())), iters)
        out.append(hbm_record("softmax_bwd", f"[{rows},{n}]", ms, 3 * rows * n * 4, pk))
        del x, y, dx, dp
    if "layernorm" in only:
        rows, n = 16384, ln_n
        x = torch.randn(rows, n, device=dev, generator=g)
        gam, bet = torch.ones(n, device=dev), torch.zeros(n, device=dev)
        y, dx = torch.empty_like(x), torch.empty_like(x)
        mean, rstd = torch.empty(rows, device=dev), torch.empty(rows, device=dev)
        dy = torch.randn(rows, n, device=dev, generator=g)
        dg, db = torch.empty(n, device=dev), torch.empty(n, device=dev)
        wsb = L.ct_layernorm_bwd_workspace_size(rows, n)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
        ms = timer(lambda: check(L.ct_layernorm_fwd(_p(x), _p(gam), _p(bet), _p(y), _p(mean),
                                                    _p(rstd), rows, n, 1e-5, _st())), iters)
        out.append(hbm_record("layernorm_fwd", f"[{rows},{n}]", ms, 2 * rows * n * 4, pk))
        ms = timer(lambda: check(L.ct_layernorm_bwd(_p(x), _p(gam), _p(mean), _p(rstd), _p(dy),
                                                    _p(dx), _p(dg), _p(db), rows, n, _p(ws), wsb,
                                                    _st())), iters)
        out.append(hbm_record("layernorm_bwd", f"[{rows},{n}]", ms, 3 * rows * n * 4, pk))
    if "gelu" in only:
        numel = 16384 * 1536
        x = torch.randn(numel, device=dev, generator=g)
        dy = torch.randn(numel, device=dev, generator=g)
        y, dx = torch.empty_like(x), torch.empty_like(x)
        ms = timer(lambda: check(L.ct_gelu_fwd(_p(x), _p(y), numel, _st())), iters)
        out.append(hbm_record("gelu_fwd", "[16384,1536]", ms, 2 * numel * 4, pk))
        ms = timer(lambda: check(L.ct_gelu_bwd(_p(x), _p(dy), _p(dx), numel, _st())), iters)
        out.append(hbm_record("gelu_bwd", "[16384,1536]", ms, 3 * numel * 4, pk))
    if "bias_grad" in only:
        m, n = 16384, 1536
        dy = torch.randn(1, m, n, device=dev, generator=g)
        db = torch.empty(n, device=dev)
        wsb = L.ct_bias_grad_workspace_size(1, m, n)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
        ms = timer(lambda: check(L.ct_bias_grad(_p(dy), _s3(dy), _p(db), 1, m, n, _p(ws), wsb,
                                                _st())), iters)
        out.append(hbm_record("bias_grad", f"[{m},{n}]", ms, m * n * 4, pk))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default="linear,softmax,layernorm,gelu,bias_grad")
    ap.add_argument("--precisions", default="3xtf32,tf32,fp32")
    ap.add_argument("--ln-cols", type=int, default=384, help="LayerNorm row width (<= 8192)")
    a = ap.parse_args()
    only = set(a.only.split(","))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pk = peaks()
    timer = Timer(dev)
    recs = []
    if "linear" in only:
        recs += linear_cases(dev, timer, a.iters, pk, a.precisions.split(","))
    recs += row_cases(dev, timer, a.iters, pk, only, a.ln_cols)
    for r in recs:
        print(json.dumps(r))
    assert device_status(0, clear=True) == 0, "device watchdog raised"


if __name__ == "__main__":
    main()
