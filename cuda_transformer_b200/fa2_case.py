"""Runs FlashAttention-2 forward + backward steps through the C ABI on one GPU
and prints per-kernel device times (CUDA events) -- a quick timing tool, and
the workload the committed Nsight Compute summaries were captured on.

  python -m cuda_transformer_b200.fa2_case [--B 4 --H 32 --N 4096 --D 64]
        [--causal 1] [--precision 3xtf32|tf32|fp32] [--steps 2] [--warmup 1]
"""
from __future__ import annotations

import argparse
import ctypes
import json

import torch

from . import PRECISION_3XTF32, PRECISION_FP32, PRECISION_TF32, check, device_status, lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=4)
    ap.add_argument("--H", type=int, default=32)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--D", type=int, default=64)
    ap.add_argument("--causal", type=int, default=1)
    ap.add_argument("--precision", default="3xtf32", choices=["3xtf32", "tf32", "fp32"])
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    a = ap.parse_args()
    prec = {"3xtf32": PRECISION_3XTF32, "tf32": PRECISION_TF32, "fp32": PRECISION_FP32}[a.precision]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    shape = (a.B, a.H, a.N, a.D)
    q, k, v, do = (torch.randn(shape, device=dev, generator=g) for _ in range(4))
    o, dq, dk, dv = (torch.empty(shape, device=dev) for _ in range(4))
    lse = torch.empty(a.B, a.H, a.N, device=dev)
    delta = torch.empty(a.B, a.H, a.N, device=dev)
    L = lib()
    s4 = (ctypes.c_int64 * 4)(*q.stride())
    s3 = (ctypes.c_int64 * 3)(*lse.stride())
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    st = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    dims = (a.B, a.H, a.N, a.D)

    def fwd():
        check(L.ct_fa2_fwd(P(q), s4, P(k), s4, P(v), s4, P(o), P(lse), *dims, a.causal, prec, st()))

    def bdelta():
        check(L.ct_fa2_bwd_delta(P(o), s4, P(do), s4, P(delta), *dims, st()))

    def bdq():
        check(L.ct_fa2_bwd_dq(P(q), s4, P(k), s4, P(v), s4, P(do), s4, P(lse), s3, P(delta),
                              P(dq), *dims, a.causal, prec, st()))

    def bdkdv():
        check(L.ct_fa2_bwd_dkdv(P(q), s4, P(k), s4, P(v), s4, P(do), s4, P(lse), s3, P(delta),
                                P(dk), P(dv), *dims, a.causal, prec, st()))

    kernels = [("fa2_fwd", fwd), ("fa2_bwd_delta", bdelta), ("fa2_bwd_dq", bdq),
               ("fa2_bwd_dkdv", bdkdv)]
    for _ in range(a.warmup):
        for _, fn in kernels:
            fn()
    torch.cuda.synchronize()
    times = {n: 0.0 for n, _ in kernels}
    for _ in range(a.steps):
        for n, fn in kernels:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            times[n] += e0.elapsed_time(e1) / a.steps
    assert device_status(0, clear=True) == 0, "device watchdog raised"
    fl = 4.0 * a.B * a.H * a.N * a.N * a.D * (0.5 if a.causal else 1.0)
    total = sum(times.values())
    print(json.dumps({"case": vars(a), "kernel_ms": times, "fwd_bwd_ms": total,
                      "tflops_fwd_bwd": 3.5 * fl / (total * 1e-3) / 1e12}))


if __name__ == "__main__":
    main()
