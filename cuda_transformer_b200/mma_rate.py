"""Measures the tcgen05 kind::tf32 tensor-pipe rate (M = 128) on every SM
through ct_diag_mma_rate and prints cycles per MMA and FLOP per cycle per SM
for each N and A-operand source, plus the chip rate at the SM clock seen.

  python -m cuda_transformer_b200.mma_rate [--reps 2000]
"""
from __future__ import annotations

import argparse
import ctypes
import json

import torch

from . import check, lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=2000)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    clk_mhz = None
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(0)
        clk_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
    except Exception:
        pass
    cyc = torch.zeros(sms, dtype=torch.int64, device=dev)
    L = lib()
    for n in (32, 64, 128, 256):
        for ts in (1, 0):
            st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            check(L.ct_diag_mma_rate(n, ts, a.reps, sms, ctypes.c_void_p(cyc.data_ptr()), st),
                  "ct_diag_mma_rate")
            torch.cuda.synchronize()
            c = cyc.double()
            assert bool((c > 0).all()), "completion wait timed out"
            per = float(c.mean()) / (a.reps * 4)
            fpc = 2.0 * 128 * n * 8 / per
            rec = {"N": n, "a": "tmem" if ts else "smem", "cycles_per_mma": per,
                   "flop_per_cycle_per_sm": fpc, "sms": sms}
            if clk_mhz:
                rec["chip_tflops_at_max_clock"] = fpc * sms * clk_mhz * 1e6 / 1e12
                rec["max_sm_mhz"] = clk_mhz
            print(json.dumps(rec))


if __name__ == "__main__":
    main()
