"""TEST-ONLY probe.  Measures the tcgen05 kind::tf32 tensor-pipe rate (M = 128)
on every SM through ct_diag_mma_rate (tests/diag/libct_diag.so) and prints cycles per MMA and FLOP per cycle per SM
for each N, A-operand source, B-operand layout and number of issuing threads,
plus the chip rate at the maximum SM clock.

  python -m tests.diag.mma_rate [--reps 2000]

With two issuing threads the cycles per MMA count the MMAs of both, i.e. the
SM's combined rate.
"""
from __future__ import annotations

import argparse
import ctypes
import json

import torch

from tests.diag import check, lib


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
        for two in (0, 1):
            if two and n > 128:
                continue
            for bmn in (0, 1):
                for ts in (1, 0):
                    flags = ts | (bmn << 1) | (two << 2)
                    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
                    check(L.ct_diag_mma_rate(n, flags, a.reps, sms,
                                             ctypes.c_void_p(cyc.data_ptr()), st),
                          "ct_diag_mma_rate")
                    torch.cuda.synchronize()
                    c = cyc.double()
                    assert bool((c > 0).all()), "completion wait timed out"
                    per = float(c.mean()) / (a.reps * 4 * (2 if two else 1))
                    fpc = 2.0 * 128 * n * 8 / per
                    rec = {"N": n, "a": "tmem" if ts else "smem",
                           "b": "mn_major" if bmn else "k_major", "issuers": 2 if two else 1,
                           "cycles_per_mma": per, "flop_per_cycle_per_sm": fpc, "sms": sms}
                    if clk_mhz:
                        rec["chip_tflops_at_max_clock"] = fpc * sms * clk_mhz * 1e6 / 1e12
                        rec["max_sm_mhz"] = clk_mhz
                    print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
