"""Measure the FP32 FMA throughput of the current GPU (FFMA2 and FFMA).

    python -m holysht_b200.tools.fp32_peak

The result is the FP32 denominator of the roofline for the FMA-bound
Legendre kernels (the driver's MEASURED_PEAKS.json records HBM and bf16
tensor peaks only).
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

LIB = Path(__file__).resolve().parents[1] / "libholysht_b200_probe.so"


def measure(iters: int = 20000) -> dict:
    lib = ctypes.CDLL(str(LIB))
    fn = lib.holysht_probe_fp32_flops
    fn.restype = ctypes.c_double
    fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    import torch

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    res = {}
    for packed, name in ((1, "ffma2"), (0, "ffma")):
        best = 0.0
        for blocks_per_sm in (4, 8):
            best = max(best, fn(packed, sms * blocks_per_sm, 256, iters))
        res[f"{name}_tflops"] = round(best / 1e12, 2)
    res["sms"] = sms
    return res


if __name__ == "__main__":
    print(json.dumps(measure()))
