"""Achievable read bandwidth of the streaming kernel's access pattern.

    python -m holysht_b200.tools.bulk_stream_probe

Streams the byte count of the benchmark's table pair (1152 warps x 512 KiB)
with the streaming kernel's grid shapes: every warp copies its own contiguous
run into a shared-memory ring with cp.async.bulk and reads it once, nothing
else.  The result is the ceiling a table-streaming Legendre kernel of that
shape can reach on this GPU (compare the measured copy peak of
MEASURED_PEAKS.json).  Prints one JSON object per configuration.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

LIB = Path(__file__).resolve().parents[1] / "libholysht_b200_probe.so"


def main() -> None:
    import torch

    lib = ctypes.CDLL(str(LIB))
    fn = lib.holysht_probe_bulk_stream
    fn.restype = ctypes.c_double
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p]
    nbytes = 1152 * 512 * 1024
    src = torch.full((nbytes // 4,), 0.5, dtype=torch.float32, device="cuda")
    sink = torch.zeros(1, dtype=torch.float32, device="cuda")
    for ctas, cluster in ((144, 1), (144, 2), (148, 1), (136, 1)):
        for stages, kb in ((4, 4), (3, 8), (2, 8), (3, 4)):
            gbs = fn(src.data_ptr(), nbytes, ctas, cluster, stages, kb, 10, sink.data_ptr())
            print(json.dumps({"ctas": ctas, "cluster": cluster, "stages": stages, "stage_kb": kb,
                              "bytes": nbytes, "gb_per_s": round(gbs, 1)}), flush=True)


if __name__ == "__main__":
    main()
