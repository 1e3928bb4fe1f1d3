"""Run the dense tensor-core RealSHT forward for profilers.

    python -m holysht_b200.tools.profile_dense [nlat] [batch] [reps]

RealSHT(nlat, 2*nlat) on cuda:0 over a (batch, nlat, 2*nlat) input with the
tcgen05 path forced; ``reps`` forwards, then the mean of 3 timed forwards.
"""
from __future__ import annotations

import os
import sys

import torch

import holysht_b200 as hs


def main(argv):
    nlat = int(argv[1]) if len(argv) > 1 else 1024
    batch = int(argv[2]) if len(argv) > 2 else 256
    reps = int(argv[3]) if len(argv) > 3 else 2
    os.environ["HOLYSHT_DENSE_TC"] = "1"
    dev = torch.device("cuda")
    m = hs.RealSHT(nlat, 2 * nlat).to(dev)
    x = torch.randn(batch, nlat, 2 * nlat, device=dev)
    with torch.no_grad():
        for _ in range(reps):
            m(x)
        torch.cuda.synchronize()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        e[0].record()
        for _ in range(3):
            m(x)
        e[1].record()
        torch.cuda.synchronize()
    print("dense RealSHT", nlat, batch, "ms", round(e[0].elapsed_time(e[1]) / 3, 4))


if __name__ == "__main__":
    main(sys.argv)
