"""Run the recurrence-variant forward (512x1024, batch 4) for profilers.

    python -m holysht_b200.tools.profile_recurrence [reps] [vector|inverse]

RealSHT(variant="recurrence") by default, RealVectorSHT(variant="recurrence")
with ``vector``, InverseRealSHT(variant="recurrence") on a (4, 512, 513)
spectrum with ``inverse``.
"""
from __future__ import annotations

import sys

import torch

import holysht_b200 as hs


def main(argv):
    reps = int(argv[1]) if len(argv) > 1 else 3
    vector = "vector" in argv
    inverse = "inverse" in argv
    dev = torch.device("cuda")
    if inverse:
        m = hs.InverseRealSHT(512, 1024, variant="recurrence").to(dev)
        x = torch.randn(4, 512, 513, dtype=torch.complex64, device=dev)
    elif vector:
        m = hs.RealVectorSHT(512, 1024, variant="recurrence").to(dev)
        x = torch.randn(4, 2, 512, 1024, device=dev)
    else:
        m = hs.RealSHT(512, 1024, variant="recurrence").to(dev)
        x = torch.randn(4, 512, 1024, device=dev)
    with torch.no_grad():
        for _ in range(reps):
            m(x)
        torch.cuda.synchronize()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        e[0].record()
        for _ in range(10):
            m(x)
        e[1].record()
        torch.cuda.synchronize()
    name = "InverseRealSHT" if inverse else "RealVectorSHT" if vector else "RealSHT"
    print("recurrence", name, "512x1024 b4 ms",
          round(e[0].elapsed_time(e[1]) / 10, 4))


if __name__ == "__main__":
    main(sys.argv)
