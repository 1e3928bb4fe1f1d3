"""Run one Legendre contraction of the module paths at the benchmark size, for
profilers (ncu -k regex:contract_kernel) and quick timing.

    python -m holysht_b200.tools.profile_case {vector|scalar} [reps] [ksplit] [grouped|grouped8|parity|strided] [inv]

Builds RealVectorSHT/RealSHT(512, 1024) on cuda:0, runs ``reps`` warm-up
launches of the forward (or, with ``inv``, the inverse-direction) contraction
on a batch of 4, then times 10 launches with CUDA events and prints the mean.
"""
from __future__ import annotations

import math
import sys

import torch

import holysht_b200 as hs
from holysht_b200 import _lib
from holysht_b200.ops import legendre_contract


def main(argv):
    kind = argv[1] if len(argv) > 1 else "vector"
    reps = int(argv[2]) if len(argv) > 2 else 3
    ks = int(argv[3]) if len(argv) > 3 else 0
    layout = argv[4] if len(argv) > 4 else "grouped"
    direction = _lib.DIR_INVERSE if "inv" in argv else _lib.DIR_FORWARD
    dev = torch.device("cuda")
    NLAT, NLON, B = 512, 1024, 4
    if kind == "vector":
        m = hs.RealVectorSHT(NLAT, NLON).to(dev)
        P, K_, dense = 2, _lib.KIND_VECTOR, (m.w0_t, m.w1_t)
    else:
        m = hs.RealSHT(NLAT, NLON).to(dev)
        P, K_, dense = 1, _lib.KIND_SCALAR, (m.weight_t, None)
    L, M = m.lmax, m.mmax
    if direction == _lib.DIR_FORWARD:
        x = torch.randn((B, P, NLAT, NLON), device=dev)
        inp = torch.fft.rfft(x, dim=-1)
        Rin, W = NLAT, inp.size(-1)
        out = torch.empty((B, P, L, M), dtype=torch.complex64, device=dev)
        Rout, ocols = L, M
    else:
        inp = torch.randn((B, P, L, M), dtype=torch.complex64, device=dev)
        Rin, W = L, M
        out = torch.empty((B, P, NLAT, NLON // 2 + 1), dtype=torch.complex64, device=dev)
        Rout, ocols = NLAT, NLON // 2 + 1
    grouped8 = layout in ("grouped8", "parity")
    parity = layout == "parity"
    if parity:
        w0, w1, grouped = m.table(direction, "parity")[0], None, False
    elif layout == "grouped":
        w0, w1, grouped = m.table(direction, "grouped")[0], None, True
    elif layout == "grouped8":
        from holysht_b200.ops import group_table8
        tabs = dense if kind == "vector" else dense[0]
        w0, w1, grouped = group_table8(tabs, direction, conj=(kind == "vector" and direction == _lib.DIR_INVERSE)), None, False
    else:
        w0, w1, grouped = dense[0], dense[1], False

    def launch():
        legendre_contract(kind=K_, direction=direction, input=inp, output=out, w0=w0, w1=w1,
                          batch=B, nlat=NLAT, lmax=L, mmax=M,
                          in_strides=(P * Rin * W, Rin * W, W), out_strides=(P * Rout * ocols, Rout * ocols, ocols),
                          out_cols=ocols, scale=2 * math.pi / NLON, ksplit=ks, grouped=grouped,
                          grouped8=grouped8, parity=parity)

    for _ in range(reps):
        launch()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(10):
        launch()
    ev[1].record()
    torch.cuda.synchronize()
    print(kind, layout, "inv" if direction else "fwd", "ks", ks, "avg ms",
          round(ev[0].elapsed_time(ev[1]) / 10, 5))


if __name__ == "__main__":
    main(sys.argv)
