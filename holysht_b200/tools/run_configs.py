"""Time the five BASELINE.json configurations on cuda:0 (device time, CUDA events).

    python -m holysht_b200.tools.run_configs [c1 c2 c3 c4 c5s c5v]

C1  RealSHT.forward 256x512 equiangular, x (4, 256, 512)
C2  RealVectorSHT.forward 256x512, band-limited (4, 2, 256, 512)
C3  RealSHT(dtype="bf16").forward 512x1024 Legendre-Gauss, x (4, 16, 512, 1024) bf16-rounded
C4  training round trip 512x1024: InverseRealSHT -> tanh -> RealSHT -> sum|c|^2 -> backward,
    spectral (8, 32, 512, 513); and the vector variant with 2 components
C5  RealSHT.forward 1024x2048 on (16, 64, 1024, 2048); RealVectorSHT on (16, 2, 1024, 2048)
Prints one JSON line per configuration.  Inputs are seeded synthetic data.
"""
from __future__ import annotations

import json
import sys

import torch

import holysht_b200 as hs


def _time(fn, reps=5, warm=2):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def c1(dev):
    g = torch.Generator(device=dev).manual_seed(0)
    m = hs.RealSHT(256, 512).to(dev)
    x = torch.randn(4, 256, 512, device=dev, generator=g)
    with torch.no_grad():
        return {"config": "C1 RealSHT.forward 256x512 b4", "ms": _time(lambda: m(x), 50, 5)}


def c2(dev):
    g = torch.Generator(device=dev).manual_seed(1)
    L, M = 256, 257
    scale = (torch.arange(L, device=dev, dtype=torch.float32) + 1.0) ** -1.5
    tri = (torch.arange(M, device=dev)[None, :] <= torch.arange(L, device=dev)[:, None])
    c = torch.complex(torch.randn(4, 2, L, M, device=dev, generator=g), torch.randn(4, 2, L, M, device=dev, generator=g))
    c = c * scale[:, None] * tri
    x = hs.InverseRealVectorSHT(256, 512).to(dev)(c)
    m = hs.RealVectorSHT(256, 512).to(dev)
    with torch.no_grad():
        return {"config": "C2 RealVectorSHT.forward 256x512 b4 band-limited", "ms": _time(lambda: m(x), 50, 5)}


def c3(dev):
    g = torch.Generator(device=dev).manual_seed(2)
    m = hs.RealSHT(512, 1024, grid="legendre-gauss", dtype="bf16").to(dev)
    x = torch.randn(4, 16, 512, 1024, device=dev, generator=g).bfloat16().float()
    with torch.no_grad():
        return {"config": "C3 RealSHT(bf16).forward 512x1024 LG (4,16)", "ms": _time(lambda: m(x), 20, 3)}


def c4(dev):
    g = torch.Generator(device=dev).manual_seed(3)
    L, M = 512, 513
    scale = (torch.arange(L, device=dev, dtype=torch.float32) + 1.0) ** -2
    tri = (torch.arange(M, device=dev)[None, :] <= torch.arange(L, device=dev)[:, None])
    out = []
    for vector in (False, True):
        shape = (8, 32, L, M) if not vector else (8, 2, L, M)
        c0 = torch.complex(torch.randn(shape, device=dev, generator=g), torch.randn(shape, device=dev, generator=g))
        c0 = c0 * scale[:, None] * tri
        inv = (hs.InverseRealVectorSHT if vector else hs.InverseRealSHT)(512, 1024).to(dev)
        fwd = (hs.RealVectorSHT if vector else hs.RealSHT)(512, 1024).to(dev)

        def step():
            c = c0.clone().requires_grad_(True)
            coef = fwd(torch.tanh(inv(c)))
            (coef.real.square().sum() + coef.imag.square().sum()).backward()
            return c.grad

        out.append({"config": f"C4 training round trip 512x1024 {'vector (8,2)' if vector else 'scalar (8,32)'}",
                    "ms": _time(step, 5, 2)})
    return out


def c5s(dev):
    g = torch.Generator(device=dev).manual_seed(4)
    m = hs.RealSHT(1024, 2048).to(dev)
    x = torch.randn(16, 64, 1024, 2048, device=dev, generator=g)
    with torch.no_grad():
        return {"config": "C5 RealSHT.forward 1024x2048 (16,64) [tcgen05 dense]", "ms": _time(lambda: m(x), 3, 1)}


def c5v(dev):
    g = torch.Generator(device=dev).manual_seed(4)
    m = hs.RealVectorSHT(1024, 2048).to(dev)
    x = torch.randn(16, 2, 1024, 2048, device=dev, generator=g)
    with torch.no_grad():
        return {"config": "C5 RealVectorSHT.forward 1024x2048 (16,2)", "ms": _time(lambda: m(x), 5, 2)}


def main(argv):
    dev = torch.device("cuda")
    which = argv[1:] or ["c1", "c2", "c3", "c4", "c5s", "c5v"]
    for name in which:
        res = globals()[name](dev)
        for r in res if isinstance(res, list) else [res]:
            r["ms"] = round(r["ms"], 4)
            print(json.dumps(r), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main(sys.argv)
