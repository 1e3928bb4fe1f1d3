"""Time the reference's own CUDA path on this GPU (the bar the sm_100a kernels must beat).

    python baseline/reference_cuda.py [--steps K] [--warmup W] [--nlat 512 --nlon 1024 --batch 4]

Runs the unmodified reference package staged in ``baseline/_ref`` by
``baseline/prepare_reference.py`` (its CUDA extension prebuilt for sm_100a),
through its public modules ``RealVectorSHT`` / ``RealSHT``
(``torch-ext/holysht/__init__.py:1228-1389``, :1430-1693), once with automatic
backend selection (the reference autotunes on the first call; its cache goes
to a fresh temporary file) and once with ``HOLYSHT_FORCE_BACKEND=tma``.

The reference's constructors call torch-harmonics, which is not installed on
either machine; a stand-in ``torch_harmonics`` hands them the tables of
``holysht_b200.weights`` (the same float64-built tables this project's
modules use), so both implementations contract identical tables.

Timing matches ``bench.py``: inputs resident on the GPU, the L2 flushed
(256 MiB write, then 256 MiB read) before every timed step, CUDA events around
the forward only, median over the steps.  Each result is also checked in
float64 against the same tables on a few orders of one slice.  Prints one JSON
line.  One GPU only; run it in its own process (it loads the reference's
extension library).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
REF_PKG = HERE / "_ref" / "torch-ext"


def _import_reference():
    if not (REF_PKG / "holysht" / "_ops.py").exists():
        raise RuntimeError("baseline/_ref is not prepared (run baseline/prepare_reference.py here first)")
    sys.path.insert(0, str(ROOT))
    from baseline.reference_cpu import stand_in_torch_harmonics

    sys.modules["torch_harmonics"] = stand_in_torch_harmonics()
    sys.path.insert(0, str(REF_PKG))
    import holysht  # the reference package

    if not holysht._HAS_NATIVE_EXT:
        raise RuntimeError("the reference's CUDA extension did not load")
    return holysht


def _time(fn, steps, warmup, dev):
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.zeros((), dtype=torch.float32, device=dev)
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(steps):
        flush_w.fill_(1)
        sink += flush_r.sum()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize(dev)
        times.append(s.elapsed_time(e))
    return float(np.median(times)), float(np.min(times))


def _parity(out, x, tables, vector, M):
    """float64 check of slice 0 on a few orders (relative L2 over them)."""
    xs = x[0].double().cpu().numpy()
    X = 2 * np.pi * np.fft.rfft(xs, axis=-1, norm="forward")[..., :M]
    ms = [0, 1, M // 2, M - 1]
    got, ref = [], []
    for m in ms:
        if vector:
            w0 = tables[0][m].astype(np.float64).T
            w1 = tables[1][m].astype(np.float64).T
            c0, c1 = X[0, :, m], X[1, :, m]
            ref.append(np.stack([c0 @ w0 + 1j * (c1 @ w1), 1j * (c0 @ w1) - c1 @ w0]))
            got.append(out[0, :, :, m].cpu().numpy())
        else:
            ref.append(X[:, m] @ tables[m].astype(np.float64).T)
            got.append(out[0, :, m].cpu().numpy())
    got, ref = np.asarray(got), np.asarray(ref)
    return float(np.linalg.norm(got - ref) / np.linalg.norm(ref))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--nlat", type=int, default=512)
    ap.add_argument("--nlon", type=int, default=1024)
    ap.add_argument("--batch", type=int, default=4)
    args = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    os.environ["HOLYSHT_AUTOTUNE_CACHE_PATH"] = str(Path(tempfile.mkdtemp(prefix="holysht_tune_")) / "cache.json")
    hs = _import_reference()
    res = {"impl": "reference-cuda", "gpu": torch.cuda.get_device_name(dev),
           "workload": f"{args.nlat}x{args.nlon} equiangular b{args.batch} fp32",
           "steps": args.steps, "warmup": args.warmup, "statistic": "median (min) of CUDA-event ms, L2 flushed"}
    g = torch.Generator(device=dev).manual_seed(1)
    xv = torch.randn(args.batch, 2, args.nlat, args.nlon, device=dev, generator=g)
    xs = torch.randn(args.batch, args.nlat, args.nlon, device=dev, generator=g)
    for backend in ("auto", "tma"):
        os.environ["HOLYSHT_FORCE_BACKEND"] = "" if backend == "auto" else backend
        for name, cls, x, vector in (("RealVectorSHT", hs.RealVectorSHT, xv, True), ("RealSHT", hs.RealSHT, xs, False)):
            mod = cls(args.nlat, args.nlon).to(dev)
            with torch.no_grad():
                med, mn = _time(lambda: mod(x), args.steps, args.warmup, dev)
                out = mod(x)
            tabs = (mod.w0.cpu().numpy(), mod.w1.cpu().numpy()) if vector else mod.weights.cpu().numpy()
            res[f"{name}.forward_ms[{backend}]"] = round(med, 4)
            res[f"{name}.forward_min_ms[{backend}]"] = round(mn, 4)
            res[f"{name}.rel_l2_vs_float64[{backend}]"] = _parity(out, x, tabs, vector, mod.mmax)
            del mod, out
            torch.cuda.empty_cache()
    os.environ.pop("HOLYSHT_FORCE_BACKEND", None)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
