"""Benchmark: RealVectorSHT.forward at 512 x 1024, batch 4, FP32 (the
reference's headline metric, README.md:79), on N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--skip-c5]

One step = one RealVectorSHT.forward (rfft on cuFFT + the fused vector
Legendre kernel) over a (4, 2, 512, 1024) float32 batch resident in HBM.
Multi-GPU: batch partition with no collective (every rank transforms its own
batch of 4, weak scaling); the timing is device time (CUDA events), the max
over ranks.  The L2 is flushed (256 MiB write, then 256 MiB read) before
every timed step.  Secondary fields: the scalar and inverse forwards (scalar and
vector), the recurrence variants (scalar and vector forward, scalar inverse),
the 1024 x 2048 configuration under both multi-GPU partitions, and
(N = 1) the reference's own CUDA path timed in a child process.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's
own CPU forward (imported unmodified from ``baseline/_ref``; the oracle's
restatement when that is absent) on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

NLAT, NLON, BATCH = 512, 1024, 4
METRIC = "RealVectorSHT.forward ms @512x1024 b4 fp32"
UNIT = "ms"
PUBLISHED_GB10_MS = 6.855  # the published HOLYSHT RealVectorSHT.forward 512x1024 b4 time on GB10
# committed ncu summaries of the vector kernel, per table layout of the module's forward
PROFILES = {"parity": ROOT / "profiles" / "stream_vector_parity_fwd_512x1024_b4.md",
            "grouped8": ROOT / "profiles" / "stream_vector_fwd_512x1024_b4.md"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-c5", action="store_true", help="skip the 1024x2048 secondary measurements")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples (100 ms) of SM clock and throttle reasons."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for t, line in self.samples:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            rows.append((t, parts))
        inside = [p for t, p in rows if self.t0 is not None and self.t0 - 0.15 <= t <= self.t1 + 0.15]
        use = inside or rows
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(p[1]) for p in use if p[1].replace(".", "").isdigit()]
        smax = [float(p[2]) for p in use if p[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for p in use for n, v in zip(names, p[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(use), "in_timed_region": bool(inside)}


# ------------------------------------------------------------------ ours

def _traffic_from_profile(layout):
    """DRAM bytes per launch of the vector kernel from the committed ncu summary
    of the table layout the module uses."""
    try:
        m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", PROFILES[layout].read_text())
        return float(m.group(1)) if m else None
    except (OSError, KeyError):
        return None


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def algorithmic_bytes(L, K, M, B, tables, table_rows=None):
    """Bytes one forward Legendre launch must move: the l >= m triangle of each
    table (fp32) over ``table_rows`` latitudes (K, or ceil(K/2) when the kernel
    folds the southern half by equatorial parity), the spectrum read
    (complex64, orders < M, all K rows) and the output."""
    pairs = sum(max(L - m, 0) for m in range(M))
    rows = K if table_rows is None else table_rows
    return tables * pairs * rows * 4 + B * tables * K * M * 8 + B * tables * L * M * 8


def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist

    import holysht_b200 as hs
    from holysht_b200 import _lib
    from holysht_b200.ops import legendre_contract

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    vsht = hs.RealVectorSHT(NLAT, NLON, table_device=dev)
    L, M = vsht.lmax, vsht.mmax
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    x = torch.randn((BATCH, 2, NLAT, NLON), generator=gen, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    clean = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush_l2():
        # write a buffer larger than L2 (evicts every line the step could reuse),
        # then read another one, so the written lines are not left dirty in L2
        # for the timed step to write back
        flush.zero_()
        torch.sum(clean, dim=0, out=sink)
    stream = torch.cuda.current_stream(dev)

    for _ in range(max(args.warmup, 3)):
        vsht(x)
    torch.cuda.synchronize(dev)

    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    clocks = ClockSampler(visible[local_rank].strip() if local_rank < len(visible) else local_rank)
    clocks.start()
    time.sleep(0.3)
    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    barrier()
    torch.cuda.synchronize(dev)
    clocks.mark("t0")
    for i in range(K):
        flush_l2()
        starts[i].record(stream)
        vsht(x)
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks.mark("t1")
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = max_over_ranks(sum(step_ms) / K)
    launches_per_step = 1  # one holysht_b200 kernel per RealVectorSHT.forward

    # ---- the dominant kernel alone (roofline): the module's own call ----
    spec = torch.fft.rfft(x, dim=-1)
    out = torch.empty((BATCH, 2, L, M), dtype=torch.complex64, device=dev)
    W = spec.size(-1)
    table, _, layout = vsht.table(_lib.DIR_FORWARD)  # the layout the module's forward uses

    def kernel():
        legendre_contract(kind=_lib.KIND_VECTOR, direction=_lib.DIR_FORWARD, input=spec, output=out,
                          w0=table, batch=BATCH, nlat=NLAT, lmax=L, mmax=M,
                          in_strides=(2 * NLAT * W, NLAT * W, W), out_strides=(2 * L * M, L * M, M),
                          out_cols=M, scale=2 * math.pi / NLON, grouped=layout == "grouped",
                          grouped8=layout in ("grouped8", "parity"), parity=layout == "parity")

    for _ in range(3):
        kernel()
    kn = max(20, K // 2)
    ks = [torch.cuda.Event(enable_timing=True) for _ in range(kn)]
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(kn)]
    for i in range(kn):
        flush_l2()
        ks[i].record(stream)
        kernel()
        ke[i].record(stream)
    torch.cuda.synchronize(dev)
    kernel_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(ks, ke))
    kernel_ms = max_over_ranks(kernel_ms)
    # algorithmic bytes as the scope table defines them (both tables' full l >= m
    # triangle, spectrum, output); the folded layout needs only the northern rows
    abytes = algorithmic_bytes(L, NLAT, M, BATCH, 2)
    fbytes = algorithmic_bytes(L, NLAT, M, BATCH, 2, (NLAT + 1) // 2) if layout == "parity" else abytes
    clocks.stop()

    # ---- secondary: RealSHT.forward on the same grid ----
    ssht = hs.RealSHT(NLAT, NLON, table_device=dev)
    xs = torch.randn((BATCH, NLAT, NLON), generator=gen, device=dev)
    for _ in range(3):
        ssht(xs)
    sn = max(20, K // 2)
    ss = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    se = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    for i in range(sn):
        flush_l2()
        ss[i].record(stream)
        ssht(xs)
        se[i].record(stream)
    torch.cuda.synchronize(dev)
    scalar_ms = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in zip(ss, se)))
    del ssht
    # the on-the-fly (recurrence) variant of the same scalar forward
    rsht = hs.RealSHT(NLAT, NLON, variant="recurrence").to(dev)
    for _ in range(3):
        rsht(xs)
    rs = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    re_ = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    for i in range(sn):
        flush_l2()
        rs[i].record(stream)
        rsht(xs)
        re_[i].record(stream)
    torch.cuda.synchronize(dev)
    rec_ms = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in zip(rs, re_)))
    del rsht
    # the on-the-fly (recurrence) variant of the vector forward
    vrsht = hs.RealVectorSHT(NLAT, NLON, variant="recurrence").to(dev)
    for _ in range(3):
        vrsht(x)
    vs_ = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    ve = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    for i in range(sn):
        flush_l2()
        vs_[i].record(stream)
        vrsht(x)
        ve[i].record(stream)
    torch.cuda.synchronize(dev)
    vrec_ms = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in zip(vs_, ve)))
    del vrsht
    # the inverse direction (InverseRealVectorSHT.forward, irfft included) on the same grid
    isht = hs.InverseRealVectorSHT(NLAT, NLON, table_device=dev)
    coef = vsht(x)
    for _ in range(3):
        isht(coef)
    is_ = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    ie = [torch.cuda.Event(enable_timing=True) for _ in range(sn)]
    for i in range(sn):
        flush_l2()
        is_[i].record(stream)
        isht(coef)
        ie[i].record(stream)
    torch.cuda.synchronize(dev)
    inv_ms = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in zip(is_, ie)))
    del isht, coef

    def time_forward(mod, inp):
        for _ in range(3):
            mod(inp)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(sn)]
        for s, e in ev:
            flush_l2()
            s.record(stream)
            mod(inp)
            e.record(stream)
        torch.cuda.synchronize(dev)
        return max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in ev))

    # InverseRealSHT.forward (irfft included): the table path and the recurrence variant
    scoef = hs.RealSHT(NLAT, NLON, table_device=dev)(xs)
    sinv_ms = time_forward(hs.InverseRealSHT(NLAT, NLON, table_device=dev), scoef)
    sinv_rec_ms = time_forward(hs.InverseRealSHT(NLAT, NLON, variant="recurrence").to(dev), scoef)
    del scoef

    # ---- the 1024 x 2048 configuration on all ranks (both partitions) ----
    c5 = run_c5(rank, world, dev, barrier, max_over_ranks) if not args.skip_c5 else {}

    # ---- end to end through the public API with host buffers ----
    xh = torch.empty((BATCH, 2, NLAT, NLON), dtype=torch.float32).pin_memory()
    xh.copy_(x.cpu())
    oh = torch.empty((BATCH, 2, L, M), dtype=torch.complex64).pin_memory()
    xd = torch.empty_like(x)
    for _ in range(3):
        xd.copy_(xh, non_blocking=True)
        oh.copy_(vsht(xd), non_blocking=True)
    torch.cuda.synchronize(dev)
    en = max(10, K // 4)
    es = [torch.cuda.Event(enable_timing=True) for _ in range(en)]
    ee = [torch.cuda.Event(enable_timing=True) for _ in range(en)]
    barrier()
    for i in range(en):
        flush_l2()
        es[i].record(stream)
        xd.copy_(xh, non_blocking=True)
        oh.copy_(vsht(xd), non_blocking=True)
        ee[i].record(stream)
    torch.cuda.synchronize(dev)
    e2e_seq_ms = max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in zip(es, ee)))
    # the same K transforms through holysht_b200.pipeline.HostStream: upload of
    # batch i+1 and download of batch i-1 overlap the transform of batch i
    from holysht_b200.pipeline import HostStream

    ring = 4
    hin = [torch.empty_like(xh).pin_memory() for _ in range(ring)]
    for i, h in enumerate(hin):
        h.copy_(torch.randn((BATCH, 2, NLAT, NLON), generator=gen, device=dev).cpu())
    hout = [torch.empty_like(oh).pin_memory() for _ in range(K)]
    inputs = [hin[i % ring] for i in range(K)]
    pipe = HostStream(vsht, dev)
    pipe.run(inputs[:3], hout[:3])
    barrier()
    ps, pe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    ps.record(stream)
    pipe.run(inputs, hout)
    pe.record(stream)
    torch.cuda.synchronize(dev)
    e2e_local = ps.elapsed_time(pe) / K
    e2e_ms = max_over_ranks(e2e_local)
    e2e_ranks = [e2e_local]
    if world > 1:
        t = torch.zeros(world, device=dev, dtype=torch.float64)
        t[rank] = e2e_local
        dist.all_reduce(t)
        e2e_ranks = [round(v, 5) for v in t.tolist()]
    e2e_ok = bool(torch.allclose(hout[K - 1], vsht(hin[(K - 1) % ring].to(dev)).cpu()))
    h2d = xh.numel() * 4
    d2h = oh.numel() * 8

    peaks, peak_kind = _peaks()
    achieved = abytes / (kernel_ms * 1e-3) / 1e9
    pairs = sum(max(L - m, 0) for m in range(M))
    flops = 2 * 4 * pairs * NLAT * BATCH  # u/v form: 4 FMA per (l, k, batch)
    traffic = _traffic_from_profile(layout)

    cpu = ref_cuda = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(vsht, x)
        ref_cuda = reference_cuda_bar()

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": round(ms, 5),
        "unit": UNIT,
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": round(ms / PUBLISHED_GB10_MS, 5),
        "dtype": "f32",
        "data": "synthetic N(0,1), seed 1+rank",
        "config": {"workload": "RealVectorSHT.forward 512x1024 equiangular lmax=512 mmax=513 ortho csphase, batch 4",
                   "global_batch": BATCH * world, "parallelism": f"batch-partition x{world}, no collective",
                   "l2": "flushed before every timed step: 256 MiB write, then a 256 MiB read so no dirty lines remain; tables 2x538 MB exceed L2"},
        "transforms_per_s": round(BATCH * world / (ms * 1e-3), 2),
        "secondary": {"RealSHT.forward_ms": round(scalar_ms, 5),
                      "RealSHT.forward_recurrence_variant_ms": round(rec_ms, 5),
                      "RealVectorSHT.forward_recurrence_variant_ms": round(vrec_ms, 5),
                      "InverseRealVectorSHT.forward_ms": round(inv_ms, 5),
                      "InverseRealSHT.forward_ms": round(sinv_ms, 5),
                      "InverseRealSHT.forward_recurrence_variant_ms": round(sinv_rec_ms, 5), **c5},
        "e2e": {"value": round(e2e_ms, 5), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "how": (f"{K} steps through holysht_b200.pipeline.HostStream (pinned host in/out; upload, transform "
                        "and download of consecutive steps overlap on three streams), total / K"),
                "matches_device_result": e2e_ok, "sequential_ms": round(e2e_seq_ms, 5),
                "per_rank_ms": e2e_ranks},
        "gpu_launches": launches_per_step * K,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic, "algorithmic_bytes": abytes, "kernel_ms": round(kernel_ms, 5),
                     "folded": {"layout": layout, "min_bytes": fbytes,
                                "frac": round(fbytes / (kernel_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                                "note": ("bytes the parity-folded layout must move (northern table rows only); "
                                         "frac against them is the kernel's distance from its own HBM floor")},
                     "fp32_flops": flops,
                     "fp32_tflops_achieved": round(flops / (kernel_ms * 1e-3) / 1e12, 2),
                     "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs (burst copy)"},
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if ref_cuda is not None:
        line["secondary"]["reference_cuda"] = ref_cuda
    print(json.dumps(line), flush=True)


def _reference_cpu_forward(vsht=None):
    """(callable x -> coefficients, kind, description) of the reference's CPU path.

    Preferred: the reference's own ``RealVectorSHT.forward`` on torch CPU,
    imported unmodified from ``baseline/_ref`` (``baseline/reference_cpu.py``;
    rfft + its einsum contractions) with the tables this project uses.  If
    ``baseline/_ref`` was not staged, the oracle's fp32 restatement of that
    path (rfft + per-order GEMMs)."""
    import numpy as np
    import torch

    from baseline import reference_cpu

    if reference_cpu.available():
        hs_ref = reference_cpu.load()
        mod = hs_ref.RealVectorSHT(NLAT, NLON)

        def fn(xh):
            with torch.no_grad():
                return mod(torch.from_numpy(xh)).numpy()
        return fn, "reference", ("the reference's RealVectorSHT.forward on torch CPU "
                                 "(torch-ext/holysht/__init__.py:1504-1693, CPU branch)")
    from oracle import sht_oracle as orc

    if vsht is not None:
        w = np.stack([vsht.w0.float().cpu().numpy(), vsht.w1.float().cpu().numpy()])
    else:
        w = orc.vector_forward_tables(NLAT, NLON).astype(np.float32)
    return orc.CpuForwardBaseline(w, vector=True), "port", "oracle restatement: rfft + per-order fp32 GEMMs"


def _time_cpu(fn, xh, steps, warmup, budget_s):
    for _ in range(max(warmup, 1)):
        fn(xh)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or (len(times) < steps and time.perf_counter() < t_end):
        t = time.perf_counter()
        fn(xh)
        times.append((time.perf_counter() - t) * 1e3)
    return statistics.median(times), len(times)


def _check_against_oracle(out, xh):
    """Relative L2 of a CPU-path result against the float64 oracle on slice 0."""
    import numpy as np

    from oracle import sht_oracle as orc

    w = orc.vector_forward_tables(NLAT, NLON)
    ref = orc.vector_sht_forward(xh[:1].astype(np.float64), w)
    return float(np.linalg.norm(out[:1] - ref) / np.linalg.norm(ref))


def cpu_baseline(vsht, x):
    """The reference's CPU path on the same workload, on this host's cores
    (about 10 s of CPU work), checked once against the float64 oracle."""
    import torch

    _use_all_cores()
    fn, kind, what = _reference_cpu_forward(vsht)
    xh = x.cpu().numpy()
    ms, n = _time_cpu(fn, xh, 20, 1, 10.0)
    rel = _check_against_oracle(fn(xh), xh)
    return {"value": round(ms, 3), "unit": UNIT, "cores": torch.get_num_threads() if kind == "reference"
            else _blas_threads(), "kind": kind,
            "sample": f"full workload (4,2,512,1024), median of {n} runs; {what}",
            "rel_l2_vs_oracle": rel}


def _timed(fn, steps, dev, barrier, max_over_ranks, warmup=2):
    """Mean CUDA-event ms of ``fn`` over ``steps`` calls (after ``warmup``),
    bracketed by barriers; the max over ranks."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize(dev)
    barrier()
    return max_over_ranks(s.elapsed_time(e) / steps)


def run_c5(rank, world, dev, barrier, max_over_ranks):
    """The 1024 x 2048 configuration (lmax 1024, mmax 1025) on ``world`` GPUs,
    both partitions of the north star:

    * RealSHT on (16, 64, 1024, 2048): batch x channel partition, 1024/world
      slices per rank, each with a full table replica, no collective (the
      tcgen05 dense path);
    * RealVectorSHT on (16, 2, 1024, 2048): order partition (each rank holds
      1/world of the tables), the input replicated, the coefficients exchanged
      by the fused multicast/peer store + barrier, and by the NCCL all-gather
      for comparison.

    Inputs are larger than L2 (no flush needed).  Returns secondary fields."""
    import torch

    import holysht_b200 as hs
    from holysht_b200 import distributed as hd

    nlat, nlon = 1024, 2048
    res = {}
    # -- scalar, batch x channel partition
    sl = hd.shard_batch(16 * 64, rank, world)
    n = sl.stop - sl.start
    m = hs.RealSHT(nlat, nlon, table_device=dev)
    gen = torch.Generator(device=dev).manual_seed(4 + rank)
    x = torch.randn((n, nlat, nlon), generator=gen, device=dev)
    with torch.no_grad():
        ms = _timed(lambda: m(x), 3, dev, barrier, max_over_ranks)
    res["C5_RealSHT_batch_split"] = {"ms": round(ms, 4), "slices_per_rank": n,
                                     "transforms_per_s": round(16 * 64 / (ms * 1e-3), 1),
                                     "path": "tcgen05 dense" if n >= 128 else "streaming",
                                     "limiter": ("no collective: each rank's own rfft, operand transposes and "
                                                 "split-TF32 GEMM over its slices against a full table replica "
                                                 "(2.15 GB per rank); time falls with the slices per rank")}
    del m, x
    torch.cuda.empty_cache()
    # -- vector, order partition (replicated input: the same seed on every rank)
    gen = torch.Generator(device=dev).manual_seed(4)
    xv = torch.randn((16, 2, nlat, nlon), generator=gen, device=dev)
    for comm in (("auto", "nccl") if world > 1 else ("auto",)):
        v = hd.OrderShardedRealVectorSHT(nlat, nlon, comm=comm, table_device=dev, return_buffer=True)
        with torch.no_grad():
            ms = _timed(lambda: v(xv), 5, dev, barrier, max_over_ranks)
        key = "C5_RealVectorSHT_order_split" + ("" if comm == "auto" else "_nccl")
        res[key] = {"ms": round(ms, 4), "comm": v.comm, "orders": list(v.ranges[rank]),
                    "transforms_per_s": round(16 / (ms * 1e-3), 1),
                    "limiter": ("every rank runs the rfft of the whole replicated input and its 1/world "
                                "of the orders' contraction (FP32 multiply-adds); the exchange moves "
                                "(world-1)/world of the 268 MB of coefficients to every rank")}
        del v
        torch.cuda.empty_cache()
    return res


def reference_cuda_bar():
    """The reference's own CUDA path timed on this GPU (``baseline/reference_cuda.py``)
    in a child process, so this process never loads the reference's library.
    None when ``baseline/_ref`` was not staged; an error string if the child failed."""
    script = ROOT / "baseline" / "reference_cuda.py"
    if not (ROOT / "baseline" / "_ref" / "torch-ext" / "holysht" / "_ops.py").exists():
        return None
    try:
        res = subprocess.run([sys.executable, str(script), "--steps", "20", "--warmup", "5"], capture_output=True,
                             text=True, timeout=600, cwd=str(ROOT))
    except subprocess.TimeoutExpired:
        return {"error": "timed out after 600 s"}
    for ln in reversed(res.stdout.splitlines()):
        if ln.startswith("{"):
            return json.loads(ln)
    return {"error": f"rc={res.returncode}: {res.stderr.strip().splitlines()[-1:]}"}


def _use_all_cores():
    """Give the CPU baseline every host core (torchrun sets OMP_NUM_THREADS=1)."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(os.cpu_count())
    except Exception:
        pass


def _blas_threads():
    try:
        from threadpoolctl import threadpool_info

        return max(d["num_threads"] for d in threadpool_info())
    except Exception:
        return os.cpu_count()


# ------------------------------------------------------------------ reference arm

def run_reference(args, rank, world):
    """The reference arm: the reference's own CPU path (see _reference_cpu_forward)
    on the same workload and seed, every host core, rank 0 only; each step is
    one full forward (about 0.1-0.2 s)."""
    if rank != 0:
        return
    import numpy as np
    import torch

    _use_all_cores()
    fn, kind, what = _reference_cpu_forward()
    rng = np.random.default_rng(1)
    x = rng.standard_normal((BATCH, 2, NLAT, NLON)).astype(np.float32)
    ms, n = _time_cpu(fn, x, args.steps, args.warmup, 120.0)
    cores = torch.get_num_threads() if kind == "reference" else _blas_threads()
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(ms, 4),
        "unit": UNIT,
        "n_gpus": world,
        "steps": n,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": round(ms / PUBLISHED_GB10_MS, 5),
        "dtype": "f32",
        "data": "synthetic N(0,1), seed 1",
        "config": {"workload": "RealVectorSHT.forward 512x1024 equiangular lmax=512 mmax=513 ortho csphase, batch 4",
                   "global_batch": BATCH, "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(ms, 4), "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": f"full workload per step, median of {n} steps; {what}"},
        "e2e": {"value": round(ms, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank, world, local_rank = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
