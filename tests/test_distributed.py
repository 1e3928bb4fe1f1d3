"""Multi-GPU partitions: host logic on CPU ranks (gloo, world size 2) and the
order-sharded transforms on the GPU (one GPU with order slices; two GPUs over
NCCL when the machine has them)."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from holysht_b200 import distributed as hd


def _close(got, ref):
    # different order slices may pick a different cluster split (summation order)
    tol = 1e-6 * float(ref.abs().max())
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=tol)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_batch_covers_evenly():
    for n in (0, 1, 5, 16, 17):
        for world in (1, 2, 3, 8):
            parts = [hd.shard_batch(n, r, world) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == n
            assert all(a.stop == b.start for a, b in zip(parts[:-1], parts[1:]))
            sizes = [p.stop - p.start for p in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        hd.shard_batch(4, 2, 2)


@pytest.mark.parametrize("M,L,world", [(513, 512, 2), (513, 512, 4), (513, 512, 8), (1025, 1024, 8),
                                       (257, 256, 3), (17, 16, 4), (70, 12, 2)])
def test_partition_orders_balanced_and_aligned(M, L, world):
    ranges = hd.partition_orders(M, L, world)
    assert len(ranges) == world
    assert ranges[0][0] == 0 and ranges[-1][1] == M
    assert all(a[1] == b[0] for a, b in zip(ranges[:-1], ranges[1:]))
    assert all(a % 32 == 0 or a == M for a, _ in ranges)
    work = [sum(max(L - m, 0) for m in range(a, b)) for a, b in ranges]
    tile_max = 32 * L
    assert max(work) - sum(work) / world <= tile_max


def _gloo_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        B, L, M = 2, 40, 70
        full = (rng.standard_normal((B, 2, L, M)) + 1j * rng.standard_normal((B, 2, L, M))).astype(np.complex64)
        ranges = hd.partition_orders(M, L, world)
        a, b = ranges[rank]
        pad = max(y - x for x, y in ranges)
        slab = torch.full((B, 2, L, pad), complex(7.0, -7.0), dtype=torch.complex64)  # padding is garbage
        slab[..., : b - a] = torch.from_numpy(full[..., a:b])
        got = hd.gather_order_slabs(slab, ranges)
        result[rank] = bool(np.array_equal(got.numpy(), full))
    finally:
        dist.destroy_process_group()


def _gloo_width_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ranges = [(0, 32), (32, 45)]
        a, b = ranges[rank]
        slab = torch.full((1, 1, 3, 32), complex(5.0, 5.0), dtype=torch.complex64)
        slab[..., : b - a] = complex(rank + 1, 0)
        got = hd.gather_order_slabs(slab, ranges, out_width=50)
        ok = got.shape == (1, 1, 3, 50) and bool((got[..., :32] == 1).all()) and bool((got[..., 32:45] == 2).all())
        result[rank] = ok and bool((got[..., 45:] == 0).all())
    finally:
        dist.destroy_process_group()


def test_gather_order_slabs_pads_zero_columns_gloo():
    """The inverse direction gathers into the irfft width: columns past the
    last order range are zero on every rank."""
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_width_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(result) == {0: True, 1: True}


def test_gather_order_slabs_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(result) == {0: True, 1: True}


# ------------------------------------------------------------------ GPU

@pytest.mark.gpu
def test_order_slices_on_one_gpu_match_the_full_transform():
    import holysht_b200 as hs
    from holysht_b200 import _lib, ops

    dev = torch.device("cuda")
    nlat, nlon = 96, 192
    v = hs.RealVectorSHT(nlat, nlon).to(dev)
    x = torch.randn(3, 2, nlat, nlon, device=dev)
    ref = v(x)
    spec = torch.fft.rfft(x, dim=-1)
    W = spec.size(-1)
    L, M = v.lmax, v.mmax
    for world in (2, 3):
        ranges = hd.partition_orders(M, L, world)
        pieces = []
        for a, b in ranges:
            if b == a:
                continue
            t = ops.group_table((v.w0_t[:, :, a:b].contiguous(), v.w1_t[:, :, a:b].contiguous()), _lib.DIR_FORWARD)
            out = torch.empty((3, 2, L, b - a), dtype=torch.complex64, device=dev)
            ops.legendre_contract(kind=_lib.KIND_VECTOR, direction=_lib.DIR_FORWARD, input=spec[..., a:],
                                  output=out, w0=t, batch=3, nlat=nlat, lmax=L, mmax=b - a,
                                  in_strides=(2 * nlat * W, nlat * W, W), out_strides=(2 * L * (b - a), L * (b - a), b - a),
                                  out_cols=b - a, scale=2 * math.pi / nlon, grouped=True, m_offset=a)
            pieces.append(out)
        _close(torch.cat(pieces, dim=-1), ref)


@pytest.mark.gpu
def test_order_sharded_modules_single_rank():
    import holysht_b200 as hs

    dev = torch.device("cuda")
    x = torch.randn(2, 2, 64, 128, device=dev)
    _close(hd.OrderShardedRealVectorSHT(64, 128).to(dev)(x), hs.RealVectorSHT(64, 128).to(dev)(x))
    _close(hd.OrderShardedRealSHT(64, 128).to(dev)(x[:, 0]), hs.RealSHT(64, 128).to(dev)(x[:, 0]))
    c = hs.RealVectorSHT(64, 128).to(dev)(x)
    _close(hd.OrderShardedInverseRealVectorSHT(64, 128, table_device=dev)(c),
           hs.InverseRealVectorSHT(64, 128).to(dev)(c))
    _close(hd.OrderShardedInverseRealSHT(64, 128, table_device=dev)(c[:, 0]),
           hs.InverseRealSHT(64, 128).to(dev)(c[:, 0]))
    # gradients through the sharded forward equal the module's
    for sharded, single, inp in ((hd.OrderShardedRealVectorSHT(64, 128, table_device=dev), hs.RealVectorSHT(64, 128),
                                  x),
                                 (hd.OrderShardedInverseRealSHT(64, 128, table_device=dev), hs.InverseRealSHT(64, 128),
                                  c[:, 0])):
        got = []
        for mod in (sharded, single.to(dev)):
            t = inp.clone().requires_grad_(True)
            y = mod(t)
            (y.abs().square().sum() if y.is_complex() else y.square().sum()).backward()
            got.append(t.grad)
        _close(got[0], got[1])


def _nccl_worker(rank, world, port, result):
    import holysht_b200 as hs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    out = {}
    try:
        nlat, nlon = 128, 256
        g = torch.Generator(device=dev).manual_seed(5)
        x = torch.randn(3, 2, nlat, nlon, device=dev, generator=g)
        c = torch.randn(3, 2, nlat, nlon // 2 + 1, device=dev, dtype=torch.complex64, generator=g)
        tri = torch.arange(nlon // 2 + 1, device=dev)[None, :] <= torch.arange(nlat, device=dev)[:, None]
        c = c * tri
        ref_v = hs.RealVectorSHT(nlat, nlon).to(dev)
        ref_s = hs.RealSHT(nlat, nlon).to(dev)
        ref_iv = hs.InverseRealVectorSHT(nlat, nlon).to(dev)
        ref_is = hs.InverseRealSHT(nlat, nlon).to(dev)

        def rel(a, b):
            return float((a - b).abs().max()) / float(b.abs().max())

        def grads(mod, inp):
            t = inp.clone().requires_grad_(True)
            y = mod(t)
            w = torch.linspace(0.5, 1.5, y.numel(), device=dev).reshape(y.shape)
            (y.abs().square() * w).sum().backward() if y.is_complex() else (y.square() * w).sum().backward()
            return y.detach(), t.grad

        for comm in ("nccl", "peer", "auto"):
            kw = dict(comm=comm, table_device=dev)
            v = hd.OrderShardedRealVectorSHT(nlat, nlon, **kw).to(dev)
            s = hd.OrderShardedRealSHT(nlat, nlon, **kw).to(dev)
            iv = hd.OrderShardedInverseRealVectorSHT(nlat, nlon, **kw).to(dev)
            is_ = hd.OrderShardedInverseRealSHT(nlat, nlon, **kw).to(dev)
            errs = []
            for _ in range(3):  # several calls: the exchange buffers alternate
                errs.append(rel(v(x), ref_v(x)))
                errs.append(rel(s(x[:, 0]), ref_s(x[:, 0])))
                errs.append(rel(iv(c), ref_iv(c)))
                errs.append(rel(is_(c[:, 0]), ref_is(c[:, 0])))
            for sharded, single, inp in ((v, ref_v, x), (s, ref_s, x[:, 0]), (iv, ref_iv, c), (is_, ref_is, c[:, 0])):
                ys, gs = grads(sharded, inp)
                yr, gr = grads(single, inp)
                errs += [rel(ys, yr), rel(gs, gr)]
            torch.cuda.synchronize(dev)
            out[comm] = (v.comm, max(errs), hd.peer_error_word())
        result[rank] = out
    finally:
        dist.destroy_process_group()


def _run_nccl(world):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    res = dict(result)
    assert sorted(res) == list(range(world))
    for rank, per in res.items():
        for comm, (used, err, perr) in per.items():
            assert err < 1e-5, (rank, comm, used, err)
            assert perr == 0, (rank, comm, used)
        assert per["nccl"][0] == "nccl" and per["peer"][0] == "peer"
    return res


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_order_sharded_transforms_two_gpus():
    """Forward and inverse, scalar and vector, values and gradients, with each
    exchange (NCCL all-gather, peer stores, and the automatic choice, which is
    the multicast store where NVSwitch offers it) against the single-GPU modules."""
    _run_nccl(2)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_order_sharded_transforms_four_gpus():
    _run_nccl(4)


def _faulty_gloo_worker(rank, world, port, result):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("injected fault before the gather")  # this rank never joins the collective
        slab = torch.zeros((1, 1, 4, 8), dtype=torch.complex64)
        try:
            hd.gather_order_slabs(slab, [(0, 8), (8, 16)])
            result.put((rank, "no error"))
        except Exception as e:  # the collective gives up after the process-group timeout
            result.put((rank, type(e).__name__))
    except RuntimeError as e:
        result.put((rank, "raised: " + str(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_failure_before_the_gather_is_reported_not_hung():
    """Host-side fault injection on CPU ranks: rank 1 raises before the
    all-gather; rank 0's collective ends with an error after the short
    process-group timeout instead of waiting forever."""
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_faulty_gloo_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(result.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got[1].startswith("raised:")
    assert got[0] != "no error"
