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


def _nccl_worker(rank, world, port, result):
    import holysht_b200 as hs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        g = torch.Generator(device=dev).manual_seed(5)
        x = torch.randn(2, 2, 128, 256, device=dev, generator=g)
        got = hd.OrderShardedRealVectorSHT(128, 256).to(dev)(x)
        ref = hs.RealVectorSHT(128, 256).to(dev)(x)
        err = float((got - ref).abs().max()) / float(ref.abs().max())
        result[rank] = err < 1e-5
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_order_sharded_vector_two_gpus_nccl():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert dict(result) == {0: True, 1: True}


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
