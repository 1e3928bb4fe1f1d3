"""Multi-GPU partitions of the transforms (one process per GPU).

Two partitions:

* batch x channel (:func:`shard_batch`): every rank transforms its own slice
  of the leading dimensions with a full table replica; no collective.
* order blocks (:class:`OrderShardedRealSHT`, :class:`OrderShardedRealVectorSHT`,
  :class:`OrderShardedInverseRealSHT`, :class:`OrderShardedInverseRealVectorSHT`):
  every rank owns a contiguous, 32-aligned range of orders m chosen so that
  the triangular work sum_m (lmax - m) is balanced, holds only that slice of
  the tables (1/G of the table bytes), contracts the replicated input for its
  orders, and every rank receives the whole output.  This is the partition
  for the large vector case, where a batch split would stream the whole table
  on every GPU.

How the order slices reach every rank (``comm``):

* ``"multicast"``: the contraction kernel stores each output element once
  through the NVLink multicast address of a buffer every rank holds
  (``multimem.st``; NVSwitch delivers it to all GPUs), then a cross-GPU
  barrier kernel orders the stores.  The exchange overlaps the contraction
  tile by tile and every element crosses NVLink once.
* ``"peer"``: the same, with one plain store per peer buffer (P2P over NVLink).
* ``"nccl"``: each rank contracts into a padded slab, ``all_gather_into_tensor``
  over NCCL, and one assembly copy (the reference design of the north star;
  also the fallback when symmetric memory is unavailable, e.g. gloo ranks).
* ``"auto"``: multicast if the GPUs support it, else peer, else nccl.

Buffers of the multicast/peer exchange are allocated with torch's symmetric
memory and used alternately (two per shape): a result returned with
``return_buffer=True`` stays valid until the second call after it on the same
stream; by default every result is a fresh tensor.

Autograd: the order-sharded forward and inverse transforms are
differentiable.  The gradient of the forward is the order-sharded conjugate
transpose (inverse direction) followed by the rfft adjoint; that of the
inverse is the order-sharded forward-direction contraction.  Every rank must
call a module with the same (replicated) input and receive the same upstream
gradient, as in any model-parallel layer whose output is replicated.

The reference has no multi-GPU code (its design notes list it as a
non-goal); both partitions are new.
"""
from __future__ import annotations

import math
import warnings
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist
import torch.nn as nn

from . import _lib, ops, weights as _weights

__all__ = [
    "shard_batch",
    "partition_orders",
    "gather_order_slabs",
    "OrderShardedRealSHT",
    "OrderShardedRealVectorSHT",
    "OrderShardedInverseRealSHT",
    "OrderShardedInverseRealVectorSHT",
    "peer_error_word",
]

TILE = 32
COMM_MODES = ("auto", "multicast", "peer", "nccl")


def shard_batch(n: int, rank: int, world: int) -> slice:
    """Contiguous slice of ``n`` batch items owned by ``rank`` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


def partition_orders(mmax: int, lmax: int, world: int) -> List[Tuple[int, int]]:
    """Split orders [0, mmax) into ``world`` contiguous ranges of whole 32-order
    tiles with balanced triangular work sum_m max(lmax - m, 0).

    Orders at or above lmax carry no work (their coefficients are zero) and go to
    the last range.  Ranges may be empty when there are fewer tiles than ranks."""
    if world <= 0:
        raise ValueError("world must be positive")
    n_tiles = (mmax + TILE - 1) // TILE
    work = np.array([sum(max(lmax - m, 0) for m in range(t * TILE, min(mmax, (t + 1) * TILE)))
                     for t in range(n_tiles)], dtype=np.float64)
    cum = np.concatenate([[0.0], np.cumsum(work)])
    total = cum[-1]
    cuts = [0]
    for r in range(1, world):
        target = total * r / world
        t = int(np.searchsorted(cum, target, side="left"))
        # choose the tile boundary closest to the target, monotone and in range
        if t > 0 and abs(cum[t - 1] - target) <= abs(cum[min(t, n_tiles)] - target):
            t -= 1
        t = min(max(t, cuts[-1]), n_tiles)
        cuts.append(t)
    cuts.append(n_tiles)
    return [(min(a * TILE, mmax), min(b * TILE, mmax)) for a, b in zip(cuts[:-1], cuts[1:])]


def gather_order_slabs(slab: torch.Tensor, ranges: Sequence[Tuple[int, int]],
                       group: Optional[dist.ProcessGroup] = None, out_width: Optional[int] = None) -> torch.Tensor:
    """All-gather per-rank coefficient slabs ``[..., R, Wpad]`` (this rank's orders
    in columns [0, width)) and assemble the full ``[..., R, out_width]`` on every
    rank (columns past the last range are zero)."""
    world = len(ranges)
    total = ranges[-1][1]
    out_width = total if out_width is None else out_width
    out = slab.new_zeros(tuple(slab.shape[:-1]) + (out_width,)) if out_width > total else None
    if world == 1:
        a, b = ranges[0]
        if out is None:
            return slab[..., : b - a].contiguous()
        out[..., a:b] = slab[..., : b - a]
        return out
    if dist.get_backend(group) == "nccl":
        gathered = torch.empty((world,) + tuple(slab.shape), dtype=slab.dtype, device=slab.device)
        dist.all_gather_into_tensor(gathered, slab.contiguous(), group=group)
        parts = list(gathered.unbind(0))
    else:
        parts = [torch.empty_like(slab) for _ in range(world)]
        dist.all_gather(parts, slab.contiguous(), group=group)
    if out is None:
        out = torch.empty(tuple(slab.shape[:-1]) + (out_width,), dtype=slab.dtype, device=slab.device)
    for p, (a, b) in zip(parts, ranges):
        out[..., a:b] = p[..., : b - a]
    return out


def peer_error_word() -> int:
    """Read and clear the cross-GPU barrier's device error word (bit 0: a peer
    did not arrive within the barrier's bounded wait).  Synchronous."""
    import ctypes

    v = ctypes.c_uint(0)
    _lib.check(_lib.load().holysht_peer_error_word(ctypes.byref(v)))
    return int(v.value)


# ---------------------------------------------------------------------------
# exchange: symmetric output buffers + barrier, or NCCL
# ---------------------------------------------------------------------------

class _Exchange:
    """Chooses and runs the exchange of an order-partitioned contraction.  The
    symmetric buffers are set up on first use, on the device of the first
    contraction (a collective: every rank makes its first call together)."""

    def __init__(self, group, comm: str):
        if comm not in COMM_MODES:
            raise ValueError(f"comm must be one of {COMM_MODES}, got {comm!r}")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.requested = comm
        self.mode = "local" if self.world == 1 else None  # decided on first use
        self.device = None
        self._bufs: Dict[tuple, list] = {}
        self._signal = None
        self._epoch = 0

    def ensure(self, device: torch.device) -> str:
        if self.mode is not None:
            return self.mode
        self.device = device
        self.mode = self.requested
        if self.mode in ("auto", "multicast", "peer"):
            try:
                self._setup_signal()
            except Exception as exc:  # no symmetric memory (CPU ranks, old driver, ...)
                if self.requested != "auto":
                    raise
                if device.type == "cuda":
                    warnings.warn(f"order-sharded exchange falls back to NCCL: {exc}")
                self.mode = "nccl"
        return self.mode

    def _group_name(self):
        g = self.group if self.group is not None else dist.group.WORLD
        return g.group_name

    def _setup_signal(self):
        if self.device.type != "cuda" or dist.get_backend(self.group) != "nccl":
            raise RuntimeError("peer exchange needs CUDA ranks on an NCCL group")
        from torch.distributed import _symmetric_memory as symm

        t = symm.empty(64, dtype=torch.int32, device=self.device)
        t.zero_()
        torch.cuda.synchronize(self.device)
        h = symm.rendezvous(t, self._group_name())
        base = t.data_ptr() - h.buffer_ptrs[self.rank]
        self._signal = (t, h, [p + base for p in h.buffer_ptrs])
        dist.barrier(group=self.group)  # every rank's signal array is zero before any barrier
        if self.mode == "auto":
            self.mode = "multicast" if h.multicast_ptr else "peer"

    def buffer(self, shape):
        """(local complex64 tensor, peer pointers, multicast pointer) of the next
        buffer of ``shape`` (two per shape, used alternately)."""
        from torch.distributed import _symmetric_memory as symm

        key = tuple(shape)
        slot = self._bufs.get(key)
        if slot is None:
            entries = []
            n = int(np.prod(shape)) * 2
            for _ in range(2):
                t = symm.empty(max(n, 2), dtype=torch.float32, device=self.device)
                h = symm.rendezvous(t, self._group_name())
                base = t.data_ptr() - h.buffer_ptrs[self.rank]
                peers = [p + base for p in h.buffer_ptrs]
                mc = (h.multicast_ptr + base) if (self.mode == "multicast" and h.multicast_ptr) else 0
                view = torch.view_as_complex(t[:n].view(*shape, 2)) if n else t[:0]
                entries.append((view, peers, mc, t, h))
            slot = [0, entries]
            self._bufs[key] = slot
        i = slot[0]
        slot[0] ^= 1
        view, peers, mc, _, _ = slot[1][i]
        return view, peers, mc

    def barrier(self, stream_ptr: int):
        import ctypes

        self._epoch += 1
        ptrs = self._signal[2]
        arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        _lib.check(_lib.load().holysht_peer_barrier(arr, len(ptrs), self.rank, ctypes.c_uint(self._epoch),
                                                     ctypes.c_void_p(stream_ptr)))


# ---------------------------------------------------------------------------
# the order-partitioned contraction
# ---------------------------------------------------------------------------

class _OrderShard:
    """This rank's slice of the tables and the contraction of its orders.

    ``local`` are the dense [lmax, nlat, width] slices (W0, W1 for the vector
    map) of the transform's own direction ``hot``; the streaming-layout tables
    are built per direction on first use (the other direction, used by
    autograd, is the conjugate map for the vector kind)."""

    def __init__(self, local, vector, L, K, M, ranges, rank, exchange: _Exchange, hot: int):
        self.local = local
        self.vector = vector
        self.L, self.K, self.M = L, K, M
        self.ranges = ranges
        self.m_lo, self.m_hi = ranges[rank]
        self.width = self.m_hi - self.m_lo
        self.width_pad = max(b - a for a, b in ranges) or 1
        self.ex = exchange
        self.hot = hot
        self._tables: Dict[int, torch.Tensor] = {}

    def table(self, direction: int) -> torch.Tensor:
        t = self._tables.get(direction)
        if t is None or t.device != self.local[0].device:
            if self.width > 0:
                conj = self.vector and direction != self.hot
                t = ops.group_table8(tuple(self.local), direction, conj=conj, m_offset=self.m_lo)
            else:
                t = torch.zeros((1, 1, 1, 2 * len(self.local), 32, 4), dtype=torch.float32,
                                device=self.local[0].device)
            self._tables[direction] = t
        return t

    def contract(self, direction: int, inp: torch.Tensor, rows: int, out_width: int, scale: float,
                 flags: int = 0, nlon: int = 0, keep_buffer: bool = False) -> torch.Tensor:
        """Full [B, P, rows, out_width] result of the contraction of ``inp``
        [B, P, S, >= m_hi] (replicated) on every rank; columns >= mmax are zero."""
        P = 2 if self.vector else 1
        B = inp.size(0)
        S = inp.size(2)
        kind = _lib.KIND_VECTOR if self.vector else _lib.KIND_SCALAR
        fwd = direction == _lib.DIR_FORWARD
        lmax = self.L
        table = self.table(direction)
        in_strides = (inp.stride(0), inp.stride(1), inp.stride(2))
        common = dict(kind=kind, direction=direction, input=inp[..., self.m_lo:] if self.width > 0 else inp,
                      w0=table, batch=B, nlat=self.K, lmax=lmax, mmax=self.width, in_strides=in_strides,
                      scale=scale, flags=flags, nlon=nlon, grouped8=True, m_offset=self.m_lo)
        assert S == (self.K if fwd else self.L)
        mode = self.ex.ensure(inp.device)
        if mode in ("local", "nccl"):
            slab = torch.empty((B, P, rows, self.width_pad), dtype=torch.complex64, device=inp.device)
            out_strides = (slab.stride(0), slab.stride(1), slab.stride(2))
            if self.width > 0:
                ops.legendre_contract(output=slab, out_strides=out_strides, out_cols=self.width, **common)
            return gather_order_slabs(slab, self.ranges, self.ex.group, out_width=out_width)
        # multicast / peer: store straight into every rank's buffer, then a barrier
        out, peers, mc = self.ex.buffer((B, P, rows, out_width))
        last = self.ex.rank == len(self.ranges) - 1
        cols = (out_width - self.m_lo) if last else self.width  # the last rank also zeroes [mmax, out_width)
        if cols > 0:
            out_strides = (out.stride(0), out.stride(1), out.stride(2))
            ops.legendre_contract_peers(peers, out_col_offset=self.m_lo, multicast_ptr=mc, output=out,
                                        out_strides=out_strides, out_cols=cols, **common)
        self.ex.barrier(ops._current_stream_handle(inp.device.index))
        return out if keep_buffer else out.clone()


class _ShardedForwardFn(torch.autograd.Function):
    """coef = Legendre(spec) on the order partition; backward: the conjugate
    transpose (inverse direction), gathered the same way."""

    @staticmethod
    def forward(ctx, spec, shard: _OrderShard, scale: float, keep_buffer: bool):
        ctx.shard, ctx.scale, ctx.W = shard, scale, spec.size(-1)
        return shard.contract(_lib.DIR_FORWARD, spec, shard.L, shard.M, scale, keep_buffer=keep_buffer)

    @staticmethod
    def backward(ctx, grad):
        sh = ctx.shard
        g = grad.contiguous()
        gspec = sh.contract(_lib.DIR_INVERSE, g, sh.K, ctx.W, ctx.scale)
        return gspec, None, None, None


class _ShardedInverseFn(torch.autograd.Function):
    """spec = irfft-ready synthesis of coef on the order partition; backward:
    the adjoint of the irfft preparation, then the forward-direction
    contraction (conjugate map for the vector kind)."""

    @staticmethod
    def forward(ctx, coef, shard: _OrderShard, nlon: int):
        ctx.shard, ctx.nlon = shard, nlon
        return shard.contract(_lib.DIR_INVERSE, coef.contiguous(), shard.K, nlon // 2 + 1, 1.0,
                              flags=_lib.FLAG_IRFFT_PREP, nlon=nlon)

    @staticmethod
    def backward(ctx, grad):
        sh = ctx.shard
        g = grad.clone(memory_format=torch.contiguous_format)
        g[..., 0] = g[..., 0].real.to(g.dtype)
        if ctx.nlon % 2 == 0:
            g[..., ctx.nlon // 2] = g[..., ctx.nlon // 2].real.to(g.dtype)
        gc = sh.contract(_lib.DIR_FORWARD, g, sh.L, sh.M, 1.0)
        return gc, None, None


class _OrderSharded(nn.Module):
    def _setup(self, dense_tables, L, K, M, nlon, group, vector, comm, hot):
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.ranges = partition_orders(M, L, self.world)
        self.lmax, self.mmax, self.nlat, self.nlon, self.vector = L, M, K, nlon, vector
        lo, hi = self.ranges[self.rank]
        self.m_lo, self.m_hi = lo, hi
        local = [t[:, :, lo:hi].contiguous() for t in dense_tables]  # [L, K, width]
        self._exchange = _Exchange(group, comm)
        self._shard = _OrderShard(local, vector, L, K, M, self.ranges, self.rank, self._exchange, hot)
        self.group = group

    @property
    def comm(self) -> str:
        """The exchange in use: "multicast", "peer", "nccl" or "local" (one
        rank); None before the first call."""
        return self._exchange.mode

    def _apply(self, fn, *args, **kwargs):
        # the local table slices follow .to() / .cuda() (they are not buffers:
        # state dicts of a sharded module would differ between ranks)
        out = super()._apply(fn, *args, **kwargs)
        sh = self._shard
        sh.local = [fn(t) for t in sh.local]
        sh._tables = {}
        return out

    def _check_cuda(self, x):
        if not x.is_cuda:
            raise RuntimeError("holysht_b200 runs on CUDA tensors only (no CPU fallback)")


class OrderShardedRealSHT(_OrderSharded):
    """``RealSHT`` with its orders partitioned across the ranks of ``group``
    (every rank passes the same full input and receives the full output).

    ``table_device`` builds the float64 tables on that device (a GPU builds
    the 1024 x 2048 tables in about a second, the host in tens of seconds);
    ``comm`` picks the exchange (module docstring); ``return_buffer`` returns
    the exchange buffer itself (valid until the second call after it) instead
    of a copy when no gradient is recorded."""

    def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                 group: Optional[dist.ProcessGroup] = None, comm: str = "auto", table_device=None,
                 return_buffer: bool = False):
        super().__init__()
        w, L, M = _weights.scalar_forward(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        wt = (torch.from_numpy(w) if table_device is None else w).permute(1, 2, 0)  # [L, K, M] view
        self.return_buffer = return_buffer
        self._setup([wt], L, nlat, M, nlon, group, False, comm, _lib.DIR_FORWARD)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self._check_cuda(x)
        assert x.shape[-2:] == (self.nlat, self.nlon)
        lead = x.shape[:-2]
        from . import _rfft

        spec = _rfft(x.float()).reshape(int(math.prod(lead)), 1, self.nlat, -1)
        keep = self.return_buffer and not (torch.is_grad_enabled() and spec.requires_grad)
        out = _ShardedForwardFn.apply(spec, self._shard, 2.0 * math.pi / self.nlon, keep)
        return out.reshape(lead + (self.lmax, self.mmax))


class OrderShardedRealVectorSHT(_OrderSharded):
    """``RealVectorSHT`` with its orders partitioned across the ranks of ``group``
    (arguments as :class:`OrderShardedRealSHT`)."""

    def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                 group: Optional[dist.ProcessGroup] = None, comm: str = "auto", table_device=None,
                 return_buffer: bool = False):
        super().__init__()
        w, L, M = _weights.vector_forward(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        wt = torch.from_numpy(w) if table_device is None else w
        self.return_buffer = return_buffer
        self._setup([wt[0].permute(1, 2, 0), wt[1].permute(1, 2, 0)], L, nlat, M, nlon, group, True, comm,
                    _lib.DIR_FORWARD)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self._check_cuda(x)
        assert x.shape[-3:] == (2, self.nlat, self.nlon)
        lead = x.shape[:-3]
        from . import _rfft

        spec = _rfft(x.float()).reshape(int(math.prod(lead)), 2, self.nlat, -1)
        keep = self.return_buffer and not (torch.is_grad_enabled() and spec.requires_grad)
        out = _ShardedForwardFn.apply(spec, self._shard, 2.0 * math.pi / self.nlon, keep)
        return out.reshape(lead + (2, self.lmax, self.mmax))


class OrderShardedInverseRealSHT(_OrderSharded):
    """``InverseRealSHT`` with its orders partitioned across the ranks of ``group``:
    every rank passes the same coefficients [..., lmax, mmax], synthesises the
    irfft input of its orders, the slices are exchanged, and every rank runs the
    irfft of the whole spectrum."""

    def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                 group: Optional[dist.ProcessGroup] = None, comm: str = "auto", table_device=None):
        super().__init__()
        p, L, M = _weights.scalar_inverse(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        pt = (torch.from_numpy(p) if table_device is None else p).permute(1, 2, 0)
        self._setup([pt], L, nlat, M, nlon, group, False, comm, _lib.DIR_INVERSE)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self._check_cuda(x)
        assert x.shape[-2:] == (self.lmax, self.mmax)
        lead = x.shape[:-2]
        from . import _irfft

        c = x.reshape(int(math.prod(lead)), 1, self.lmax, self.mmax).to(torch.complex64)
        spec = _ShardedInverseFn.apply(c, self._shard, self.nlon)
        return _irfft(spec, self.nlon).reshape(lead + (self.nlat, self.nlon))


class OrderShardedInverseRealVectorSHT(_OrderSharded):
    """``InverseRealVectorSHT`` with its orders partitioned across the ranks of ``group``."""

    def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                 group: Optional[dist.ProcessGroup] = None, comm: str = "auto", table_device=None):
        super().__init__()
        d, L, M = _weights.vector_inverse(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        dt = torch.from_numpy(d) if table_device is None else d
        self._setup([dt[0].permute(1, 2, 0), dt[1].permute(1, 2, 0)], L, nlat, M, nlon, group, True, comm,
                    _lib.DIR_INVERSE)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self._check_cuda(x)
        assert x.shape[-3:] == (2, self.lmax, self.mmax)
        lead = x.shape[:-3]
        from . import _irfft

        c = x.reshape(int(math.prod(lead)), 2, self.lmax, self.mmax).to(torch.complex64)
        spec = _ShardedInverseFn.apply(c, self._shard, self.nlon)
        return _irfft(spec, self.nlon).reshape(lead + (2, self.nlat, self.nlon))
