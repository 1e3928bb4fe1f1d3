"""Multi-GPU partitions of the forward transforms (one process per GPU).

Two partitions:

* batch x channel (:func:`shard_batch`): every rank transforms its own slice
  of the leading dimensions with a full table replica; no collective.  This is
  what ``bench.py --gpus N`` runs.
* order blocks (:class:`OrderShardedRealSHT`, :class:`OrderShardedRealVectorSHT`):
  every rank owns a contiguous, 32-aligned range of orders m chosen so that
  the triangular work sum_m (lmax - m) is balanced, holds only that slice of
  the tables (1/G of the table bytes), contracts the full input's spectrum
  for its orders, and the coefficient slabs are all-gathered over NCCL into
  every rank's HBM.  This is the partition for the large vector case, where a
  batch split would stream the whole table on every GPU.

The reference has no multi-GPU code (its design notes list it as a
non-goal); both partitions are new.  The order-sharded modules are
forward-only (inference); use the single-GPU modules for training.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

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
]

TILE = 32


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
                       group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather per-rank coefficient slabs ``[..., L, Mpad]`` (this rank's orders
    in columns [0, width)) and assemble the full ``[..., L, mmax]`` on every rank."""
    world = len(ranges)
    if world == 1:
        a, b = ranges[0]
        return slab[..., : b - a].contiguous()
    if dist.get_backend(group) == "nccl":
        gathered = torch.empty((world,) + tuple(slab.shape), dtype=slab.dtype, device=slab.device)
        dist.all_gather_into_tensor(gathered, slab.contiguous(), group=group)
        parts = list(gathered.unbind(0))
    else:
        parts = [torch.empty_like(slab) for _ in range(world)]
        dist.all_gather(parts, slab.contiguous(), group=group)
    return torch.cat([p[..., : b - a] for p, (a, b) in zip(parts, ranges)], dim=-1)


class _OrderSharded(nn.Module):
    def _setup(self, dense_tables, L, K, M, nlon, group, vector):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.ranges = partition_orders(M, L, self.world)
        self.lmax, self.mmax, self.nlat, self.nlon, self.vector = L, M, K, nlon, vector
        lo, hi = self.ranges[self.rank]
        self.m_lo, self.m_hi = lo, hi
        self.width_pad = max(b - a for a, b in self.ranges) or 1
        local = [t[:, :, lo:hi].contiguous() for t in dense_tables]  # [L, K, width]
        if hi > lo:
            # streaming layout, (W0+W1, W0-W1) for vector, zero above the global diagonal
            grouped = ops.group_table8(tuple(local), _lib.DIR_FORWARD, m_offset=lo)
        else:
            grouped = torch.zeros((1, 1, 1, 2 * len(local), 32, 4), dtype=torch.float32)
        self.register_buffer("table_local", grouped, persistent=False)

    def _forward(self, x: torch.Tensor, P: int) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("holysht_b200 runs on CUDA tensors only (no CPU fallback)")
        if torch.is_grad_enabled() and x.requires_grad:
            raise RuntimeError("order-sharded transforms are forward-only; use the single-GPU modules for training")
        from . import _rfft

        spec = _rfft(x.float())
        lead = spec.shape[: -3] if P == 2 else spec.shape[:-2]
        spec = spec.reshape((int(math.prod(lead)), P, self.nlat, spec.size(-1)))
        B, W = spec.size(0), spec.size(-1)
        slab = torch.zeros((B, P, self.lmax, self.width_pad), dtype=torch.complex64, device=x.device)
        width = self.m_hi - self.m_lo
        if width > 0:
            ops.legendre_contract(
                kind=_lib.KIND_VECTOR if P == 2 else _lib.KIND_SCALAR, direction=_lib.DIR_FORWARD,
                input=spec[..., self.m_lo:], output=slab, w0=self.table_local, batch=B, nlat=self.nlat,
                lmax=self.lmax, mmax=width, in_strides=(P * self.nlat * W, self.nlat * W, W),
                out_strides=(P * self.lmax * self.width_pad, self.lmax * self.width_pad, self.width_pad),
                out_cols=width, scale=2.0 * math.pi / self.nlon, grouped8=True, m_offset=self.m_lo)
        full = gather_order_slabs(slab, self.ranges, self.group)
        shape = lead + ((2,) if P == 2 else ()) + (self.lmax, self.mmax)
        return full.reshape(shape)


class OrderShardedRealSHT(_OrderSharded):
    """``RealSHT`` with its orders partitioned across the ranks of ``group``
    (every rank passes the same full input and receives the full output)."""

    def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                 group: Optional[dist.ProcessGroup] = None):
        super().__init__()
        w, L, M = _weights.scalar_forward(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32)
        wt = torch.from_numpy(w).permute(1, 2, 0)  # [L, K, M] view
        self._setup([wt], L, nlat, M, nlon, group, vector=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        assert x.shape[-2:] == (self.nlat, self.nlon)
        return self._forward(x.unsqueeze(-3), 1).reshape(x.shape[:-2] + (self.lmax, self.mmax))


class OrderShardedRealVectorSHT(_OrderSharded):
    """``RealVectorSHT`` with its orders partitioned across the ranks of ``group``."""

    def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                 group: Optional[dist.ProcessGroup] = None):
        super().__init__()
        w, L, M = _weights.vector_forward(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32)
        wt = torch.from_numpy(w)
        self._setup([wt[0].permute(1, 2, 0), wt[1].permute(1, 2, 0)], L, nlat, M, nlon, group, vector=True)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        assert x.shape[-3:] == (2, self.nlat, self.nlon)
        return self._forward(x, 2)
