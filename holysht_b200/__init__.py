"""holysht_b200: B200-native (sm_100a) Legendre kernels behind HOLYSHT's API.

Drop-in replacements for the reference's public modules and functions
(chrisvoncsefalvay/holysht ``torch-ext/holysht/__init__.py``):

* ``RealSHT`` / ``InverseRealSHT`` / ``RealVectorSHT`` / ``InverseRealVectorSHT``
  (reference :1228-1791) with the same constructor arguments
  ``(nlat, nlon, lmax, mmax, grid, norm, csphase[, dtype])``, the same
  buffer names (``weights``/``weight_t``, ``pct``/``pct_t``,
  ``w0``/``w1``/``w0_t``/``w1_t``, ``d0``/``d1``/``d0_t``/``d1_t``) and autograd;
* ``GraphedModule`` (reference :1794-1866), the function API
  ``legendre_forward`` / ``legendre_inverse`` / ``sht_forward`` /
  ``sht_inverse`` and the ``Fused*`` aliases (:1869-1878).

Every transform runs the longitude FFT on cuFFT (``torch.fft``) and the
Legendre stage on the kernels of ``libholysht_b200.so`` on the same stream.
The forward kernels read the rfft output in place (no slice copy) and fold the
2*pi spectrum scale; the inverse kernels write straight into the irfft input
(zero padding and the DC/Nyquist imaginary parts handled in the kernel).
There is no CPU fallback: CUDA tensors only.
"""
from __future__ import annotations

import math
from enum import IntEnum
from typing import Optional

import numpy as np
import torch
import torch.nn as nn

from . import _lib, ops, weights as _weights
from .ops import legendre_contract as _contract

__all__ = [
    "RealSHT",
    "InverseRealSHT",
    "RealVectorSHT",
    "InverseRealVectorSHT",
    "GraphedModule",
    "legendre_forward",
    "legendre_inverse",
    "sht_forward",
    "sht_inverse",
]

TWO_PI = 2.0 * math.pi
_HAS_NATIVE_EXT = _lib.LIB_PATH.exists()


class _ForwardBackend(IntEnum):
    """Backend hints of the reference's ``*_ex`` operators (``__init__.py:192-197``).
    Accepted for compatibility; all hints run the FP32 sm_100a kernel."""

    AUTO = 0
    FMA = 1
    TMA = 2
    TC_TF32 = 3
    TC_BF16 = 4


def _need_cuda(x: torch.Tensor, what: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(f"{what}: holysht_b200 runs on CUDA tensors only (no CPU fallback)")


def _rfft(x: torch.Tensor, norm: str = "backward") -> torch.Tensor:
    """``torch.fft.rfft`` over the last dimension; cuFFT rejects a zero-sized
    batch, whose spectrum is just an empty tensor of the right shape."""
    if x.numel() == 0:
        return torch.empty(x.shape[:-1] + (x.size(-1) // 2 + 1,), dtype=torch.complex64, device=x.device)
    return torch.fft.rfft(x, dim=-1, norm=norm)


def _irfft(spec: torch.Tensor, n: int) -> torch.Tensor:
    """``torch.fft.irfft(..., norm="forward")`` over the last dimension, empty
    batches included."""
    if spec.numel() == 0:
        return torch.empty(spec.shape[:-1] + (n,), dtype=torch.float32, device=spec.device)
    return torch.fft.irfft(spec, n=n, dim=-1, norm="forward")


def _flat_batch(shape, trailing: int) -> int:
    """Number of slices in the leading dimensions (``reshape(-1, ...)`` cannot
    infer it for an empty tensor)."""
    n = 1
    for d in shape[: len(shape) - trailing]:
        n *= d
    return n


def _strides3(t: torch.Tensor, vector: bool):
    """(batch, component, row) element strides of a [B,(2),R,C] tensor."""
    if vector:
        return t.stride(0), t.stride(1), t.stride(2)
    return t.stride(0), 0, t.stride(1)


# ---------------------------------------------------------------------------
# table sources: where a transform's Legendre tables live
# ---------------------------------------------------------------------------

class _DenseTables:
    """Tables in the reference operator layout [lmax, nlat, mmax] (strided path)."""

    def __init__(self, w0: torch.Tensor, w1: Optional[torch.Tensor] = None):
        self.w0, self.w1 = w0, w1
        self.vector = w1 is not None
        self.lmax, self.nlat, self.mmax = w0.shape

    def table(self, direction: int, layout=None):
        return self.w0, self.w1, "strided"


class _GroupedTablesMixin:
    """Module mixin: dense buffers plus cached row-grouped copies per direction
    (``ops.group_table8`` / ``ops.group_table``), built on the first
    contraction in that direction on the tables' device.  The copies
    are non-persistent buffers (they follow ``.to()``) and are dropped when a
    state dict is loaded into the dense buffers."""

    def _init_tables(self, names, hot_direction: int) -> None:
        self._table_names = tuple(names)
        self.vector = len(self._table_names) == 2
        self._hot_direction = hot_direction
        self.register_buffer("_grouped_fwd", None, persistent=False)
        self.register_buffer("_grouped_inv", None, persistent=False)
        self.register_buffer("_grouped8_fwd", None, persistent=False)
        self.register_buffer("_grouped8_inv", None, persistent=False)
        self.register_buffer("_grouped8p_fwd", None, persistent=False)
        self.register_buffer("_grouped8p_inv", None, persistent=False)
        # the streaming copies are built on first use, on the tables' device
        # (a GPU builds them in milliseconds; the host takes tens of seconds
        # at 1024 x 2048)
        self.register_load_state_dict_post_hook(lambda module, _keys: module._drop_grouped())

    def _spectrum(self, x: torch.Tensor):
        """(rfft spectrum, kernel scale, round-to-bf16 flag) of a real field.

        FP32: the unnormalised rfft, with the 2*pi/nlon of the reference's
        ``2*pi*rfft(x, norm="forward")`` folded into the Legendre kernel (no
        separate scaling pass).  BF16/FP16 modules round the scaled spectrum,
        as the reference does (``__init__.py:1291-1295``), so it is scaled
        before the kernel rounds it."""
        low = bool(getattr(self, "_use_bf16", False) or getattr(self, "_use_fp16", False))
        if low:
            return TWO_PI * _rfft(x.float(), "forward"), 1.0, True
        return _rfft(x.float()), TWO_PI / self.nlon, False

    def _apply(self, fn, *args, **kwargs):
        # .to() / .cuda() / dtype casts move the tables: prepared launches must not outlive them
        self.__dict__.pop("_contract_plans", None)
        self.__dict__.pop("_fast_forward", None)
        self.__dict__.pop("_dense_split_fwd", None)
        self.__dict__.pop("_dense_split_inv", None)
        return super()._apply(fn, *args, **kwargs)

    def _drop_grouped(self) -> None:
        self.__dict__.pop("_dense_split_fwd", None)
        self.__dict__.pop("_dense_split_inv", None)
        self.__dict__.pop("_contract_plans", None)
        self.__dict__.pop("_fast_forward", None)
        self._grouped_fwd = None
        self._grouped_inv = None
        self._grouped8_fwd = None
        self._grouped8_inv = None
        self._grouped8p_fwd = None
        self._grouped8p_inv = None
        self.__dict__.pop("_symmetric", None)
        if hasattr(self, "_dense_inv"):
            self._dense_inv = None

    def dense_table(self, direction: int) -> torch.Tensor:
        """Per-order fp32 table for the tensor-core path: forward [mmax, lmax, nlat]
        (the reference's ``weights`` / ``pct`` layout), inverse [mmax, nlat, lmax]
        (built on first use, non-persistent buffer)."""
        mlk = getattr(self, self._mlk_name)
        if mlk.dtype != torch.float32:
            mlk = getattr(self, self._table_names[0]).permute(2, 0, 1)
        if direction == _lib.DIR_FORWARD:
            return mlk.contiguous()
        t = getattr(self, "_dense_inv", None)
        if t is None or t.device != mlk.device:
            t = mlk.transpose(1, 2).contiguous()
            if "_dense_inv" not in self._buffers:
                self.register_buffer("_dense_inv", t, persistent=False)
            else:
                self._dense_inv = t
        return t

    def dense_table_split(self, direction: int) -> torch.Tensor:
        """The tensor-core path's table split into tf32 and residual planes
        (``ops.split_dense_table``), built once per direction on first use."""
        name = "_dense_split_fwd" if direction == _lib.DIR_FORWARD else "_dense_split_inv"
        t = self.__dict__.get(name)
        dense = self.dense_table(direction)
        if t is None or t.device != dense.device:
            t = ops.split_dense_table(dense)
            self.__dict__[name] = t
        return t

    def _equatorial_symmetry(self) -> bool:
        """True when the forward tables obey the equatorial parity the folded
        (``"parity"``) layout relies on: W(K-1-k) = s W(k) for the scalar table
        and W1, W0(K-1-k) = -s W0(k), s = (-1)^(l+m), to 1e-6 of the largest
        entry (every grid this package builds is symmetric; tables loaded from
        elsewhere are checked)."""
        sym = self.__dict__.get("_symmetric")
        if sym is None:
            dense = [getattr(self, n) for n in self._table_names]
            L, K, M = dense[0].shape
            dev = dense[0].device
            sgn = 1.0 - 2.0 * ((torch.arange(L, device=dev)[:, None, None]
                                + torch.arange(M, device=dev)[None, None, :]) % 2).float()
            sym = True
            for i, d in enumerate(dense):
                f = -sgn if (self.vector and i == 0) else sgn
                err = (d.flip(1) - f * d).abs().max()
                sym = sym and bool(err <= 1e-6 * d.abs().max().clamp_min(1e-30))
            self.__dict__["_symmetric"] = sym
        return sym

    def table(self, direction: int, layout=None):
        """(table, None, layout) for one contraction direction.

        ``layout`` "grouped8" (``ops.group_table8``, the streaming kernel) is
        the default for both directions (BF16/FP16 modules included: the
        kernel rounds the staged spectrum); "grouped" (``ops.group_table``,
        4-row groups) is the 4-row kernel, which ``HOLYSHT_TABLE_LAYOUT=grouped``
        selects everywhere."""
        if layout is None:
            import os

            stream = os.environ.get("HOLYSHT_TABLE_LAYOUT", "grouped8") != "grouped"
            layout = "grouped8" if stream else "grouped"
            # the folded layout halves the table bytes; it is the forward default
            # (512 x 1024 b4: scalar 61.5 -> 57.3 us, vector 118.8 -> 98.3 us);
            # HOLYSHT_PARITY=0 turns it off.
            # The scalar inverse direction can fold too (half the table bytes and FMAs),
            # but with half the output rows it has half the work items and was measured
            # slower at 512 x 1024 b4 (85 vs 77 us per InverseRealSHT.forward), so it
            # is used only with HOLYSHT_PARITY_INV=1.
            par = os.environ.get("HOLYSHT_PARITY", "1")
            fold_inv = os.environ.get("HOLYSHT_PARITY_INV", "0") == "1"
            if direction == _lib.DIR_FORWARD:
                want = par != "0"
            else:
                want = fold_inv and not self.vector
            if stream and want and self._equatorial_symmetry():
                layout = "parity"
        if layout == "parity":
            pname = "_grouped8p_fwd" if direction == _lib.DIR_FORWARD else "_grouped8p_inv"
            t = getattr(self, pname)
            dense = tuple(getattr(self, n) for n in self._table_names)
            if t is None or t.device != dense[0].device:
                half = (self.nlat + 1) // 2
                north = [d[:, :half, :].contiguous() for d in dense]
                if self.vector:
                    # (Wp, Wn) = (W0 + c W1, -(-1)^l (W0 - c W1)), c = -1 for the
                    # conjugate map (autograd of an inverse transform)
                    c = -1.0 if direction != self._hot_direction else 1.0
                    w0, w1 = north
                    lsign = 1.0 - 2.0 * (torch.arange(w0.shape[0], device=w0.device) % 2).float()
                    north = [w0 + c * w1, -lsign[:, None, None] * (w0 - c * w1)]
                t = ops.group_table8(tuple(north) if self.vector else north[0], direction, combine=False)
                setattr(self, pname, t)
                self.__dict__.pop("_contract_plans", None)
                self.__dict__.pop("_fast_forward", None)
            return t, None, layout
        if layout == "grouped8":
            name = "_grouped8_fwd" if direction == _lib.DIR_FORWARD else "_grouped8_inv"
        else:
            name = "_grouped_fwd" if direction == _lib.DIR_FORWARD else "_grouped_inv"
        t = getattr(self, name)
        dense = tuple(getattr(self, n) for n in self._table_names)
        if t is None or t.device != dense[0].device:
            # the non-hot direction serves autograd: for the vector map it is the
            # conjugate transpose, whose grouped table carries the sign of W1
            conj = self.vector and direction != self._hot_direction
            build = ops.group_table8 if layout == "grouped8" else ops.group_table
            t = build(dense, direction, conj=conj)
            setattr(self, name, t)
            self.__dict__.pop("_contract_plans", None)  # prepared calls point at the old table
            self.__dict__.pop("_fast_forward", None)
        return t, None, layout


DENSE_TC_MIN_BATCH = 128  # flattened batch from which the scalar forward runs on tcgen05


def _dense_tc_eligible(src, B: int, direction: int) -> bool:
    """Scalar modules with fp32 per-order tables, a reduction extent that is a
    multiple of 4 (nlat forward, lmax inverse) and a large flattened batch
    (N = 2B GEMM columns).  ``HOLYSHT_DENSE_TC`` = 0 / 1 forces it off / on
    (when the layout allows)."""
    import os

    if src.vector or not hasattr(src, "dense_table"):
        return False
    red = src.nlat if direction == _lib.DIR_FORWARD else src.lmax
    if red % 4:
        return False
    force = os.environ.get("HOLYSHT_DENSE_TC", "")
    if force in ("0", "1"):
        return force == "1"
    ref = _reference_backend()
    if ref is not None:
        return ref
    return B >= DENSE_TC_MIN_BATCH


_REF_FLAGS_WARNED = set()


def _reference_backend():
    """The reference's backend environment flags (``torch-ext/holysht/__init__.py:253-288``),
    mapped onto this package's paths: ``HOLYSHT_FORCE_BACKEND`` = ``tc_tf32`` / ``tc_bf16``
    forces the tensor-core path (True), ``fma`` / ``tma`` the streaming kernel (False),
    ``auto`` or unset chooses by batch size (None).  ``HOLYSHT_FORCE_VECTOR_STRATEGY``
    and the ``HOLYSHT_AUTOTUNE*`` flags select among reference kernels that have no
    counterpart here (one kernel per case, nothing timed at run time): they are
    accepted, ignored, and reported once with a warning."""
    import os
    import warnings

    for name in ("HOLYSHT_FORCE_VECTOR_STRATEGY", "HOLYSHT_AUTOTUNE", "HOLYSHT_AUTOTUNE_REBENCH",
                 "HOLYSHT_AUTOTUNE_CACHE_PATH"):
        if os.environ.get(name) and name not in _REF_FLAGS_WARNED:
            _REF_FLAGS_WARNED.add(name)
            warnings.warn(f"{name} is a reference autotuning flag; holysht_b200 has a fixed kernel choice "
                          "and ignores it")
    raw = os.environ.get("HOLYSHT_FORCE_BACKEND", "").strip().lower()
    if raw in ("tc_tf32", "tc_bf16"):
        return True
    if raw in ("fma", "tma"):
        return False
    return None


_MAX_PLANS = 32  # prepared contraction calls cached per table source


def _run(src, direction, inp, out, B, M, in_vec_strides, out_vec_strides, out_cols, scale, flags, nlon=0):
    w0, w1, layout = src.table(direction)
    if layout != "strided" and src.vector:
        # grouped vector tables already encode the conjugate map (see table())
        assert bool(flags & _lib.FLAG_CONJ_W1) == (direction != src._hot_direction)
        flags &= ~_lib.FLAG_CONJ_W1
    # the descriptor of a repeated call is built and checked once (ops.ContractPlan)
    key = (direction, B, M, tuple(in_vec_strides), tuple(out_vec_strides), out_cols, scale, flags, nlon, layout,
           w0.data_ptr(), None if w1 is None else w1.data_ptr(), inp.dtype, out.dtype, inp.device.index,
           tuple(inp.shape), inp.stride(), tuple(out.shape), out.stride())
    plans = src.__dict__.setdefault("_contract_plans", {})
    plan = plans.get(key)
    if plan is None:
        if len(plans) >= _MAX_PLANS:
            plans.clear()
        plan = ops.ContractPlan(input_like=inp, output_like=out, kind=_lib.KIND_VECTOR if src.vector else _lib.KIND_SCALAR,
                                direction=direction, w0=w0, w1=w1, batch=B, nlat=src.nlat, lmax=src.lmax, mmax=M,
                                in_strides=in_vec_strides, out_strides=out_vec_strides, out_cols=out_cols,
                                scale=scale, flags=flags, nlon=nlon, grouped=layout == "grouped",
                                grouped8=layout in ("grouped8", "parity"), parity=layout == "parity")
        plans[key] = plan
    plan.launch(inp, out)
    return plan


# ---------------------------------------------------------------------------
# module-level autograd functions (spectrum in rfft layout)
# ---------------------------------------------------------------------------

def _legendre_forward(spec, src, round_bf16: bool, scale: float):
    """coef = scale * Legendre(spec[..., :mmax]) (the body of the module forward)."""
    return _legendre_forward_planned(spec, src, round_bf16, scale)[0]


def _legendre_forward_planned(spec, src, round_bf16: bool, scale: float):
    """(coef, the prepared contraction it ran or None): the table path returns
    its ``ops.ContractPlan`` so the caller can reuse it."""
    plan = None
    vector = src.vector
    B, K = spec.size(0), spec.size(-2)
    if K != src.nlat:
        raise RuntimeError(f"spectrum has {K} latitudes, tables {src.nlat}")
    L, M = src.lmax, src.mmax
    shape = (B, 2, L, M) if vector else (B, L, M)
    out = torch.empty(shape, device=spec.device, dtype=torch.complex64)
    if getattr(src, "variant", "table") == "recurrence" and not round_bf16:
        # on-the-fly Legendre functions: no table stream
        seeds, coef, ct = src.recurrence_tables()
        if vector:
            ops.legendre_vector_forward_recurrence(out, spec, seeds, coef, ct, scale,
                                                   parity=getattr(src, "rec_parity", False))
        else:
            ops.legendre_forward_recurrence(out, spec, seeds, coef, ct, scale,
                                            parity=getattr(src, "rec_parity", False))
    elif _dense_tc_eligible(src, B, _lib.DIR_FORWARD):
        # large batch: the per-order contraction is a dense GEMM -> tcgen05
        ops.legendre_dense_tc(_lib.DIR_FORWARD, out, spec, src.dense_table_split(_lib.DIR_FORWARD), nlat=K,
                              lmax=L, mmax=M, scale=scale, flags=_lib.FLAG_ROUND_BF16 if round_bf16 else 0)
    else:
        plan = _run(src, _lib.DIR_FORWARD, spec, out, B, M, _strides3(spec, vector), _strides3(out, vector),
                    M, scale, _lib.FLAG_ROUND_BF16 if round_bf16 else 0)
    return out, plan


class _FastForward:
    """The module forward for one input shape, once it has run through the
    general path: rfft, output allocation and the prepared contraction (no
    table lookups, checks or autograd).  Used only when no gradient is
    wanted, for FP32 modules on the table path; dropped with the tables.
    For a contiguous input the rfft and the contraction are one library call
    (``holysht_rfft_contract``: cuFFT's R2C, then the Legendre kernel, on the
    current stream); otherwise torch's rfft feeds the prepared launch."""

    __slots__ = ("plan", "spec_shape", "out_shape", "final_shape", "device", "rows", "nlon", "fft_work")

    def __init__(self, plan, spec_shape, out_shape, final_shape, device, nlon):
        self.plan, self.spec_shape, self.out_shape = plan, spec_shape, out_shape
        self.final_shape, self.device = final_shape, device
        self.nlon = nlon
        self.rows = 1
        for d in spec_shape[:-1]:
            self.rows *= d
        self.fft_work = ops.rfft_workspace(self.rows, nlon, device) if self.rows > 0 else None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        # the output is allocated before the rfft is enqueued, so only the
        # pointer hand-off runs on the host between the two launches
        out = torch.empty(self.out_shape, dtype=torch.complex64, device=self.device)
        if self.fft_work is not None and x.is_contiguous():
            spec = torch.empty(self.spec_shape, dtype=torch.complex64, device=self.device)
            work = torch.empty(self.fft_work, dtype=torch.uint8, device=self.device) if self.fft_work else None
            self.plan.launch_rfft(x.data_ptr(), self.rows, self.nlon, spec.data_ptr(),
                                  0 if work is None else work.data_ptr(), self.fft_work, out.data_ptr())
            return out.view(self.final_shape)
        spec = _rfft(x).view(self.spec_shape)
        self.plan.launch_ptrs(spec.data_ptr(), out.data_ptr())
        return out.view(self.final_shape)


def _module_forward(module, x: torch.Tensor, comp_dims: int) -> torch.Tensor:
    """Forward of RealSHT (comp_dims 0) / RealVectorSHT (comp_dims 1)."""
    fast_ok = not (x.requires_grad and torch.is_grad_enabled())
    fast = module.__dict__.get("_fast_forward") if fast_ok else None
    if fast is not None:
        f = fast.get((x.shape, x.dtype, x.device))
        if f is not None:
            return f(x)
    what = "RealVectorSHT" if comp_dims else "RealSHT"
    _need_cuda(x, what)
    assert x.shape[-2] == module.nlat and x.shape[-1] == module.nlon and (not comp_dims or x.shape[-3] == 2)
    spec, scale, low = module._spectrum(x)
    lead = spec.shape[:-2 - comp_dims]
    flat = spec.reshape((_flat_batch(spec.shape, 2 + comp_dims),) + ((2,) if comp_dims else ())
                        + (module.nlat, spec.size(-1)))
    final = lead + ((2,) if comp_dims else ()) + (module.lmax, module.mmax)
    if not fast_ok:
        return _forward_coefficients(flat, module, low, scale).reshape(final)
    out, plan = _legendre_forward_planned(flat, module, low, scale)
    if (plan is not None and not low and x.dtype == torch.float32 and x.is_contiguous()
            and flat.data_ptr() == spec.data_ptr()):
        cache = module.__dict__.setdefault("_fast_forward", {})
        if len(cache) >= _MAX_PLANS:
            cache.clear()
        cache[(x.shape, x.dtype, x.device)] = _FastForward(plan, tuple(flat.shape), tuple(out.shape), final, x.device,
                                                           module.nlon)
    return out.reshape(final)


def _forward_coefficients(spec, src, round_bf16: bool, scale: float):
    """Module forward: through autograd only when a gradient is wanted."""
    if torch.is_grad_enabled() and spec.requires_grad:
        return _SpectrumLegendreForward.apply(spec, src, round_bf16, scale)
    return _legendre_forward(spec, src, round_bf16, scale)


class _SpectrumLegendreForward(torch.autograd.Function):
    """coef = 2*pi * Legendre(spec[..., :mmax]) for an rfft spectrum
    ``spec`` [B,(2),K,W]; backward is the transposed (conjugate for the
    vector map) contraction written straight into a [B,(2),K,W] gradient."""

    @staticmethod
    def forward(ctx, spec, src, round_bf16: bool, scale: float):
        out = _legendre_forward(spec, src, round_bf16, scale)
        ctx.src = src
        ctx.dims = (spec.size(0), spec.size(-2), spec.size(-1))
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, grad):
        src = ctx.src
        B, K, W = ctx.dims
        vector = src.vector
        g = grad.contiguous()
        shape = (B, 2, K, W) if vector else (B, K, W)
        gspec = torch.empty(shape, device=g.device, dtype=torch.complex64)
        if _dense_tc_eligible(src, B, _lib.DIR_INVERSE):
            ops.legendre_dense_tc(_lib.DIR_INVERSE, gspec, g, src.dense_table_split(_lib.DIR_INVERSE), nlat=K,
                                  lmax=src.lmax, mmax=src.mmax, scale=ctx.scale)
        else:
            _run(src, _lib.DIR_INVERSE, g, gspec, B, src.mmax, _strides3(g, vector), _strides3(gspec, vector),
                 W, ctx.scale, _lib.FLAG_CONJ_W1 if vector else 0)
        return gspec, None, None, None


class _SpectrumLegendreInverse(torch.autograd.Function):
    """spec[B,(2),K,W] = irfft-ready synthesis of coef [B,(2),L,M]: columns
    m >= M are zero and Im at m = 0 (and m = nlon/2 for even nlon) dropped."""

    @staticmethod
    def forward(ctx, coef, src, nlon: int):
        vector = src.vector
        B, L, M = coef.size(0), coef.size(-2), coef.size(-1)
        if (L, M) != (src.lmax, src.mmax):
            raise RuntimeError(f"coefficients are {L}x{M}, tables {src.lmax}x{src.mmax}")
        K = src.nlat
        W = nlon // 2 + 1
        c = coef.contiguous()
        shape = (B, 2, K, W) if vector else (B, K, W)
        spec = torch.empty(shape, device=c.device, dtype=torch.complex64)
        if getattr(src, "variant", "table") == "recurrence" and not vector:
            seeds, rc, ct = src.recurrence_tables()
            ops.legendre_inverse_recurrence(spec, c, seeds, rc, ct, 1.0, parity=getattr(src, "rec_parity", False),
                                            irfft_prep=True, nlon=nlon)
        elif _dense_tc_eligible(src, B, _lib.DIR_INVERSE):
            ops.legendre_dense_tc(_lib.DIR_INVERSE, spec, c, src.dense_table_split(_lib.DIR_INVERSE), nlat=K, lmax=L,
                                  mmax=M, scale=1.0, flags=_lib.FLAG_IRFFT_PREP, nlon=nlon)
        else:
            _run(src, _lib.DIR_INVERSE, c, spec, B, M, _strides3(c, vector), _strides3(spec, vector),
                 W, 1.0, _lib.FLAG_IRFFT_PREP, nlon)
        ctx.src = src
        ctx.dims = (B, K, W, L, M)
        ctx.nyq = nlon // 2 if nlon % 2 == 0 else None
        return spec

    @staticmethod
    def backward(ctx, grad):
        src = ctx.src
        B, K, W, L, M = ctx.dims
        vector = src.vector
        g = grad.clone(memory_format=torch.contiguous_format)
        # adjoint of dropping Im at m = 0 / m = nlon/2: drop it from the gradient
        g[..., 0] = g[..., 0].real.to(g.dtype)
        if ctx.nyq is not None:
            g[..., ctx.nyq] = g[..., ctx.nyq].real.to(g.dtype)
        shape = (B, 2, L, M) if vector else (B, L, M)
        gc = torch.empty(shape, device=g.device, dtype=torch.complex64)
        if _dense_tc_eligible(src, B, _lib.DIR_FORWARD):
            ops.legendre_dense_tc(_lib.DIR_FORWARD, gc, g, src.dense_table_split(_lib.DIR_FORWARD), nlat=K, lmax=L,
                                  mmax=M, scale=1.0)
        else:
            _run(src, _lib.DIR_FORWARD, g, gc, B, M, _strides3(g, vector), _strides3(gc, vector),
                 M, 1.0, _lib.FLAG_CONJ_W1 if vector else 0)
        return gc, None, None


# ---------------------------------------------------------------------------
# operator-level autograd functions (reference layouts, :976-1093)
# ---------------------------------------------------------------------------

def _dense_contract(kind, direction, inp, out, w0, w1, conj=False):
    vector = kind == _lib.KIND_VECTOR
    L, K, M = w0.shape
    _contract(kind=kind, direction=direction, input=inp, output=out, w0=w0, w1=w1, batch=inp.size(0),
              nlat=K, lmax=L, mmax=M, in_strides=_strides3(inp, vector),
              out_strides=_strides3(out, vector), out_cols=M, scale=1.0,
              flags=_lib.FLAG_CONJ_W1 if conj else 0)


class _FusedLegendreForwardFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, weight_t):
        x = input.contiguous()
        out = torch.empty(x.size(0), weight_t.size(0), x.size(2), device=x.device, dtype=torch.complex64)
        ops.fused_legendre_forward(out, x, weight_t)
        ctx.save_for_backward(weight_t)
        return out

    @staticmethod
    def backward(ctx, grad):
        (weight_t,) = ctx.saved_tensors
        g = grad.contiguous()
        gi = torch.empty(g.size(0), weight_t.size(1), g.size(2), device=g.device, dtype=torch.complex64)
        ops.fused_legendre_inverse(gi, g, weight_t)
        return gi, None


class _FusedLegendreInverseFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, weight_t):
        x = input.contiguous()
        out = torch.empty(x.size(0), weight_t.size(1), x.size(2), device=x.device, dtype=torch.complex64)
        ops.fused_legendre_inverse(out, x, weight_t)
        ctx.save_for_backward(weight_t)
        return out

    @staticmethod
    def backward(ctx, grad):
        (weight_t,) = ctx.saved_tensors
        g = grad.contiguous()
        gi = torch.empty(g.size(0), weight_t.size(0), g.size(2), device=g.device, dtype=torch.complex64)
        ops.fused_legendre_forward(gi, g, weight_t)
        return gi, None


class _FusedLegendreForwardRealFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, weight_t):
        x = input.contiguous()
        out = torch.empty(x.size(0), weight_t.size(0), x.size(2), device=x.device, dtype=torch.float32)
        ops.fused_legendre_forward_real(out, x, weight_t)
        ctx.save_for_backward(weight_t)
        ctx.in_dtype = x.dtype
        return out

    @staticmethod
    def backward(ctx, grad):
        (weight_t,) = ctx.saved_tensors
        g = grad.contiguous().float()
        gi = torch.empty(g.size(0), weight_t.size(1), g.size(2), device=g.device, dtype=torch.float32)
        ops.fused_legendre_inverse_real(gi, g, weight_t)
        return gi.to(ctx.in_dtype), None


class _FusedVectorLegendreForwardFn(torch.autograd.Function):
    """Backward applies the conjugate transpose A^H = [[W0, -iW1], [-iW1, -W0]]
    (PyTorch's complex-gradient convention).  The reference applies A^T here
    (``__init__.py:1061-1069``), which is not the adjoint."""

    @staticmethod
    def forward(ctx, input, weight0_t, weight1_t):
        x = input.contiguous()
        out = torch.empty(x.size(0), 2, weight0_t.size(0), x.size(3), device=x.device, dtype=torch.complex64)
        ops.fused_vector_legendre_forward(out, x, weight0_t, weight1_t)
        ctx.save_for_backward(weight0_t, weight1_t)
        return out

    @staticmethod
    def backward(ctx, grad):
        w0, w1 = ctx.saved_tensors
        g = grad.contiguous()
        gi = torch.empty(g.size(0), 2, w0.size(1), g.size(3), device=g.device, dtype=torch.complex64)
        _dense_contract(_lib.KIND_VECTOR, _lib.DIR_INVERSE, g, gi, w0, w1, conj=True)
        return gi, None, None


class _FusedVectorLegendreInverseFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, weight0_t, weight1_t):
        x = input.contiguous()
        out = torch.empty(x.size(0), 2, weight0_t.size(1), x.size(3), device=x.device, dtype=torch.complex64)
        ops.fused_vector_legendre_inverse(out, x, weight0_t, weight1_t)
        ctx.save_for_backward(weight0_t, weight1_t)
        return out

    @staticmethod
    def backward(ctx, grad):
        w0, w1 = ctx.saved_tensors
        g = grad.contiguous()
        gi = torch.empty(g.size(0), 2, w0.size(0), g.size(3), device=g.device, dtype=torch.complex64)
        _dense_contract(_lib.KIND_VECTOR, _lib.DIR_FORWARD, g, gi, w0, w1, conj=True)
        return gi, None, None


# ---------------------------------------------------------------------------
# function API (reference :1100-1221)
# ---------------------------------------------------------------------------

def _as_weight_t(weights: torch.Tensor, weight_t: Optional[torch.Tensor]) -> torch.Tensor:
    if weight_t is None:
        weight_t = weights.float().permute(1, 2, 0).contiguous()
    return weight_t


def fused_legendre_forward(input: torch.Tensor, weights: torch.Tensor,
                           weight_t: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[b,l,m] = sum_k weights[m,l,k] input[b,k,m]; input [B,nlat,mmax] complex64,
    weights [mmax,lmax,nlat] (torch-harmonics layout) or weight_t [lmax,nlat,mmax]."""
    _need_cuda(input, "fused_legendre_forward")
    return _FusedLegendreForwardFn.apply(input, _as_weight_t(weights, weight_t))


def fused_legendre_inverse(input: torch.Tensor, pct: torch.Tensor,
                           pct_t: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[b,k,m] = sum_l pct[m,l,k] input[b,l,m]; input [B,lmax,mmax] complex64."""
    _need_cuda(input, "fused_legendre_inverse")
    return _FusedLegendreInverseFn.apply(input, _as_weight_t(pct, pct_t))


def fused_legendre_forward_real(input: torch.Tensor, weight_t: torch.Tensor) -> torch.Tensor:
    """Real-valued forward Legendre transform with float accumulation."""
    _need_cuda(input, "fused_legendre_forward_real")
    return _FusedLegendreForwardRealFn.apply(input, weight_t)


def fused_legendre_inverse_real(input: torch.Tensor, weight_t: torch.Tensor) -> torch.Tensor:
    """Real-valued inverse Legendre transform with float accumulation."""
    _need_cuda(input, "fused_legendre_inverse_real")
    x = input.contiguous().float()
    out = torch.empty(x.size(0), weight_t.size(1), x.size(2), device=x.device, dtype=torch.float32)
    ops.fused_legendre_inverse_real(out, x, weight_t)
    return out


def fused_sht_forward(x: torch.Tensor, weights: torch.Tensor, mmax: int,
                      weight_t: Optional[torch.Tensor] = None) -> torch.Tensor:
    """rfft -> Legendre: [B, nlat, nlon] float32 -> [B, lmax, mmax] complex64."""
    _need_cuda(x, "fused_sht_forward")
    spec = _rfft(x.float())
    lead = spec.shape[:-2]
    spec = spec.reshape(_flat_batch(spec.shape, 2), spec.size(-2), spec.size(-1))
    wt = _as_weight_t(weights, weight_t)
    if wt.size(2) != int(mmax):
        raise RuntimeError(f"weight_t has mmax={wt.size(2)}, expected {int(mmax)}")
    out = _SpectrumLegendreForward.apply(spec, _DenseTables(wt), False, TWO_PI / x.size(-1))
    return out.reshape(lead + out.shape[-2:])


def fused_sht_inverse(coeffs: torch.Tensor, pct: torch.Tensor, nlon: int,
                      pct_t: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Legendre -> irfft: [B, lmax, mmax] complex64 -> [B, nlat, nlon] float32."""
    _need_cuda(coeffs, "fused_sht_inverse")
    lead = coeffs.shape[:-2]
    c = coeffs.reshape(_flat_batch(coeffs.shape, 2), coeffs.size(-2), coeffs.size(-1))
    if c.dtype != torch.complex64:
        c = c.to(torch.complex64)
    spec = _SpectrumLegendreInverse.apply(c, _DenseTables(_as_weight_t(pct, pct_t)), int(nlon))
    y = _irfft(spec, int(nlon))
    return y.reshape(lead + y.shape[-2:])


def _prepare_irfft_input(x: torch.Tensor, nlon: int, active_mmax: Optional[int] = None) -> torch.Tensor:
    """Pad an rFFT-format complex tensor to nlon//2+1 and drop Im at DC/Nyquist
    (reference ``__init__.py:949-973``), on the native kernel."""
    _need_cuda(x, "_prepare_irfft_input")
    active_mmax = x.size(-1) if active_mmax is None else active_mmax
    full = nlon // 2 + 1
    if x.size(-1) == full:
        out = x.contiguous().clone() if x.is_contiguous() else x.contiguous()
    else:
        out = torch.zeros(x.shape[:-1] + (full,), dtype=x.dtype, device=x.device)
        n = min(full, x.size(-1))
        out[..., :n] = x[..., :n]
    flat = out.reshape(_flat_batch(out.shape, 2), out.size(-2), out.size(-1))
    ops.sht_prepare_irfft(flat, active_mmax, nlon)
    return flat.reshape(out.shape)


def _stack_vector_forward_real_inputs(input: torch.Tensor):
    """[B,2,K,M] complex64 -> (stacked_w0, stacked_w1) [4B,K,M] (reference :429-445)."""
    _need_cuda(input, "_stack_vector_forward_real_inputs")
    B, _, K, M = input.shape
    s0 = torch.empty((4 * B, K, M), device=input.device, dtype=torch.float32)
    s1 = torch.empty_like(s0)
    ops.fused_vector_forward_pack_real(s0, s1, input.contiguous())
    return s0, s1


def _recompose_vector_forward_real_outputs(out_w0, out_w1, *, batch_size: int, lmax: int, mmax: int):
    """Inverse of the packing above on the two real outputs (reference :448-477)."""
    _need_cuda(out_w0, "_recompose_vector_forward_real_outputs")
    out = torch.empty((batch_size, 2, lmax, mmax), device=out_w0.device, dtype=torch.complex64)
    ops.fused_vector_forward_recompose_real(out, out_w0.contiguous(), out_w1.contiguous())
    return out


# ---------------------------------------------------------------------------
# modules (reference :1228-1791)
# ---------------------------------------------------------------------------

def _w_dtype(dtype: str) -> torch.dtype:
    if dtype == "fp32":
        return torch.float32
    if dtype == "bf16":
        return torch.bfloat16
    if dtype == "fp16":
        return torch.float16
    raise ValueError(f"dtype must be 'fp32', 'bf16' or 'fp16', got {dtype!r}")


def _check_mmax(mmax: int, nlon: int) -> None:
    if mmax > nlon // 2 + 1:
        raise ValueError(f"mmax={mmax} exceeds nlon//2+1={nlon // 2 + 1}")


class RealSHT(_GroupedTablesMixin, nn.Module):
    """Drop-in ``RealSHT``: ``x`` [..., nlat, nlon] real -> [..., lmax, mmax] complex64.

    ``dtype="bf16"`` rounds the post-FFT spectrum to bfloat16 and contracts it
    with the FP32 table in FP32 (the reference's BF16 path, ``__init__.py:1289-1337``).
    ``variant="recurrence"`` (an addition) computes the Legendre functions on the
    fly in the forward pass instead of streaming the table (the backward pass
    uses the table).  ``table_device`` (an addition, every module) runs the
    float64 table recurrence on that device and keeps the tables there (a GPU
    builds the 1024 x 2048 tables in about a second; default: the host, as the
    reference does through torch-harmonics).
    """

    def __init__(self, nlat: int, nlon: int, lmax: Optional[int] = None, mmax: Optional[int] = None,
                 grid: str = "equiangular", norm: str = "ortho", csphase: bool = True,
                 dtype: str = "fp32", variant: str = "table", table_device=None):
        super().__init__()
        if variant not in ("table", "recurrence"):
            raise ValueError(f"variant must be 'table' or 'recurrence', got {variant!r}")
        self.variant = variant
        w_dtype = _w_dtype(dtype)
        w, L, M = _weights.scalar_forward(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        _check_mmax(M, nlon)
        self.nlat, self.nlon, self.lmax, self.mmax = nlat, nlon, L, M
        self.grid, self.norm, self.csphase = grid, norm, csphase
        self._use_bf16 = dtype == "bf16"
        self._use_fp16 = dtype == "fp16"
        wt = torch.from_numpy(w) if table_device is None else w
        self.register_buffer("weights", wt.to(w_dtype))
        self.register_buffer("weight_t", wt.permute(1, 2, 0).contiguous())
        self._mlk_name = "weights"
        self._init_tables(("weight_t",), _lib.DIR_FORWARD)
        if variant == "recurrence":
            seeds, coef, ct = _weights.scalar_recurrence_tables(nlat, nlon, lmax, mmax, grid, norm, csphase)
            self.rec_parity = _weights.recurrence_seeds_symmetric(seeds, ct)
            seeds = _weights.compact_recurrence_seeds(seeds, coef.shape[1])
            self.register_buffer("rec_seeds", torch.from_numpy(seeds), persistent=False)
            self.register_buffer("rec_coef", torch.from_numpy(coef), persistent=False)
            self.register_buffer("rec_cos_theta", torch.from_numpy(ct), persistent=False)

    def recurrence_tables(self):
        return self.rec_seeds, self.rec_coef, self.rec_cos_theta

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _module_forward(self, x, 0)


class InverseRealSHT(_GroupedTablesMixin, nn.Module):
    """Drop-in ``InverseRealSHT``: [..., lmax, mmax] complex -> [..., nlat, nlon] real."""

    def __init__(self, nlat: int, nlon: int, lmax: Optional[int] = None, mmax: Optional[int] = None,
                 grid: str = "equiangular", norm: str = "ortho", csphase: bool = True, table_device=None,
                 variant: str = "table"):
        super().__init__()
        if variant not in ("table", "recurrence"):
            raise ValueError(f"variant must be 'table' or 'recurrence', got {variant!r}")
        self.variant = variant
        p, L, M = _weights.scalar_inverse(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        _check_mmax(M, nlon)
        self.nlat, self.nlon, self.lmax, self.mmax = nlat, nlon, L, M
        self.grid, self.norm, self.csphase = grid, norm, csphase
        pt = torch.from_numpy(p) if table_device is None else p
        self.register_buffer("pct", pt)
        self.register_buffer("pct_t", pt.permute(1, 2, 0).contiguous())
        self._mlk_name = "pct"
        self._init_tables(("pct_t",), _lib.DIR_INVERSE)
        if variant == "recurrence":
            # the synthesis from functions generated in registers (the gradient
            # keeps to the table path)
            seeds, coef, ct = _weights.scalar_recurrence_tables(nlat, nlon, lmax, mmax, grid, norm, csphase,
                                                                inverse=True, segment=8)
            self.rec_parity = _weights.recurrence_seeds_symmetric(seeds, ct)
            self.register_buffer("rec_seeds", torch.from_numpy(seeds), persistent=False)
            self.register_buffer("rec_coef", torch.from_numpy(coef), persistent=False)
            self.register_buffer("rec_cos_theta", torch.from_numpy(ct), persistent=False)

    def recurrence_tables(self):
        return self.rec_seeds, self.rec_coef, self.rec_cos_theta

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _need_cuda(x, "InverseRealSHT")
        assert x.shape[-2] == self.lmax and x.shape[-1] == self.mmax
        lead = x.shape[:-2]
        c = x.reshape(_flat_batch(x.shape, 2), self.lmax, self.mmax)
        if c.dtype != torch.complex64:
            c = c.to(torch.complex64)
        spec = _SpectrumLegendreInverse.apply(c, self, self.nlon)
        y = _irfft(spec, self.nlon)
        return y.reshape(lead + (self.nlat, self.nlon))


class RealVectorSHT(_GroupedTablesMixin, nn.Module):
    """Drop-in ``RealVectorSHT``: [..., 2, nlat, nlon] -> [..., 2, lmax, mmax] complex64
    (spheroidal, toroidal), both tables fused in one pass.

    ``variant="recurrence"`` (an addition) generates the two vector tables on the
    fly in the forward pass from the Legendre recurrences of orders m - 1 and
    m + 1 (ladder identities) instead of streaming them (the backward pass uses
    the tables)."""

    def __init__(self, nlat: int, nlon: int, lmax: Optional[int] = None, mmax: Optional[int] = None,
                 grid: str = "equiangular", norm: str = "ortho", csphase: bool = True,
                 dtype: str = "fp32", variant: str = "table", table_device=None):
        super().__init__()
        if variant not in ("table", "recurrence"):
            raise ValueError(f"variant must be 'table' or 'recurrence', got {variant!r}")
        self.variant = variant
        w_dtype = _w_dtype(dtype)
        w, L, M = _weights.vector_forward(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        _check_mmax(M, nlon)
        self.nlat, self.nlon, self.lmax, self.mmax = nlat, nlon, L, M
        self.grid, self.norm, self.csphase = grid, norm, csphase
        self._use_bf16 = dtype == "bf16"
        self._use_fp16 = dtype == "fp16"
        wt = torch.from_numpy(w) if table_device is None else w
        self.register_buffer("w0", wt[0].to(w_dtype))
        self.register_buffer("w1", wt[1].to(w_dtype))
        self.register_buffer("w0_t", wt[0].permute(1, 2, 0).contiguous())
        self.register_buffer("w1_t", wt[1].permute(1, 2, 0).contiguous())
        self._mlk_name = "w0"
        self._init_tables(("w0_t", "w1_t"), _lib.DIR_FORWARD)
        if variant == "recurrence":
            seeds, coef, ct = _weights.vector_recurrence_tables(nlat, nlon, lmax, mmax, grid, norm, csphase)
            self.rec_parity = _weights.recurrence_seeds_symmetric(seeds, ct)
            seeds = _weights.compact_recurrence_seeds(seeds, coef.shape[1])
            self.register_buffer("rec_seeds", torch.from_numpy(seeds), persistent=False)
            self.register_buffer("rec_coef", torch.from_numpy(coef), persistent=False)
            self.register_buffer("rec_cos_theta", torch.from_numpy(ct), persistent=False)

    def recurrence_tables(self):
        return self.rec_seeds, self.rec_coef, self.rec_cos_theta

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _module_forward(self, x, 1)


class InverseRealVectorSHT(_GroupedTablesMixin, nn.Module):
    """Drop-in ``InverseRealVectorSHT``: [..., 2, lmax, mmax] -> [..., 2, nlat, nlon]."""

    def __init__(self, nlat: int, nlon: int, lmax: Optional[int] = None, mmax: Optional[int] = None,
                 grid: str = "equiangular", norm: str = "ortho", csphase: bool = True, table_device=None):
        super().__init__()
        d, L, M = _weights.vector_inverse(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                          device=table_device)
        _check_mmax(M, nlon)
        self.nlat, self.nlon, self.lmax, self.mmax = nlat, nlon, L, M
        self.grid, self.norm, self.csphase = grid, norm, csphase
        dt = torch.from_numpy(d) if table_device is None else d
        self.register_buffer("d0", dt[0].contiguous())
        self.register_buffer("d1", dt[1].contiguous())
        self.register_buffer("d0_t", dt[0].permute(1, 2, 0).contiguous())
        self.register_buffer("d1_t", dt[1].permute(1, 2, 0).contiguous())
        self._mlk_name = "d0"
        self._init_tables(("d0_t", "d1_t"), _lib.DIR_INVERSE)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _need_cuda(x, "InverseRealVectorSHT")
        assert x.shape[-2] == self.lmax and x.shape[-1] == self.mmax and x.shape[-3] == 2
        lead = x.shape[:-3]
        c = x.reshape(_flat_batch(x.shape, 3), 2, self.lmax, self.mmax)
        if c.dtype != torch.complex64:
            c = c.to(torch.complex64)
        spec = _SpectrumLegendreInverse.apply(c, self, self.nlon)
        y = _irfft(spec, self.nlon)
        return y.reshape(lead + (2, self.nlat, self.nlon))


class GraphedModule(nn.Module):
    """CUDA-graph capture/replay of a module's forward (reference :1794-1866).

    The first call per (shape, dtype) warms the module up on a side stream and
    captures one graph; later calls copy the input into the captured buffer,
    replay and return a clone of the captured output.  Inputs off CUDA or
    requiring grad run the module directly.  At most ``max_cached_shapes``
    graphs are kept (least recently used is dropped).
    """

    def __init__(self, module: nn.Module, num_warmup: int = 3, max_cached_shapes: int = 4):
        super().__init__()
        self.module = module
        self._num_warmup = num_warmup
        self._max_cached_shapes = max_cached_shapes
        self._graph_cache = {}
        self._graph_lru = []

    def reset_graph_cache(self) -> None:
        self._graph_cache.clear()
        self._graph_lru.clear()

    def _capture(self, x: torch.Tensor):
        static_in = x.detach().clone()
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(self._num_warmup):
                self.module(static_in)
        torch.cuda.current_stream(x.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = self.module(static_in)
        return static_in, static_out, graph

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or x.requires_grad:
            return self.module(x)
        key = (tuple(x.shape), x.dtype, x.device)
        entry = self._graph_cache.get(key)
        if entry is None:
            entry = self._capture(x)
            self._graph_cache[key] = entry
            self._graph_lru.append(key)
            while len(self._graph_lru) > self._max_cached_shapes:
                self._graph_cache.pop(self._graph_lru.pop(0), None)
        else:
            self._graph_lru.remove(key)
            self._graph_lru.append(key)
        static_in, static_out, graph = entry
        static_in.copy_(x)
        graph.replay()
        return static_out.clone()


legendre_forward = fused_legendre_forward
legendre_inverse = fused_legendre_inverse
sht_forward = fused_sht_forward
sht_inverse = fused_sht_inverse

FusedRealSHT = RealSHT
FusedInverseRealSHT = InverseRealSHT
FusedRealVectorSHT = RealVectorSHT
FusedInverseRealVectorSHT = InverseRealVectorSHT
