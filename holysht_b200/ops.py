"""Reference-named operators over the C ABI.

Each function here has the name, argument order and in-place semantics of
one operator of the reference's torch binding (``torch-ext/torch_binding.cpp``
:12-24): the caller allocates ``output``, the operator fills it on the
current CUDA stream.  Argument checks raise ``RuntimeError`` for the same
conditions the reference's ``TORCH_CHECK``s reject
(``cuda/fused_legendre.cu:3157-3335``).

``legendre_contract`` is the strided entry the modules use (no reference
counterpart): it reads the rfft output in place, folds the 2*pi spectrum
scale, writes irfft-ready buffers and runs the conjugate-transpose vector map.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional

import torch

from . import _lib

__all__ = [
    "fused_legendre_forward",
    "fused_legendre_inverse",
    "fused_legendre_forward_real",
    "fused_legendre_forward_real_ex",
    "fused_legendre_inverse_real",
    "fused_vector_legendre_forward",
    "fused_vector_legendre_forward_ex",
    "fused_vector_legendre_inverse",
    "fused_vector_forward_pack_real",
    "fused_vector_forward_recompose_real",
    "sht_prepare_irfft",
    "legendre_contract",
    "ContractPlan",
    "tile_table",
    "group_table",
    "group_table8",
    "stream_error_word",
    "stream_launch_plan",
    "legendre_dense_tc",
    "tc_error_word",
    "legendre_forward_recurrence",
    "legendre_vector_forward_recurrence",
    "legendre_inverse_recurrence",
]


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        _require(t.is_cuda, "holysht_b200 operators take CUDA tensors only")
        _require(t.device == dev, "all tensors must be on the same CUDA device")
    return dev


def _contig(*ts: torch.Tensor) -> None:
    for t in ts:
        _require(t.is_contiguous(), "tensors must be contiguous")


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check_scalar(output, input, weight_t, inverse: bool, in_dtypes, out_dtype, what):
    dev = _cuda(output, input, weight_t)
    _contig(output, input, weight_t)
    _require(input.dtype in in_dtypes, f"{what}: input has dtype {input.dtype}")
    _require(output.dtype == out_dtype, f"{what}: output must be {out_dtype}")
    _require(weight_t.dtype == torch.float32, f"{what}: weight must be float32")
    _require(input.dim() == 3, f"{what}: input must be rank 3")
    _require(output.dim() == 3, f"{what}: output must be rank 3")
    _require(weight_t.dim() == 3, f"{what}: weight_t must be rank 3")
    L, K, M = weight_t.shape
    B = input.size(0)
    if not inverse:
        _require(input.size(1) == K, "weight dim 1 must match nlat")
        _require(input.size(2) == M, "weight dim 2 must match mmax")
        _require(tuple(output.shape) == (B, L, M), "output must be [batch, lmax, mmax]")
    else:
        _require(input.size(1) == L, "weight dim 0 must match lmax")
        _require(input.size(2) == M, "weight dim 2 must match mmax")
        _require(tuple(output.shape) == (B, K, M), "output must be [batch, nlat, mmax]")
    return dev, B, K, L, M


def _check_vector(output, input, w0, w1, inverse: bool, what):
    dev = _cuda(output, input, w0, w1)
    _contig(output, input, w0, w1)
    _require(input.dtype == torch.complex64 and output.dtype == torch.complex64,
             f"{what}: input and output must be complex64")
    _require(w0.dtype == torch.float32 and w1.dtype == torch.float32, f"{what}: weights must be float32")
    _require(input.dim() == 4 and output.dim() == 4, f"{what}: input and output must be rank 4")
    _require(input.size(1) == 2 and output.size(1) == 2, f"{what}: component dimension must be 2")
    _require(w0.dim() == 3 and w0.shape == w1.shape, f"{what}: weights must be matching rank-3 tensors")
    L, K, M = w0.shape
    B = input.size(0)
    if not inverse:
        _require(input.size(2) == K and input.size(3) == M, "input must be [batch, 2, nlat, mmax]")
        _require(tuple(output.shape) == (B, 2, L, M), "output must be [batch, 2, lmax, mmax]")
    else:
        _require(input.size(2) == L and input.size(3) == M, "input must be [batch, 2, lmax, mmax]")
        _require(tuple(output.shape) == (B, 2, K, M), "output must be [batch, 2, nlat, mmax]")
    return dev, B, K, L, M


def fused_legendre_forward(output: torch.Tensor, input: torch.Tensor, weight_t: torch.Tensor) -> None:
    dev, B, K, L, M = _check_scalar(output, input, weight_t, False, (torch.complex64,),
                                    torch.complex64, "fused_legendre_forward")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_legendre_forward(
            _p(output), _p(input), _p(weight_t), B, K, L, M, _stream(dev)))


def fused_legendre_inverse(output: torch.Tensor, input: torch.Tensor, weight_t: torch.Tensor) -> None:
    dev, B, K, L, M = _check_scalar(output, input, weight_t, True, (torch.complex64,),
                                    torch.complex64, "fused_legendre_inverse")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_legendre_inverse(
            _p(output), _p(input), _p(weight_t), B, K, L, M, _stream(dev)))


def fused_legendre_forward_real_ex(output: torch.Tensor, input: torch.Tensor, weight_t: torch.Tensor,
                                   backend_hint: int) -> None:
    dev, B, K, L, M = _check_scalar(output, input, weight_t, False, (torch.float32, torch.bfloat16),
                                    torch.float32, "fused_legendre_forward_real")
    dt = _lib.DTYPE_BF16 if input.dtype == torch.bfloat16 else _lib.DTYPE_F32
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_legendre_forward_real(
            _p(output), _p(input), dt, _p(weight_t), B, K, L, M, int(backend_hint), _stream(dev)))


def fused_legendre_forward_real(output: torch.Tensor, input: torch.Tensor, weight_t: torch.Tensor) -> None:
    fused_legendre_forward_real_ex(output, input, weight_t, 0)


def fused_legendre_inverse_real(output: torch.Tensor, input: torch.Tensor, weight_t: torch.Tensor) -> None:
    dev, B, K, L, M = _check_scalar(output, input, weight_t, True, (torch.float32,), torch.float32,
                                    "fused_legendre_inverse_real")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_legendre_inverse_real(
            _p(output), _p(input), _p(weight_t), B, K, L, M, _stream(dev)))


def fused_vector_legendre_forward_ex(output: torch.Tensor, input: torch.Tensor, weight0_t: torch.Tensor,
                                     weight1_t: torch.Tensor, backend_hint: int) -> None:
    dev, B, K, L, M = _check_vector(output, input, weight0_t, weight1_t, False,
                                    "fused_vector_legendre_forward")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_vector_legendre_forward(
            _p(output), _p(input), _p(weight0_t), _p(weight1_t), B, K, L, M, int(backend_hint),
            _stream(dev)))


def fused_vector_legendre_forward(output: torch.Tensor, input: torch.Tensor, weight0_t: torch.Tensor,
                                  weight1_t: torch.Tensor) -> None:
    fused_vector_legendre_forward_ex(output, input, weight0_t, weight1_t, 0)


def fused_vector_legendre_inverse(output: torch.Tensor, input: torch.Tensor, weight0_t: torch.Tensor,
                                  weight1_t: torch.Tensor) -> None:
    dev, B, K, L, M = _check_vector(output, input, weight0_t, weight1_t, True,
                                    "fused_vector_legendre_inverse")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_vector_legendre_inverse(
            _p(output), _p(input), _p(weight0_t), _p(weight1_t), B, K, L, M, _stream(dev)))


def fused_vector_forward_pack_real(stacked_w0: torch.Tensor, stacked_w1: torch.Tensor,
                                   input: torch.Tensor) -> None:
    dev = _cuda(stacked_w0, stacked_w1, input)
    _contig(stacked_w0, stacked_w1, input)
    _require(input.dtype == torch.complex64, "input must be complex64")
    _require(stacked_w0.dtype == torch.float32, "stacked_w0 must be float32")
    _require(stacked_w1.dtype == torch.float32, "stacked_w1 must be float32")
    _require(input.dim() == 4, "input must be rank 4")
    _require(input.size(1) == 2, "input component dimension must be 2")
    _require(stacked_w0.dim() == 3 and stacked_w1.dim() == 3, "stacked outputs must be rank 3")
    B, _, K, M = input.shape
    _require(stacked_w0.shape == stacked_w1.shape, "stacked outputs must match")
    _require(tuple(stacked_w0.shape) == (4 * B, K, M), "stacked outputs must be [4*batch, nlat, mmax]")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_vector_forward_pack_real(
            _p(stacked_w0), _p(stacked_w1), _p(input), B, K, M, _stream(dev)))


def fused_vector_forward_recompose_real(output: torch.Tensor, out_w0: torch.Tensor,
                                        out_w1: torch.Tensor) -> None:
    dev = _cuda(output, out_w0, out_w1)
    _contig(output, out_w0, out_w1)
    _require(output.dtype == torch.complex64, "output must be complex64")
    _require(out_w0.dtype == torch.float32 and out_w1.dtype == torch.float32, "real outputs must be float32")
    _require(output.dim() == 4 and output.size(1) == 2, "output must be [batch, 2, lmax, mmax]")
    _require(out_w0.dim() == 3 and out_w0.shape == out_w1.shape, "real outputs must match")
    _require(out_w0.size(0) % 4 == 0, "real output batch dimension must be divisible by 4")
    B, _, L, M = output.shape
    _require(tuple(out_w0.shape) == (4 * B, L, M), "real outputs must be [4*batch, lmax, mmax]")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_fused_vector_forward_recompose_real(
            _p(output), _p(out_w0), _p(out_w1), B, L, M, _stream(dev)))


def sht_prepare_irfft(data: torch.Tensor, mmax: int, nlon: int) -> None:
    dev = _cuda(data)
    _contig(data)
    _require(data.dtype == torch.complex64, "data must be complex64")
    _require(data.dim() == 3, "data must be rank 3")
    rows = data.size(0) * data.size(1)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_sht_prepare_irfft(
            _p(data), rows, data.size(2), int(mmax), int(nlon), _stream(dev)))


def tile_table(weight_t: torch.Tensor) -> torch.Tensor:
    """[lmax, nlat, mmax] -> m-tiled [lmax, ceil(mmax/32), nlat, 32] (orders
    padded with zeros): every 32-order row segment starts a 128-byte line, so
    each warp-wide table load is exactly one aligned line."""
    L, K, M = weight_t.shape
    mt = (M + 31) // 32
    padded = torch.zeros((L, K, mt * 32), dtype=torch.float32, device=weight_t.device)
    padded[..., :M] = weight_t
    return padded.view(L, K, mt, 32).permute(0, 2, 1, 3).contiguous()


def group_table(tables, direction: int, conj: bool = False, m_offset: int = 0) -> torch.Tensor:
    """Row-grouped table for the contraction kernel (``HOLYSHT_TABLE_GROUPED``).

    ``tables``: one dense [lmax, nlat, mmax] table, or a (W0, W1) pair for the
    vector kind.  ``direction``: ``DIR_FORWARD`` (rows = l, steps = k) or
    ``DIR_INVERSE`` (rows = k, steps = l).  Result [R/4, ceil(M/32), S, 32, 4, T]:
    per 4-row group, m tile and step, the 32 lanes' rows x tables are
    contiguous, zero outside the tables and above the diagonal (l < m, with m
    the global order ``m_offset + column``: the kernel streams whole blocks
    without per-entry predicates, so the zeros are part of the layout).  A
    vector pair is stored as (W0 + s W1, W0 - s W1), s = -1 when ``conj`` (the
    conjugate-transpose map autograd needs), which is the form the kernel
    contracts."""
    if torch.is_tensor(tables):
        tables = (tables,)
    if len(tables) == 2:
        w0, w1 = tables
        s1 = -1.0 if conj else 1.0
        tables = (w0 + s1 * w1, w0 - s1 * w1)
    L, K, M = tables[0].shape
    mt = (M + 31) // 32
    fwd = direction == _lib.DIR_FORWARD
    R, S = (L, K) if fwd else (K, L)
    rg = (R + 3) // 4
    dev = tables[0].device
    out = torch.zeros((rg, mt, S, 32, 4, len(tables)), dtype=torch.float32, device=dev)
    tri = (torch.arange(M, device=dev)[None, :] + m_offset <= torch.arange(L, device=dev)[:, None])
    for t, w in enumerate(tables):
        _require(tuple(w.shape) == (L, K, M) and w.dtype == torch.float32, "tables must match, float32")
        pad = torch.zeros((rg * 4 if fwd else L, K if fwd else rg * 4, mt * 32), dtype=torch.float32, device=dev)
        pad[:L, :K, :M] = w * tri[:, None, :]
        if fwd:   # [l, k, m] -> [g, r, k, mt, lane] -> [g, mt, k, lane, r]
            v = pad.view(rg, 4, K, mt, 32).permute(0, 3, 2, 4, 1)
        else:     # [l, k, m] -> [l, g, r, mt, lane] -> [g, mt, l, lane, r]
            v = pad.view(L, rg, 4, mt, 32).permute(1, 3, 0, 4, 2)
        out[..., t] = v
    return out


def group_table8(tables, direction: int, conj: bool = False, m_offset: int = 0, combine: bool = True) -> torch.Tensor:
    """Table in the ``HOLYSHT_TABLE_GROUPED8`` layout of the streaming kernel.

    Rows (l for ``DIR_FORWARD``, k for ``DIR_INVERSE``) in groups of 8; per
    group, 32-order m tile and reduction step, each lane's 8 rows x T tables
    are stored as 2T quads of 4 floats, quad-major across the lanes:
    result [ceil(R/8), ceil(M/32), S, 2T, 32, 4].  Vector quads hold
    (row 2q: W0 + s W1, W0 - s W1, row 2q+1: the same), s = -1 when ``conj``;
    scalar quads hold rows 4q .. 4q+3.  Zero outside the tables and above the
    diagonal (l < m_offset + column)."""
    if torch.is_tensor(tables):
        tables = (tables,)
    if len(tables) == 2 and combine:  # combine=False keeps (W0, W1) as they are
        w0, w1 = tables
        s1 = -1.0 if conj else 1.0
        tables = (w0 + s1 * w1, w0 - s1 * w1)
    L, K, M = tables[0].shape
    T = len(tables)
    mt = (M + 31) // 32
    fwd = direction == _lib.DIR_FORWARD
    R, S = (L, K) if fwd else (K, L)
    rg = (R + 7) // 8
    dev = tables[0].device
    x = torch.zeros((rg, mt, S, 32, 8, T), dtype=torch.float32, device=dev)
    tri = (torch.arange(M, device=dev)[None, :] + m_offset <= torch.arange(L, device=dev)[:, None])
    for t, w in enumerate(tables):
        _require(tuple(w.shape) == (L, K, M) and w.dtype == torch.float32, "tables must match, float32")
        pad = torch.zeros((rg * 8 if fwd else L, K if fwd else rg * 8, mt * 32), dtype=torch.float32, device=dev)
        pad[:L, :K, :M] = w * tri[:, None, :]
        if fwd:   # [l, k, m] -> [g, r, k, mt, lane] -> [g, mt, k, lane, r]
            v = pad.view(rg, 8, K, mt, 32).permute(0, 3, 2, 4, 1)
        else:     # [l, k, m] -> [l, g, r, mt, lane] -> [g, mt, l, lane, r]
            v = pad.view(L, rg, 8, mt, 32).permute(1, 3, 0, 4, 2)
        x[..., t] = v
        del pad, v
    return x.view(rg, mt, S, 32, 2 * T, 4).permute(0, 1, 2, 4, 3, 5).contiguous()


def _current_stream_handle(dev_index: int) -> int:
    getter = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if getter is not None:
        return getter(dev_index)
    return torch.cuda.current_stream(dev_index).cuda_stream


class ContractPlan:
    """A prepared :func:`legendre_contract` call: the descriptor is built and
    checked once, :meth:`launch` only fills in the input and output pointers
    (for callers that launch the same contraction repeatedly, such as the
    modules' forward).  ``input_like`` / ``output_like`` fix the dtypes, shapes,
    strides and the device; later tensors must match them.  One plan may be
    launched from several threads (the descriptor is filled and passed under a
    lock; the launch itself is asynchronous)."""

    __slots__ = ("_desc", "_dev", "_in_sig", "_out_sig", "_keep", "_lock")

    def __init__(self, *, input_like: torch.Tensor, output_like: torch.Tensor, **kw):
        self._desc = _contract_desc(input=input_like, output=output_like, **kw)
        self._dev = input_like.device.index
        self._in_sig = (input_like.dtype, tuple(input_like.shape), input_like.stride())
        self._out_sig = (output_like.dtype, tuple(output_like.shape), output_like.stride())
        self._keep = (kw.get("w0"), kw.get("w1"))  # the tables stay alive with the plan
        self._lock = threading.Lock()

    def launch(self, input: torch.Tensor, output: torch.Tensor) -> None:
        _require(input.is_cuda and input.device.index == self._dev and output.device == input.device
                 and (input.dtype, tuple(input.shape), input.stride()) == self._in_sig
                 and (output.dtype, tuple(output.shape), output.stride()) == self._out_sig,
                 "tensors do not match the contraction plan")
        lib = _lib.load()
        with self._lock:
            d = self._desc
            d.in_, d.out = input.data_ptr(), output.data_ptr()
            if torch.cuda.current_device() == self._dev:
                _lib.check(lib.holysht_legendre_contract(ctypes.byref(d), _current_stream_handle(self._dev)))
            else:
                with torch.cuda.device(self._dev):
                    _lib.check(lib.holysht_legendre_contract(ctypes.byref(d), _current_stream_handle(self._dev)))


    def launch_ptrs(self, in_ptr: int, out_ptr: int) -> None:
        """:meth:`launch` for a caller that has already matched the tensors to
        the plan (the modules' cached forward: same input shape, its own rfft
        output and a fresh output of the planned shape): pointers only."""
        lib = _lib.load()
        with self._lock:
            d = self._desc
            d.in_, d.out = in_ptr, out_ptr
            if torch.cuda.current_device() == self._dev:
                st = lib.holysht_legendre_contract(ctypes.byref(d), _current_stream_handle(self._dev))
            else:
                with torch.cuda.device(self._dev):
                    st = lib.holysht_legendre_contract(ctypes.byref(d), _current_stream_handle(self._dev))
        _lib.check(st)


    def launch_rfft(self, field_ptr: int, rows: int, nlon: int, spec_ptr: int, work_ptr: int, work_bytes: int,
                    out_ptr: int) -> None:
        """The longitude rFFT of ``rows`` contiguous float32 rows into the
        spectrum buffer ``spec_ptr`` (this plan's input layout), then this
        contraction, in one library call (``holysht_rfft_contract``); for a caller
        that has matched the buffers to the plan, like :meth:`launch_ptrs`."""
        lib = _lib.load()
        with self._lock:
            d = self._desc
            d.out = out_ptr
            if torch.cuda.current_device() == self._dev:
                st = lib.holysht_rfft_contract(field_ptr, rows, nlon, spec_ptr, work_ptr, work_bytes,
                                               ctypes.byref(d), _current_stream_handle(self._dev))
            else:
                with torch.cuda.device(self._dev):
                    st = lib.holysht_rfft_contract(field_ptr, rows, nlon, spec_ptr, work_ptr, work_bytes,
                                                   ctypes.byref(d), _current_stream_handle(self._dev))
        _lib.check(st)


def legendre_inverse_recurrence(output: torch.Tensor, coef_in: torch.Tensor, seeds: torch.Tensor,
                                coef: torch.Tensor, cos_theta: torch.Tensor, scale: float = 1.0,
                                parity: bool = False, irfft_prep: bool = False, nlon: int = 0) -> None:
    """Scalar inverse contraction with on-the-fly Legendre functions
    (``holysht_legendre_inverse_recurrence``): output [B, nlat, W >= mmax]
    complex64 (columns >= mmax written as zeros; ``irfft_prep`` drops Im at m = 0
    and m = nlon/2) from coefficients ``coef_in`` [B, lmax, mmax]; ``seeds``,
    ``coef`` and ``cos_theta`` from
    :func:`holysht_b200.weights.scalar_recurrence_tables` with ``inverse=True, segment=8``."""
    dev = _cuda(output, coef_in, seeds, coef, cos_theta)
    _require(coef_in.dtype == torch.complex64 and output.dtype == torch.complex64, "coefficients and output are complex64")
    _require(coef_in.dim() == 3 and coef_in.stride(2) == 1 and output.dim() == 3 and output.stride(2) == 1,
             "coefficients [B, lmax, mmax] and output [B, nlat, W] with contiguous orders")
    _contig(seeds, coef, cos_theta)
    M, nseg, K, two = seeds.shape
    L = coef.size(1)
    B = coef_in.size(0)
    _require(two == 2 and nseg == (L + 7) // 8 and tuple(coef.shape) == (M, L, 2) and cos_theta.numel() == K,
             "inconsistent tables (the inverse kernel's checkpoints are 8 degrees apart)")
    _require(tuple(coef_in.shape) == (B, L, M), "coefficients must be [B, lmax, mmax]")
    _require(output.size(0) == B and output.size(1) == K and output.size(2) >= M, "output must be [B, nlat, >= mmax]")
    flags = (_lib.FLAG_EQUATORIAL_PARITY if parity else 0) | (_lib.FLAG_IRFFT_PREP if irfft_prep else 0)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_legendre_inverse_recurrence(
            _p(output), output.stride(0), output.stride(1), output.size(2), _p(coef_in), coef_in.stride(0),
            coef_in.stride(1), _p(seeds), _p(coef), _p(cos_theta), B, K, L, M, float(scale), flags, int(nlon),
            _stream(dev)))


def rfft_workspace(rows: int, nlon: int, device) -> Optional[int]:
    """Work-area bytes of the library's cuFFT plan for ``rows`` transforms of
    ``nlon`` points on ``device`` (``holysht_rfft_workspace``), or None when
    cuFFT cannot be opened."""
    v = ctypes.c_int64(0)
    with torch.cuda.device(device):
        st = _lib.load().holysht_rfft_workspace(rows, nlon, ctypes.byref(v))
    if st == _lib.HOLYSHT_ERR_UNSUPPORTED:
        return None
    _lib.check(st)
    return int(v.value)


def legendre_contract(*, kind: int, direction: int, input: torch.Tensor, output: torch.Tensor,
                      w0: torch.Tensor, w1: Optional[torch.Tensor] = None, batch: int, nlat: int,
                      lmax: int, mmax: int, in_strides, out_strides, out_cols: int,
                      scale: float = 1.0, flags: int = 0, nlon: int = 0, ksplit: int = 0,
                      w_strides=None, grouped: bool = False, m_offset: int = 0,
                      grouped8: bool = False, parity: bool = False) -> None:
    """Strided contraction; strides are (batch, component, row) in elements.

    ``w0``/``w1`` are either dense [lmax, nlat, mmax] tables (m contiguous) or
    m-tiled tables from :func:`tile_table` ([lmax, ceil(mmax/32), nlat, 32]);
    ``w_strides`` = (l, k, m-tile) strides in floats overrides the inference.
    ``grouped``: ``w0`` is a :func:`group_table` table (``w1`` unused);
    ``grouped8``: ``w0`` is a :func:`group_table8` table (streaming kernel);
    ``parity`` (forward, with ``grouped8``): ``w0`` holds the northern rows only
    (:func:`group_table8` of ``table[:, :ceil(nlat/2)]``, vector tables not
    combined), for grids symmetric about the equator."""
    d = _contract_desc(kind=kind, direction=direction, input=input, output=output, w0=w0, w1=w1, batch=batch,
                       nlat=nlat, lmax=lmax, mmax=mmax, in_strides=in_strides, out_strides=out_strides,
                       out_cols=out_cols, scale=scale, flags=flags, nlon=nlon, ksplit=ksplit, w_strides=w_strides,
                       grouped=grouped, m_offset=m_offset, grouped8=grouped8, parity=parity)
    dev = input.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_legendre_contract(ctypes.byref(d), _stream(dev)))


def legendre_contract_peers(peer_ptrs, *, out_col_offset: int = 0, multicast_ptr: int = 0, **kwargs) -> None:
    """:func:`legendre_contract` (``grouped8`` tables) with every output element
    stored at column ``out_col_offset + m`` of each buffer in ``peer_ptrs``
    (device addresses valid on this GPU: its own buffer and peers' buffers
    mapped into it, all laid out like ``output``), or once through the NVLink
    multicast address ``multicast_ptr`` when it is not 0
    (``holysht_legendre_contract_peers``).  ``output`` is this GPU's own buffer
    (used for checks only).  The caller orders the stores with the peers
    (a cross-GPU barrier) before anyone reads them."""
    _require(kwargs.get("grouped8", False), "output to several GPUs needs grouped8 tables")
    n = len(peer_ptrs)
    _require(1 <= n <= 8, "1 to 8 peer buffers")
    d = _contract_desc(**kwargs)
    arr = (ctypes.c_void_p * n)(*[int(p) for p in peer_ptrs])
    dev = kwargs["input"].device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_legendre_contract_peers(
            ctypes.byref(d), arr, n, int(out_col_offset), ctypes.c_void_p(int(multicast_ptr) or None), _stream(dev)))


def _contract_desc(*, kind, direction, input, output, w0, w1=None, batch, nlat, lmax, mmax, in_strides,
                   out_strides, out_cols, scale=1.0, flags=0, nlon=0, ksplit=0, w_strides=None, grouped=False,
                   m_offset=0, grouped8=False, parity=False):
    """Checked ``holysht_contract_desc`` for :func:`legendre_contract` / :class:`ContractPlan`."""
    _cuda(output, input, w0)
    if w1 is not None:
        _cuda(output, w1)
        _require(w1.stride() == w0.stride(), "W0 and W1 must share strides")
    _require(w0.dtype == torch.float32, "tables must be float32")
    if grouped8:
        _require(w0.dim() == 6 and w0.is_contiguous() and w0.size(-1) == 4 and w0.size(-2) == 32,
                 "GROUPED8 tables come from group_table8()")
        w_strides = (0, 0, 0)
    elif grouped:
        _require(w0.dim() == 6 and w0.is_contiguous(), "grouped tables come from group_table()")
        w_strides = (0, 0, 0)
    elif w_strides is None:
        if w0.dim() == 4:
            _require(w0.is_contiguous() and w0.size(3) == 32, "m-tiled tables must be contiguous [L, Mt, K, 32]")
            w_strides = (w0.stride(0), w0.stride(2), w0.stride(1))
        else:
            _require(w0.dim() == 3 and w0.stride(2) == 1,
                     "tables must be [lmax, nlat, mmax] with contiguous mmax")
            w_strides = (w0.stride(0), w0.stride(1), 32)
    if input.dtype == torch.complex64:
        dt = _lib.DTYPE_C64
    elif input.dtype == torch.float32:
        dt = _lib.DTYPE_F32
    elif input.dtype == torch.bfloat16:
        dt = _lib.DTYPE_BF16
    else:
        raise RuntimeError(f"unsupported input dtype {input.dtype}")
    d = _lib.ContractDesc()
    d.kind, d.direction, d.in_dtype, d.flags = kind, direction, dt, flags
    d.in_, d.out, d.w0, d.w1 = _p(input), _p(output), _p(w0), _p(w1)
    d.batch, d.nlat, d.lmax, d.mmax = batch, nlat, lmax, mmax
    d.in_batch_stride, d.in_comp_stride, d.in_row_stride = in_strides
    d.out_batch_stride, d.out_comp_stride, d.out_row_stride = out_strides
    d.out_cols = out_cols
    d.w_l_stride, d.w_k_stride, d.w_m_tile_stride = w_strides
    d.nlon = nlon
    d.scale = scale
    d.ksplit = ksplit
    d.table_layout = (_lib.TABLE_GROUPED8_PARITY if (grouped8 and parity) else _lib.TABLE_GROUPED8 if grouped8 else
                      _lib.TABLE_GROUPED if grouped else _lib.TABLE_STRIDED)
    d.m_offset = m_offset
    return d


def split_dense_table(table: torch.Tensor) -> torch.Tensor:
    """[2, *table.shape] split of a dense-path table (``holysht_legendre_dense_tc_split_table``):
    plane 0 the tf32-rounded values, plane 1 the fp32 residuals."""
    _cuda(table)
    _require(table.dtype == torch.float32 and table.is_contiguous(), "table must be contiguous float32")
    out = torch.empty((2,) + tuple(table.shape), dtype=torch.float32, device=table.device)
    with torch.cuda.device(table.device):
        _lib.check(_lib.load().holysht_legendre_dense_tc_split_table(_p(table), _p(out), table.numel(),
                                                                     _stream(table.device)))
    return out


def legendre_dense_tc(direction: int, output: torch.Tensor, input: torch.Tensor, table: torch.Tensor,
                      *, nlat: int, lmax: int, mmax: int, scale: float = 1.0, flags: int = 0,
                      nlon: int = 0) -> None:
    """Dense tensor-core contraction (SCALAR kind, ``holysht_legendre_dense_tc``).

    forward: output [B, lmax, >= mmax] <- input [B, nlat, >= mmax], table [mmax, lmax, nlat];
    inverse: output [B, nlat, >= mmax] <- input [B, lmax, >= mmax], table [mmax, nlat, lmax].
    Rows of input and output may be strided (rfft / irfft buffers); orders are
    contiguous.  The GEMM workspace comes from torch's caching allocator."""
    dev = _cuda(output, input, table)
    _require(input.dtype == torch.complex64 and output.dtype == torch.complex64, "input and output are complex64")
    _require(table.dtype == torch.float32 and table.is_contiguous(), "table must be contiguous float32")
    _require(input.dim() == 3 and output.dim() == 3 and input.stride(2) == 1 and output.stride(2) == 1,
             "input and output must be [B, rows, cols] with contiguous orders")
    fwd = direction == _lib.DIR_FORWARD
    want = (mmax, lmax, nlat) if fwd else (mmax, nlat, lmax)
    if tuple(table.shape) == (2,) + want:  # a split_dense_table() table
        flags |= _lib.FLAG_TABLE_SPLIT
    else:
        _require(tuple(table.shape) == want, f"table must be {want} or a split (2, {want}) table")
    B = input.size(0)
    lib = _lib.load()
    nbytes = ctypes.c_int64(0)
    _lib.check(lib.holysht_legendre_dense_tc_workspace_ex(direction, B, nlat, lmax, mmax, int(flags),
                                                          ctypes.byref(nbytes)))
    with torch.cuda.device(dev):
        ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=dev)
        _lib.check(lib.holysht_legendre_dense_tc(
            direction, _p(output), output.stride(0), output.stride(1), output.size(2), _p(input),
            input.stride(0), input.stride(1), _p(table), B, nlat, lmax, mmax, float(scale), int(flags), int(nlon),
            _p(ws), nbytes.value, _stream(dev)))


def tc_error_word() -> int:
    """Read and clear the tensor-core kernel's device error word (synchronous)."""
    v = ctypes.c_uint(0)
    _lib.check(_lib.load().holysht_tc_error_word(ctypes.byref(v)))
    return int(v.value)


def stream_launch_plan(kind: int, direction: int, *, batch: int, nlat: int, lmax: int, mmax: int,
                       out_cols: Optional[int] = None, m_offset: int = 0, ksplit: int = 0,
                       sm_count: int = 0) -> dict:
    """Launch plan of the streaming kernel (host-only): ``ks`` (cluster size /
    reduction split), ``clusters`` and ``items`` (compute tile x batch group).
    ``sm_count`` > 0 plans for that many SMs without a GPU."""
    ks, cl, it = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.load().holysht_stream_launch_plan(
        kind, direction, batch, nlat, lmax, mmax, mmax if out_cols is None else out_cols, m_offset, ksplit,
        sm_count, ctypes.byref(ks), ctypes.byref(cl), ctypes.byref(it)))
    return {"ks": ks.value, "clusters": cl.value, "items": it.value}


def stream_error_word() -> int:
    """Read and clear the streaming kernel's device error word (synchronous)."""
    v = ctypes.c_uint(0)
    _lib.check(_lib.load().holysht_stream_error_word(ctypes.byref(v)))
    return int(v.value)


def _nsegs(L: int, M: int) -> int:
    """Number of 16-degree checkpoint segments of the orders m < min(M, L)."""
    return sum((L - m + 15) // 16 for m in range(min(M, L)))


def legendre_vector_forward_recurrence(output: torch.Tensor, spec: torch.Tensor, seeds: torch.Tensor,
                                       coef: torch.Tensor, cos_theta: torch.Tensor, scale: float = 1.0,
                                       parity: bool = False) -> None:
    """Vector forward with on-the-fly tables (``holysht_legendre_vector_forward_recurrence_ex``):
    output [B, 2, L, M] complex64 from an rfft-layout spectrum [B, 2, K, W >= M];
    ``seeds``, ``coef`` and ``cos_theta`` from
    :func:`holysht_b200.weights.vector_recurrence_tables`.  ``parity`` folds the
    grid's equatorial symmetry (see :func:`holysht_b200.weights.recurrence_seeds_symmetric`).
    Seeds [K, nsegs, 4] are the compact layout
    (:func:`holysht_b200.weights.compact_recurrence_seeds`)."""
    dev = _cuda(output, spec, seeds, coef, cos_theta)
    _require(spec.dtype == torch.complex64 and output.dtype == torch.complex64, "spectrum and output are complex64")
    _require(spec.dim() == 4 and spec.size(1) == 2 and spec.stride(3) == 1,
             "spectrum must be [B, 2, K, W] with contiguous orders")
    _contig(output, seeds, coef, cos_theta)
    flags = _lib.FLAG_EQUATORIAL_PARITY if parity else 0
    M, L = coef.size(0), coef.size(1)
    if seeds.dim() == 3:
        K, nsegs, four = seeds.shape
        _require(nsegs == _nsegs(L, M), "compact seeds do not match lmax / mmax")
        flags |= _lib.FLAG_SEEDS_COMPACT
    else:
        _require(seeds.dim() == 4 and seeds.size(0) == M, "seeds must be [M, nseg, K, 4] or [K, nsegs, 4]")
        _, nseg, K, four = seeds.shape
        _require(nseg == (L + 15) // 16, "seeds must hold ceil(lmax / 16) segments per order")
    B = spec.size(0)
    _require(four == 4 and tuple(coef.shape) == (M, L, 8) and cos_theta.numel() == K, "inconsistent tables")
    _require(spec.size(2) == K and spec.size(3) >= M, "spectrum must be [B, 2, nlat, >= mmax]")
    _require(tuple(output.shape) == (B, 2, L, M), "output must be [B, 2, lmax, mmax]")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_legendre_vector_forward_recurrence_ex(
            _p(output), _p(spec), spec.stride(0), spec.stride(1), spec.stride(2), _p(seeds), _p(coef),
            _p(cos_theta), B, K, L, M, float(scale), flags, _stream(dev)))


def legendre_forward_recurrence(output: torch.Tensor, spec: torch.Tensor, seeds: torch.Tensor, coef: torch.Tensor,
                                cos_theta: torch.Tensor, scale: float = 1.0, parity: bool = False) -> None:
    """Scalar forward with on-the-fly Legendre functions (``holysht_legendre_forward_recurrence_ex``):
    output [B, L, M] complex64 from an rfft-layout spectrum [B, K, W >= M]; ``seeds``,
    ``coef`` and ``cos_theta`` from :func:`holysht_b200.weights.scalar_recurrence_tables`.
    ``parity`` folds the grid's equatorial symmetry (the seeds must come from a
    grid symmetric about the equator; see :func:`holysht_b200.weights.recurrence_seeds_symmetric`).
    Seeds [K, nsegs, 2] are the compact layout
    (:func:`holysht_b200.weights.compact_recurrence_seeds`)."""
    dev = _cuda(output, spec, seeds, coef, cos_theta)
    _require(spec.dtype == torch.complex64 and output.dtype == torch.complex64, "spectrum and output are complex64")
    _require(spec.dim() == 3 and spec.stride(2) == 1, "spectrum must be [B, K, W] with contiguous orders")
    _contig(output, seeds, coef, cos_theta)
    flags = _lib.FLAG_EQUATORIAL_PARITY if parity else 0
    M, L = coef.size(0), coef.size(1)
    if seeds.dim() == 3:
        K, nsegs, two = seeds.shape
        _require(nsegs == _nsegs(L, M), "compact seeds do not match lmax / mmax")
        flags |= _lib.FLAG_SEEDS_COMPACT
    else:
        _require(seeds.dim() == 4 and seeds.size(0) == M, "seeds must be [M, nseg, K, 2] or [K, nsegs, 2]")
        _, nseg, K, two = seeds.shape
        _require(nseg == (L + 15) // 16, "seeds must hold ceil(lmax / 16) segments per order")
    B = spec.size(0)
    _require(two == 2 and tuple(coef.shape) == (M, L, 2) and cos_theta.numel() == K, "inconsistent tables")
    _require(spec.size(1) == K and spec.size(2) >= M, "spectrum must be [B, nlat, >= mmax]")
    _require(tuple(output.shape) == (B, L, M), "output must be [B, lmax, mmax]")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().holysht_legendre_forward_recurrence_ex(
            _p(output), _p(spec), spec.stride(0), spec.stride(1), _p(seeds), _p(coef), _p(cos_theta),
            B, K, L, M, float(scale), flags, _stream(dev)))
