"""The allocation-free dense tensor-core entry point.

``holysht_legendre_dense_tc_noalloc`` serves callers that cannot allocate
device memory themselves (a host whose allocator owns the GPU, a loop that
must not allocate per call, a plugin handed no allocator): it takes its
scratch from a 64 MiB array built into the library instead of a caller
workspace.  These tests call it through the C ABI and compare it with the
workspace entry point ``holysht_legendre_dense_tc`` on two calls in a row (the
second call must not be affected by what the first left in the shared
scratch), and check that a problem too large for the built-in scratch is
refused with a clear message.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from holysht_b200 import _lib, ops

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP32_REL = 1e-6
FP32_MAXABS = 1e-5


def _close(got, ref):
    got = got.cpu().numpy().astype(np.complex128)
    ref = ref.cpu().numpy().astype(np.complex128)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel <= FP32_REL, rel
    assert np.abs(got - ref).max() <= FP32_MAXABS * np.abs(ref).max()


def _noalloc(direction, out, inp, table, nlat, lmax, mmax, scale=1.0, flags=0, nlon=0):
    lib = _lib.load()
    st = lib.holysht_legendre_dense_tc_noalloc(
        direction, out.data_ptr(), out.stride(0), out.stride(1), out.size(2), inp.data_ptr(), inp.stride(0),
        inp.stride(1), table.data_ptr(), inp.size(0), nlat, lmax, mmax, ctypes.c_float(scale), flags, nlon,
        torch.cuda.current_stream().cuda_stream)
    return st


def _problem(rng, B, K, L, M):
    w = rng.standard_normal((L, K, M)).astype(np.float32)
    w *= np.arange(M)[None, None, :] <= np.arange(L)[:, None, None]
    spec = (rng.standard_normal((B, K, M + 3)) + 1j * rng.standard_normal((B, K, M + 3))).astype(np.complex64)
    coef = (rng.standard_normal((B, L, M)) + 1j * rng.standard_normal((B, L, M))).astype(np.complex64)
    return w, torch.from_numpy(spec).to(DEV), torch.from_numpy(coef).to(DEV)


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    B, K, L, M = 96, 64, 160, 97
    rng = np.random.default_rng(2024)
    for call in range(2):
        w, spec, coef = _problem(rng, B, K, L, M)
        fwd_table = torch.from_numpy(np.ascontiguousarray(w.transpose(2, 0, 1))).to(DEV)  # [M, L, K]
        inv_table = torch.from_numpy(np.ascontiguousarray(w.transpose(2, 1, 0))).to(DEV)  # [M, K, L]

        ref = torch.empty((B, L, M), dtype=torch.complex64, device=DEV)
        ops.legendre_dense_tc(_lib.DIR_FORWARD, ref, spec, fwd_table, nlat=K, lmax=L, mmax=M, scale=0.75)
        got = torch.full((B, L, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
        assert _noalloc(_lib.DIR_FORWARD, got, spec, fwd_table, K, L, M, scale=0.75) == _lib.HOLYSHT_OK
        _close(got, ref)

        nlon = 2 * (M - 1) + 4
        W = nlon // 2 + 1
        ref_i = torch.empty((B, K, W), dtype=torch.complex64, device=DEV)
        ops.legendre_dense_tc(_lib.DIR_INVERSE, ref_i, coef, inv_table, nlat=K, lmax=L, mmax=M,
                              flags=_lib.FLAG_IRFFT_PREP, nlon=nlon)
        got_i = torch.full((B, K, W), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
        assert _noalloc(_lib.DIR_INVERSE, got_i, coef, inv_table, K, L, M, flags=_lib.FLAG_IRFFT_PREP,
                        nlon=nlon) == _lib.HOLYSHT_OK
        _close(got_i, ref_i)
    torch.cuda.synchronize()
    assert ops.tc_error_word() == 0


def test_noalloc_rejects_problems_larger_than_its_scratch():
    B, K, L, M = 512, 256, 256, 257  # needs ~270 MB of scratch
    spec = torch.zeros((B, K, M), dtype=torch.complex64, device=DEV)
    table = torch.zeros((M, L, K), dtype=torch.float32, device=DEV)
    out = torch.zeros((B, L, M), dtype=torch.complex64, device=DEV)
    st = _noalloc(_lib.DIR_FORWARD, out, spec, table, K, L, M)
    assert st == _lib.HOLYSHT_ERR_INVALID
    msg = _lib.load().holysht_last_error().decode()
    assert "built-in scratch" in msg and "64 MiB" in msg


def _workspace_entry_nan(direction, out, inp, table, nlat, lmax, mmax, scale=1.0, flags=0, nlon=0):
    """The workspace entry point with its workspace pre-filled with NaN, so any
    scratch element read before it is written shows up in the output."""
    lib = _lib.load()
    nbytes = ctypes.c_int64(0)
    _lib.check(lib.holysht_legendre_dense_tc_workspace(direction, inp.size(0), nlat, lmax, mmax,
                                                       ctypes.byref(nbytes)))
    ws = torch.full((max(nbytes.value, 4) // 4,), float("nan"), dtype=torch.float32, device=DEV)
    _lib.check(lib.holysht_legendre_dense_tc(
        direction, out.data_ptr(), out.stride(0), out.stride(1), out.size(2), inp.data_ptr(), inp.stride(0),
        inp.stride(1), table.data_ptr(), inp.size(0), nlat, lmax, mmax, ctypes.c_float(scale), flags, nlon,
        ws.data_ptr(), nbytes.value, torch.cuda.current_stream().cuda_stream))


def test_noalloc_larger_problem_then_smaller_problem():
    """A large call leaves its rows in the shared scratch; a following smaller
    call with a different row count and batch must not read any of them."""
    rng = np.random.default_rng(77)
    for B, K, L, M in ((120, 96, 160, 97), (24, 32, 48, 33)):
        w, spec, _ = _problem(rng, B, K, L, M)
        fwd_table = torch.from_numpy(np.ascontiguousarray(w.transpose(2, 0, 1))).to(DEV)
        ref = torch.empty((B, L, M), dtype=torch.complex64, device=DEV)
        _workspace_entry_nan(_lib.DIR_FORWARD, ref, spec, fwd_table, K, L, M, scale=1.25)
        got = torch.full((B, L, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
        assert _noalloc(_lib.DIR_FORWARD, got, spec, fwd_table, K, L, M, scale=1.25) == _lib.HOLYSHT_OK
        assert torch.isfinite(torch.view_as_real(ref)).all()
        _close(got, ref)
    torch.cuda.synchronize()
    assert ops.tc_error_word() == 0
