"""ctypes binding of ``libholysht_b200.so`` (the C ABI in include/holysht_b200.h).

There is deliberately no fallback: if the shared library is missing or does
not load, every operator raises.  Build it with ``python -m holysht_b200.build``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import os

LIB_PATH = Path(os.environ.get("HOLYSHT_B200_LIBRARY") or Path(__file__).resolve().parent / "libholysht_b200.so")

HOLYSHT_OK = 0
HOLYSHT_ERR_INVALID = 1
HOLYSHT_ERR_CUDA = 2
HOLYSHT_ERR_UNSUPPORTED = 3

DTYPE_C64, DTYPE_F32, DTYPE_BF16 = 0, 1, 2
KIND_SCALAR, KIND_VECTOR, KIND_REAL = 0, 1, 2
DIR_FORWARD, DIR_INVERSE = 0, 1
FLAG_CONJ_W1, FLAG_ROUND_BF16, FLAG_IRFFT_PREP, FLAG_TABLE_SPLIT = 1, 2, 4, 16
FLAG_EQUATORIAL_PARITY, FLAG_SEEDS_COMPACT = 32, 64
TABLE_STRIDED, TABLE_GROUPED, TABLE_GROUPED8, TABLE_GROUPED8_PARITY = 0, 1, 2, 3

# every symbol include/holysht_b200.h declares
EXPORTS = (
    "holysht_version",
    "holysht_last_error",
    "holysht_fused_legendre_forward",
    "holysht_fused_legendre_inverse",
    "holysht_fused_legendre_forward_real",
    "holysht_fused_legendre_inverse_real",
    "holysht_fused_vector_legendre_forward",
    "holysht_fused_vector_legendre_inverse",
    "holysht_fused_vector_forward_pack_real",
    "holysht_fused_vector_forward_recompose_real",
    "holysht_sht_prepare_irfft",
    "holysht_legendre_contract",
    "holysht_legendre_contract_peers",
    "holysht_peer_barrier",
    "holysht_peer_error_word",
    "holysht_legendre_dense_tc_workspace",
    "holysht_legendre_dense_tc_workspace_ex",
    "holysht_legendre_dense_tc_split_table",
    "holysht_legendre_dense_tc",
    "holysht_tc_error_word",
    "holysht_stream_error_word",
    "holysht_stream_launch_plan",
    "holysht_legendre_dense_tc_noalloc",
    "holysht_legendre_forward_recurrence",
    "holysht_legendre_forward_recurrence_ex",
    "holysht_legendre_vector_forward_recurrence",
    "holysht_legendre_vector_forward_recurrence_ex",
    "holysht_legendre_inverse_recurrence",
    "holysht_rfft_workspace",
    "holysht_rfft_contract",
)


class ContractDesc(ctypes.Structure):
    """Mirror of ``holysht_contract_desc``."""

    _fields_ = [
        ("kind", ctypes.c_int),
        ("direction", ctypes.c_int),
        ("in_dtype", ctypes.c_int),
        ("flags", ctypes.c_int),
        ("in_", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("w0", ctypes.c_void_p),
        ("w1", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("nlat", ctypes.c_int64),
        ("lmax", ctypes.c_int64),
        ("mmax", ctypes.c_int64),
        ("in_batch_stride", ctypes.c_int64),
        ("in_comp_stride", ctypes.c_int64),
        ("in_row_stride", ctypes.c_int64),
        ("out_batch_stride", ctypes.c_int64),
        ("out_comp_stride", ctypes.c_int64),
        ("out_row_stride", ctypes.c_int64),
        ("out_cols", ctypes.c_int64),
        ("w_l_stride", ctypes.c_int64),
        ("w_k_stride", ctypes.c_int64),
        ("nlon", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("ksplit", ctypes.c_int),
        ("w_m_tile_stride", ctypes.c_int64),
        ("table_layout", ctypes.c_int),
        ("m_offset", ctypes.c_int64),
    ]


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and type the shared library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"holysht_b200 native library not found at {LIB_PATH}; "
                "build it with `python -m holysht_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        sig = {
            "holysht_version": ([], i32),
            "holysht_last_error": ([], ctypes.c_char_p),
            "holysht_fused_legendre_forward": ([vp, vp, vp, i64, i64, i64, i64, vp], i32),
            "holysht_fused_legendre_inverse": ([vp, vp, vp, i64, i64, i64, i64, vp], i32),
            "holysht_fused_legendre_forward_real": ([vp, vp, i32, vp, i64, i64, i64, i64, i32, vp], i32),
            "holysht_fused_legendre_inverse_real": ([vp, vp, vp, i64, i64, i64, i64, vp], i32),
            "holysht_fused_vector_legendre_forward": ([vp, vp, vp, vp, i64, i64, i64, i64, i32, vp], i32),
            "holysht_fused_vector_legendre_inverse": ([vp, vp, vp, vp, i64, i64, i64, i64, vp], i32),
            "holysht_fused_vector_forward_pack_real": ([vp, vp, vp, i64, i64, i64, vp], i32),
            "holysht_fused_vector_forward_recompose_real": ([vp, vp, vp, i64, i64, i64, vp], i32),
            "holysht_sht_prepare_irfft": ([vp, i64, i64, i64, i64, vp], i32),
            "holysht_legendre_contract": ([ctypes.POINTER(ContractDesc), vp], i32),
            "holysht_peer_barrier": ([ctypes.POINTER(vp), i32, i32, ctypes.c_uint, vp], i32),
            "holysht_peer_error_word": ([ctypes.POINTER(ctypes.c_uint)], i32),
            "holysht_legendre_contract_peers": ([ctypes.POINTER(ContractDesc), ctypes.POINTER(vp), i32, i64, vp, vp],
                                                i32),
            "holysht_legendre_dense_tc_workspace_ex": ([i32, i64, i64, i64, i64, i32,
                                                        ctypes.POINTER(ctypes.c_int64)], i32),
            "holysht_legendre_dense_tc_split_table": ([vp, vp, i64, vp], i32),
            "holysht_legendre_dense_tc_workspace": ([i32, i64, i64, i64, i64, ctypes.POINTER(ctypes.c_int64)], i32),
            "holysht_legendre_dense_tc": ([i32, vp, i64, i64, i64, vp, i64, i64, vp, i64, i64, i64, i64,
                                           ctypes.c_float, i32, i64, vp, i64, vp], i32),
            "holysht_tc_error_word": ([ctypes.POINTER(ctypes.c_uint)], i32),
            "holysht_stream_error_word": ([ctypes.POINTER(ctypes.c_uint)], i32),
            "holysht_stream_launch_plan": ([i32, i32, i64, i64, i64, i64, i64, i64, i32, i32,
                                            ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                            ctypes.POINTER(ctypes.c_int)], i32),
            "holysht_legendre_forward_recurrence": ([vp, vp, i64, i64, vp, vp, vp, i64, i64, i64, i64,
                                                     ctypes.c_float, vp], i32),
            "holysht_legendre_forward_recurrence_ex": ([vp, vp, i64, i64, vp, vp, vp, i64, i64, i64, i64,
                                                        ctypes.c_float, i32, vp], i32),
            "holysht_legendre_vector_forward_recurrence": ([vp, vp, i64, i64, i64, vp, vp, vp, i64, i64, i64, i64,
                                                            ctypes.c_float, vp], i32),
            "holysht_legendre_vector_forward_recurrence_ex": ([vp, vp, i64, i64, i64, vp, vp, vp, i64, i64, i64,
                                                               i64, ctypes.c_float, i32, vp], i32),
            "holysht_legendre_inverse_recurrence": ([vp, i64, i64, i64, vp, i64, i64, vp, vp, vp, i64, i64, i64,
                                                     i64, ctypes.c_float, i32, i64, vp], i32),
            "holysht_rfft_workspace": ([i64, i64, ctypes.POINTER(ctypes.c_int64)], i32),
            "holysht_rfft_contract": ([vp, i64, i64, vp, vp, i64, ctypes.POINTER(ContractDesc), vp], i32),
            "holysht_legendre_dense_tc_noalloc": ([i32, vp, i64, i64, i64, vp, i64, i64, vp, i64, i64, i64, i64,
                                                   ctypes.c_float, i32, i64, vp], i32),
        }
        for name, (args, res) in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def check(status: int) -> None:
    """Raise RuntimeError with the library's message for a failing status."""
    if status == HOLYSHT_OK:
        return
    msg = load().holysht_last_error().decode(errors="replace")
    raise RuntimeError(f"holysht_b200: {msg} (status {status})")
