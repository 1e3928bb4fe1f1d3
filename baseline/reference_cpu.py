"""The reference's own CPU path, imported from ``baseline/_ref`` without its CUDA extension.

``load()`` returns the reference package (``torch-ext/holysht/__init__.py``,
unmodified) imported from a temporary copy of that one file, so neither the
packaged ops module nor the JIT loader is found and the package takes its CPU
branch (``_HAS_NATIVE_EXT`` false): rfft on the host, then the einsum
contractions (``__init__.py:1130-1132`` scalar, the stacked vector
composition :1680-1692).  Its constructors call torch-harmonics, absent on
both machines; a stand-in hands them the tables of ``holysht_b200.weights``
(the tables this project's modules use), so both sides contract identical
tables.  ``bench.py`` times this path as the CPU baseline and as its
reference arm.
"""
from __future__ import annotations

import importlib
import shutil
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
REF_INIT = HERE / "_ref" / "torch-ext" / "holysht" / "__init__.py"


def available() -> bool:
    return REF_INIT.exists()


def stand_in_torch_harmonics() -> types.ModuleType:
    """A ``torch_harmonics`` module whose transforms only carry the tables."""
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    from holysht_b200 import weights as W

    th = types.ModuleType("torch_harmonics")

    def make(builder, attr):
        class _T:
            def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True):
                t, self.lmax, self.mmax = builder(nlat, nlon, lmax, mmax, grid, norm, csphase, dtype=np.float32,
                                                  restated=True)
                self.nlat, self.nlon = nlat, nlon
                setattr(self, attr, torch.from_numpy(t))
        return _T

    th.RealSHT = make(W.scalar_forward, "weights")
    th.InverseRealSHT = make(W.scalar_inverse, "pct")
    th.RealVectorSHT = make(W.vector_forward, "weights")
    th.InverseRealVectorSHT = make(W.vector_inverse, "dpct")
    return th


def load():
    """The reference package on its CPU path (raises if ``baseline/_ref`` is absent)."""
    if not available():
        raise FileNotFoundError("baseline/_ref is not prepared (baseline/prepare_reference.py)")
    tmp = Path(tempfile.mkdtemp(prefix="holysht_ref_cpu_"))
    pkg = tmp / "holysht_ref_cpu"
    pkg.mkdir()
    shutil.copy(REF_INIT, pkg / "__init__.py")
    sys.modules.setdefault("torch_harmonics", stand_in_torch_harmonics())
    sys.path.insert(0, str(tmp))
    try:
        mod = importlib.import_module("holysht_ref_cpu")
    finally:
        sys.path.remove(str(tmp))
        shutil.rmtree(tmp, ignore_errors=True)
    if mod._HAS_NATIVE_EXT:
        raise RuntimeError("the reference CPU import found a native extension")
    return mod
