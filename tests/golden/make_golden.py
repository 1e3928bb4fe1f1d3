"""Generate golden fixtures from the reference's own CPU code path.

Run from the repository root with the reference checkout's path in
``HOLYSHT_REFERENCE`` (required; there is no default):

    HOLYSHT_REFERENCE=<reference checkout> python tests/golden/make_golden.py

The reference package ``torch-ext/holysht/__init__.py`` is imported from a
temporary copy (importing it in place would create a build directory inside
the read-only checkout).  Its module constructors call torch-harmonics, which
is not installed, so a stand-in ``torch_harmonics`` module is registered that
hands the constructors the tables restated by ``oracle/sht_oracle.py``.  Every
forward below then runs the reference's unmodified CPU path (rfft, the einsum
contractions, the stacked vector composition, ``_prepare_irfft_input`` and
irfft), and torch autograd through it for the gradients.

The fixtures therefore pin the contraction, composition and FFT conventions
to the reference code.  The tables themselves are pinned to mathematics in
``tests/test_oracle.py`` (not to torch-harmonics, which is absent).
"""
from __future__ import annotations

import os
import shutil
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import sht_oracle as orc  # noqa: E402

OUT = Path(__file__).resolve().parent


def _stub_torch_harmonics():
    th = types.ModuleType("torch_harmonics")

    def _mk(kind):
        class _Ref:
            def __init__(self, nlat, nlon, lmax=None, mmax=None, grid="equiangular",
                         norm="ortho", csphase=True):
                self.nlat, self.nlon = nlat, nlon
                self.lmax = lmax or orc.default_lmax(nlat, grid)
                self.mmax = mmax or orc.default_mmax(nlon)
                args = (nlat, nlon, self.lmax, self.mmax, grid, norm, csphase)
                if kind == "fwd":
                    self.weights = torch.from_numpy(orc.scalar_forward_table(*args))
                elif kind == "inv":
                    self.pct = torch.from_numpy(orc.scalar_inverse_table(*args))
                elif kind == "vfwd":
                    self.weights = torch.from_numpy(orc.vector_forward_tables(*args))
                else:
                    self.dpct = torch.from_numpy(orc.vector_inverse_tables(*args))
        return _Ref

    th.RealSHT = _mk("fwd")
    th.InverseRealSHT = _mk("inv")
    th.RealVectorSHT = _mk("vfwd")
    th.InverseRealVectorSHT = _mk("vinv")
    return th


def _import_reference(ref_root: Path):
    tmp = Path(tempfile.mkdtemp(prefix="holysht_ref_"))
    pkg = tmp / "holysht"
    pkg.mkdir()
    shutil.copy(ref_root / "torch-ext" / "holysht" / "__init__.py", pkg / "__init__.py")
    sys.modules["torch_harmonics"] = _stub_torch_harmonics()
    sys.path.insert(0, str(tmp))
    import holysht  # noqa: WPS433
    assert not holysht._HAS_NATIVE_EXT, "the golden path must be the reference's CPU path"
    return holysht, tmp


CASES = [
    # name, nlat, nlon, lmax, mmax, grid, batch shape
    ("eq12x24", 12, 24, None, None, "equiangular", (2,)),
    ("lg10x20_l8_m7", 10, 20, 8, 7, "legendre-gauss", (3,)),
    ("eq9x17_odd", 9, 17, None, None, "equiangular", (2, 2)),
    ("lob8x16", 8, 16, None, None, "lobatto", (1,)),
]


def main():
    if not os.environ.get("HOLYSHT_REFERENCE"):
        raise SystemExit("set HOLYSHT_REFERENCE to the reference checkout's root")
    ref_root = Path(os.environ["HOLYSHT_REFERENCE"])
    hs, tmp = _import_reference(ref_root)
    torch.manual_seed(1234)
    rng = np.random.default_rng(1234)
    try:
        for name, nlat, nlon, lmax, mmax, grid, bshape in CASES:
            kw = dict(lmax=lmax, mmax=mmax, grid=grid)
            sht = hs.RealSHT(nlat, nlon, **kw)
            isht = hs.InverseRealSHT(nlat, nlon, **kw)
            vsht = hs.RealVectorSHT(nlat, nlon, **kw)
            ivsht = hs.InverseRealVectorSHT(nlat, nlon, **kw)
            L, M = sht.lmax, sht.mmax
            x = torch.from_numpy(rng.standard_normal(bshape + (nlat, nlon)).astype(np.float32))
            xv = torch.from_numpy(rng.standard_normal(bshape + (2, nlat, nlon)).astype(np.float32))
            tri = (np.arange(M)[None, :] <= np.arange(L)[:, None])
            c = (rng.standard_normal(bshape + (L, M)) + 1j * rng.standard_normal(bshape + (L, M))) * tri
            cv = (rng.standard_normal(bshape + (2, L, M)) + 1j * rng.standard_normal(bshape + (2, L, M))) * tri
            c = torch.from_numpy(c.astype(np.complex64))
            cv = torch.from_numpy(cv.astype(np.complex64))

            xg = x.clone().requires_grad_(True)
            coef = sht(xg)
            (coef.real.square().sum() + coef.imag.square().sum()).backward()
            xvg = xv.clone().requires_grad_(True)
            vcoef = vsht(xvg)
            (vcoef.real.square().sum() + vcoef.imag.square().sum()).backward()
            cg = c.clone().requires_grad_(True)
            y = isht(cg)
            torch.tanh(y).sum().backward()
            cvg = cv.clone().requires_grad_(True)
            yv = ivsht(cvg)
            torch.tanh(yv).sum().backward()

            np.savez_compressed(
                OUT / f"{name}.npz",
                nlat=nlat, nlon=nlon, lmax=L, mmax=M, grid=grid,
                x=x.numpy(), xv=xv.numpy(), c=c.numpy(), cv=cv.numpy(),
                sht=coef.detach().numpy(), vsht=vcoef.detach().numpy(),
                isht=y.detach().numpy(), ivsht=yv.detach().numpy(),
                grad_sht=xg.grad.numpy(), grad_vsht=xvg.grad.numpy(),
                grad_isht=cg.grad.numpy(), grad_ivsht=cvg.grad.numpy(),
            )
            print("wrote", name)

        # op-level known answers on random lower-triangular tables (the
        # reference's fused_legendre_forward/inverse CPU branches)
        L, K, M, B = 7, 6, 9, 3
        tri = (np.arange(M)[None, None, :] <= np.arange(L)[:, None, None])
        wt = (rng.standard_normal((L, K, M)) * tri).astype(np.float32)
        xin = (rng.standard_normal((B, K, M)) + 1j * rng.standard_normal((B, K, M))).astype(np.complex64)
        cin = (rng.standard_normal((B, L, M)) + 1j * rng.standard_normal((B, L, M))).astype(np.complex64)
        weights = torch.from_numpy(wt).permute(2, 0, 1).contiguous()  # [M, L, K]
        fwd = hs.fused_legendre_forward(torch.from_numpy(xin), weights)
        inv = hs.fused_legendre_inverse(torch.from_numpy(cin), weights)
        re = hs.fused_legendre_forward_real(torch.from_numpy(xin.real.copy()), torch.from_numpy(wt))
        ire = hs.fused_legendre_inverse_real(torch.from_numpy(cin.real.copy()), torch.from_numpy(wt))
        pre_even = hs._prepare_irfft_input(torch.from_numpy(cin), 20, M)
        pre_odd = hs._prepare_irfft_input(torch.from_numpy(cin), 19, M)
        np.savez_compressed(
            OUT / "ops_tri.npz", weight_t=wt, x=xin, c=cin,
            fwd=fwd.numpy(), inv=inv.numpy(), fwd_real=re.numpy(), inv_real=ire.numpy(),
            prep_even=pre_even.numpy(), prep_odd=pre_odd.numpy(),
        )
        print("wrote ops_tri")
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    main()
