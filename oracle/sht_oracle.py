"""CPU oracle for the HOLYSHT Legendre hot path (TEST INFRASTRUCTURE ONLY).

This module is a float64 numpy restatement of what the reference computes on
the path ``rfft -> per-order Legendre contraction`` (and its inverse).  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and only as the checker.  The product package
never imports it.

What it restates (reference = chrisvoncsefalvay/holysht):

* the module forward/inverse maths of ``torch-ext/holysht/__init__.py``:
  ``fused_sht_forward`` :1195-1208, ``fused_legendre_forward`` einsum
  :1130-1132, ``fused_legendre_inverse`` einsum :1158-1160,
  ``_prepare_irfft_input`` :949-973, the vector composition of
  ``RealVectorSHT`` :1680-1692 / ``_recompose_vector_forward_real_outputs``
  :448-477 and ``InverseRealVectorSHT`` :1769-1791;
* the weight tables the reference pulls from torch-harmonics (third-party,
  not vendored, version unpinned; call sites ``__init__.py:1247-1256``,
  :1406-1415, :1452-1461, :1710-1719).  Their published construction is
  restated here from the mathematics:
    - Clenshaw-Curtis nodes/weights by Waldvogel's FFT construction
      (J. Waldvogel, BIT 43 (2003) 1-18) for ``grid="equiangular"``;
    - Gauss-Legendre nodes/weights (numpy ``leggauss``) for
      ``grid="legendre-gauss"``; Gauss-Lobatto by Newton iteration on
      P'_{n-1} for ``grid="lobatto"``;
    - orthonormal associated Legendre functions by the standard
      three-term recurrence in l (Schaeffer, G3 14 (2013) 751-758), with the
      Condon-Shortley phase (-1)^m when ``csphase``;
    - the vector tables from dP/dtheta and m P / sin(theta) via the standard
      ladder identities, scaled by 1/(l(l+1)) in the analysis direction.

Parity status: the Legendre/vector contraction and the module pipelines are
pinned against the reference's own CPU code path (golden fixtures generated
by ``tests/golden/make_golden.py`` from the reference package).  The weight
tables are pinned against independent mathematics (scipy's spherical
Legendre functions, quadrature exactness, orthonormality), but NOT against
torch-harmonics itself, which is absent here: table parity vs torch-harmonics
is "unpinned".
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "quadrature",
    "legendre_table",
    "dlegendre_tables",
    "scalar_forward_table",
    "scalar_inverse_table",
    "vector_forward_tables",
    "vector_inverse_tables",
    "legendre_forward",
    "legendre_inverse",
    "vector_legendre_forward",
    "vector_legendre_inverse",
    "prepare_irfft",
    "sht_forward",
    "sht_inverse",
    "vector_sht_forward",
    "vector_sht_inverse",
    "default_lmax",
    "default_mmax",
]


# --------------------------------------------------------------------------
# quadrature
# --------------------------------------------------------------------------

def _clenshaw_curtis_waldvogel(n: int):
    """Clenshaw-Curtis rule on [-1, 1] through Waldvogel's FFT construction.

    Nodes are cos(pi j/(n-1)) reversed, i.e. ascending from -1 to 1.
    """
    if n < 2:
        raise ValueError("Clenshaw-Curtis needs at least two points")
    x = np.cos(np.linspace(np.pi, 0.0, n))
    if n == 2:
        return x, np.array([1.0, 1.0])
    N = n - 1
    odd = np.arange(1, N, 2)
    n_odd = odd.size
    n_rest = N - n_odd
    # Fejer-2 moment vector, then the Clenshaw-Curtis correction g.
    v0 = np.concatenate([2.0 / odd / (odd - 2.0), [1.0 / odd[-1]], np.zeros(n_rest)])
    v2 = -v0[:-1] - v0[:0:-1]
    g0 = -np.ones(N)
    g0[n_odd] += N
    g0[n_rest] += N
    g = g0 / (N * N - 1 + (N % 2))
    w = np.fft.ifft(v2 + g).real
    w = np.concatenate([w, w[:1]])
    return x, w


def _gauss_lobatto(n: int):
    """Gauss-Lobatto-Legendre rule: endpoints plus roots of P'_{n-1}."""
    if n < 2:
        raise ValueError("Lobatto needs at least two points")
    N = n - 1
    # Chebyshev-Gauss-Lobatto initial guess, then Newton on (1-x^2) P'_N.
    x = -np.cos(np.pi * np.arange(n) / N)
    for _ in range(100):
        p_prev = np.ones_like(x)
        p = x.copy()
        for k in range(2, N + 1):
            p_prev, p = p, ((2 * k - 1) * x * p - (k - 1) * p_prev) / k
        # p = P_N, p_prev = P_{N-1}; Newton step for the LGL nodes
        dx = (x * p - p_prev) / (n * p)
        x_new = x - dx
        x_new[0], x_new[-1] = -1.0, 1.0
        if np.max(np.abs(x_new - x)) < 1e-16:
            x = x_new
            break
        x = x_new
    p_prev = np.ones_like(x)
    p = x.copy()
    for k in range(2, N + 1):
        p_prev, p = p, ((2 * k - 1) * x * p - (k - 1) * p_prev) / k
    w = 2.0 / (N * n * p * p)
    return x, w


def quadrature(nlat: int, grid: str):
    """(cos theta nodes ascending in x, weights) exactly as the reference's
    torch-harmonics constructor orders them before the flip."""
    if grid == "equiangular":
        return _clenshaw_curtis_waldvogel(nlat)
    if grid == "legendre-gauss":
        return np.polynomial.legendre.leggauss(nlat)
    if grid == "lobatto":
        return _gauss_lobatto(nlat)
    raise ValueError(f"unknown grid {grid!r}")


def default_lmax(nlat: int, grid: str) -> int:
    return nlat - 1 if grid == "lobatto" else nlat


def default_mmax(nlon: int) -> int:
    return nlon // 2 + 1


def _colatitudes(nlat: int, grid: str):
    cost, w = quadrature(nlat, grid)
    theta = np.flip(np.arccos(cost))  # north pole first
    return theta, np.asarray(w, dtype=np.float64)


# --------------------------------------------------------------------------
# associated Legendre functions
# --------------------------------------------------------------------------

def legendre_table(mmax: int, lmax: int, theta: np.ndarray, norm: str = "ortho",
                   inverse: bool = False, csphase: bool = True) -> np.ndarray:
    """P[m, l, k] = normalised P_l^m(cos theta_k) (zero for m > l).

    ``norm``: "ortho" (unit L2 norm on the sphere), "four-pi", "schmidt".
    """
    x = np.cos(theta)
    s = np.sqrt((1.0 + x) * (1.0 - x))
    nmax = max(mmax, lmax)
    out = np.zeros((nmax, nmax, x.size), dtype=np.float64)
    base = 1.0 if norm == "ortho" else math.sqrt(4.0 * math.pi)
    if inverse:
        base = 1.0 / base
    diag = np.full_like(x, base / math.sqrt(4.0 * math.pi))
    for m in range(nmax):
        if m > 0:
            diag = math.sqrt((2.0 * m + 1.0) / (2.0 * m)) * s * diag
        out[m, m] = diag
        if m + 1 < nmax:
            out[m, m + 1] = math.sqrt(2.0 * m + 3.0) * x * diag
        for l in range(m + 2, nmax):
            a = math.sqrt((4.0 * l * l - 1.0) / (l * l - m * m))
            b = math.sqrt(((l - 1.0) ** 2 - m * m) * (2.0 * l + 1.0)
                          / ((2.0 * l - 3.0) * (l * l - m * m)))
            out[m, l] = a * x * out[m, l - 1] - b * out[m, l - 2]
    if norm == "schmidt":
        scale = np.sqrt(2.0 * np.arange(nmax) + 1.0)
        out *= (scale if inverse else 1.0 / scale)[None, :, None]
    out = out[:mmax, :lmax]
    if csphase:
        out[1::2] *= -1.0
    return np.ascontiguousarray(out)


def dlegendre_tables(mmax: int, lmax: int, theta: np.ndarray, norm: str = "ortho",
                     inverse: bool = False, csphase: bool = True) -> np.ndarray:
    """D[0] = dP_l^m/dtheta, D[1] = m P_l^m / sin(theta) (as its ladder
    identity, finite at the poles); shape [2, mmax, lmax, nlat]."""
    p = legendre_table(mmax + 1, lmax + 1, theta, norm=norm, inverse=inverse, csphase=False)
    out = np.zeros((2, mmax, lmax, theta.size), dtype=np.float64)
    l = np.arange(lmax, dtype=np.float64)[:, None]
    for m in range(mmax):
        up = p[m + 1, :lmax]          # P_l^{m+1}, zero where m+1 > l
        if m == 0:
            out[0, 0] = -np.sqrt(l * (l + 1.0)) * up
        else:
            down = p[m - 1, :lmax]
            out[0, m] = 0.5 * (np.sqrt(np.maximum((l + m) * (l - m + 1.0), 0.0)) * down
                               - np.sqrt(np.maximum((l - m) * (l + m + 1.0), 0.0)) * up)
            out[1, m] = 0.5 * np.sqrt((2.0 * l + 1.0) / (2.0 * l + 3.0)) * (
                np.sqrt(np.maximum((l - m + 1.0) * (l - m + 2.0), 0.0)) * p[m - 1, 1 : lmax + 1]
                + np.sqrt((l + m + 1.0) * (l + m + 2.0)) * p[m + 1, 1 : lmax + 1])
        out[:, m, :m] = 0.0  # only l >= m exists
    if csphase:
        out[:, 1::2] *= -1.0
    return out


def scalar_forward_table(nlat, nlon, lmax=None, mmax=None, grid="equiangular",
                         norm="ortho", csphase=True) -> np.ndarray:
    """RealSHT weights [mmax, lmax, nlat]: quadrature weight x P."""
    lmax = lmax or default_lmax(nlat, grid)
    mmax = mmax or default_mmax(nlon)
    theta, w = _colatitudes(nlat, grid)
    return legendre_table(mmax, lmax, theta, norm, False, csphase) * w[None, None, :]


def scalar_inverse_table(nlat, nlon, lmax=None, mmax=None, grid="equiangular",
                         norm="ortho", csphase=True) -> np.ndarray:
    """InverseRealSHT pct [mmax, lmax, nlat]."""
    lmax = lmax or default_lmax(nlat, grid)
    mmax = mmax or default_mmax(nlon)
    theta, _ = _colatitudes(nlat, grid)
    return legendre_table(mmax, lmax, theta, norm, True, csphase)


def vector_forward_tables(nlat, nlon, lmax=None, mmax=None, grid="equiangular",
                          norm="ortho", csphase=True) -> np.ndarray:
    """RealVectorSHT weights [2, mmax, lmax, nlat]."""
    lmax = lmax or default_lmax(nlat, grid)
    mmax = mmax or default_mmax(nlon)
    theta, w = _colatitudes(nlat, grid)
    d = dlegendre_tables(mmax, lmax, theta, norm, False, csphase)
    l = np.arange(lmax, dtype=np.float64)
    lscale = np.ones(lmax)
    lscale[1:] = 1.0 / (l[1:] * (l[1:] + 1.0))
    d = d * w[None, None, None, :] * lscale[None, None, :, None]
    d[1] *= -1.0
    return d


def vector_inverse_tables(nlat, nlon, lmax=None, mmax=None, grid="equiangular",
                          norm="ortho", csphase=True) -> np.ndarray:
    """InverseRealVectorSHT dpct [2, mmax, lmax, nlat]."""
    lmax = lmax or default_lmax(nlat, grid)
    mmax = mmax or default_mmax(nlon)
    theta, _ = _colatitudes(nlat, grid)
    return dlegendre_tables(mmax, lmax, theta, norm, True, csphase)


# --------------------------------------------------------------------------
# contractions (op level)  -- tables in the reference op layout [L, K, M]
# --------------------------------------------------------------------------

def legendre_forward(x: np.ndarray, weight_t: np.ndarray) -> np.ndarray:
    """out[b,l,m] = sum_k weight_t[l,k,m] x[b,k,m]  (fused_legendre_forward)."""
    return np.einsum("bkm,lkm->blm", x, weight_t)


def legendre_inverse(c: np.ndarray, weight_t: np.ndarray) -> np.ndarray:
    """out[b,k,m] = sum_l weight_t[l,k,m] c[b,l,m]  (fused_legendre_inverse)."""
    return np.einsum("blm,lkm->bkm", c, weight_t)


def vector_legendre_forward(x: np.ndarray, w0_t: np.ndarray, w1_t: np.ndarray,
                            conj_w1: bool = False) -> np.ndarray:
    """[B,2,K,M] -> [B,2,L,M]: sph = W0 c0 + i W1 c1, tor = i W1 c0 - W0 c1.

    ``conj_w1`` flips the sign of the W1 terms, which turns the map into the
    conjugate transpose used by autograd."""
    s1 = -1.0 if conj_w1 else 1.0
    c0, c1 = x[:, 0], x[:, 1]
    a00 = np.einsum("bkm,lkm->blm", c0, w0_t)
    a11 = np.einsum("bkm,lkm->blm", c1, w1_t) * s1
    a10 = np.einsum("bkm,lkm->blm", c0, w1_t) * s1
    a01 = np.einsum("bkm,lkm->blm", c1, w0_t)
    return np.stack([a00 + 1j * a11, 1j * a10 - a01], axis=1)


def vector_legendre_inverse(c: np.ndarray, w0_t: np.ndarray, w1_t: np.ndarray,
                            conj_w1: bool = False) -> np.ndarray:
    """[B,2,L,M] -> [B,2,K,M]: c0 = D0 sph + i D1 tor, c1 = i D1 sph - D0 tor."""
    s1 = -1.0 if conj_w1 else 1.0
    sph, tor = c[:, 0], c[:, 1]
    a00 = np.einsum("blm,lkm->bkm", sph, w0_t)
    a11 = np.einsum("blm,lkm->bkm", tor, w1_t) * s1
    a10 = np.einsum("blm,lkm->bkm", sph, w1_t) * s1
    a01 = np.einsum("blm,lkm->bkm", tor, w0_t)
    return np.stack([a00 + 1j * a11, 1j * a10 - a01], axis=1)


def prepare_irfft(x: np.ndarray, nlon: int) -> np.ndarray:
    """Zero-pad m to nlon//2+1 and drop Im at m=0 and (even nlon) m=nlon/2."""
    full = nlon // 2 + 1
    out = np.zeros(x.shape[:-1] + (full,), dtype=np.complex128)
    mm = min(full, x.shape[-1])
    out[..., :mm] = x[..., :mm]
    out[..., 0] = out[..., 0].real
    if nlon % 2 == 0:
        out[..., nlon // 2] = out[..., nlon // 2].real
    return out


# --------------------------------------------------------------------------
# full transforms (module level), tables in the torch-harmonics layout
# --------------------------------------------------------------------------

def _spectrum(x: np.ndarray, mmax: int) -> np.ndarray:
    return 2.0 * np.pi * np.fft.rfft(np.asarray(x, np.float64), axis=-1, norm="forward")[..., :mmax]


def sht_forward(x: np.ndarray, weights: np.ndarray) -> np.ndarray:
    """RealSHT.forward: weights [M, L, K]; x [..., K, nlon] -> [..., L, M]."""
    X = _spectrum(x, weights.shape[0])
    return np.einsum("...km,mlk->...lm", X, weights)


def sht_inverse(c: np.ndarray, pct: np.ndarray, nlon: int) -> np.ndarray:
    """InverseRealSHT.forward: pct [M, L, K]; c [..., L, M] -> [..., K, nlon]."""
    y = np.einsum("...lm,mlk->...km", c, pct)
    return np.fft.irfft(prepare_irfft(y, nlon), n=nlon, axis=-1, norm="forward")


def vector_sht_forward(x: np.ndarray, weights: np.ndarray) -> np.ndarray:
    """RealVectorSHT.forward: weights [2, M, L, K]; x [..., 2, K, nlon]."""
    X = _spectrum(x, weights.shape[1])
    c0, c1 = X[..., 0, :, :], X[..., 1, :, :]
    w0, w1 = weights[0], weights[1]
    f = lambda a, w: np.einsum("...km,mlk->...lm", a, w)
    sph = f(c0, w0) + 1j * f(c1, w1)
    tor = 1j * f(c0, w1) - f(c1, w0)
    return np.stack([sph, tor], axis=-3)


def vector_sht_inverse(c: np.ndarray, dpct: np.ndarray, nlon: int) -> np.ndarray:
    """InverseRealVectorSHT.forward: dpct [2, M, L, K]; c [..., 2, L, M]."""
    sph, tor = c[..., 0, :, :], c[..., 1, :, :]
    d0, d1 = dpct[0], dpct[1]
    f = lambda a, w: np.einsum("...lm,mlk->...km", a, w)
    c0 = f(sph, d0) + 1j * f(tor, d1)
    c1 = 1j * f(sph, d1) - f(tor, d0)
    y = np.stack([c0, c1], axis=-3)
    return np.fft.irfft(prepare_irfft(y, nlon), n=nlon, axis=-1, norm="forward")


# --------------------------------------------------------------------------
# fp32 CPU path used only as the timed CPU baseline (bench.py cpu_baseline)
# --------------------------------------------------------------------------

class CpuForwardBaseline:
    """The reference's CPU path restated for timing: rfft then one per-order
    GEMM per table (the reference's CPU branch is a torch einsum over the same
    tables, ``__init__.py:1130-1132`` and ``:1680-1692``).  fp32, all cores
    through the BLAS numpy links against."""

    def __init__(self, weights: np.ndarray, vector: bool):
        self.vector = vector
        w = np.asarray(weights, np.float32)
        # [.., M, L, K] -> [.., M, K, L] so each order is one contiguous GEMM
        self.w = np.ascontiguousarray(np.swapaxes(w, -1, -2))
        self.mmax = w.shape[-3]

    def __call__(self, x: np.ndarray) -> np.ndarray:
        X = (2.0 * np.pi) * np.fft.rfft(x, axis=-1, norm="forward")[..., : self.mmax]
        X = X.astype(np.complex64)
        if not self.vector:
            lead = X.shape[:-2]
            K = X.shape[-2]
            Xr = X.reshape(-1, K, self.mmax)
            planes = np.concatenate([Xr.real, Xr.imag], axis=0)  # [2B, K, M]
            pm = np.ascontiguousarray(planes.transpose(2, 0, 1))  # [M, 2B, K]
            o = np.matmul(pm, self.w)  # [M, 2B, L]
            B = Xr.shape[0]
            res = (o[:, :B] + 1j * o[:, B:]).transpose(1, 2, 0)
            return res.reshape(lead + res.shape[1:])
        lead = X.shape[:-3]
        K = X.shape[-2]
        Xr = X.reshape(-1, 2, K, self.mmax)
        B = Xr.shape[0]
        planes = np.concatenate([Xr[:, 0].real, Xr[:, 0].imag, Xr[:, 1].real, Xr[:, 1].imag], axis=0)
        pm = np.ascontiguousarray(planes.transpose(2, 0, 1))  # [M, 4B, K]
        r = np.matmul(pm, self.w[0])  # W0 applied to (c0re, c0im, c1re, c1im)
        s = np.matmul(pm, self.w[1])  # W1 applied
        c0re, c0im, c1re, c1im = (slice(i * B, (i + 1) * B) for i in range(4))
        sph = (r[:, c0re] - s[:, c1im]) + 1j * (r[:, c0im] + s[:, c1re])
        tor = (-s[:, c0im] - r[:, c1re]) + 1j * (s[:, c0re] - r[:, c1im])
        out = np.stack([sph, tor], axis=1).transpose(2, 1, 3, 0)  # [B, 2, L, M]
        return out.reshape(lead + out.shape[1:])
