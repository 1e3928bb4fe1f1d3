"""Host-side construction of the Legendre weight tables.

The reference's modules obtain their tables from torch-harmonics at
construction time (``torch-ext/holysht/__init__.py:1247-1273`` for RealSHT,
:1406-1424 InverseRealSHT, :1452-1480 RealVectorSHT, :1710-1730
InverseRealVectorSHT).  When torch-harmonics is importable this module does
exactly that.  Otherwise it builds the same tables in float64 from the
mathematics they are defined by:

* equiangular grid: Clenshaw-Curtis weights from the closed-form cosine sum
  w_j = c_j/(n-1) * (1 - sum_k b_k cos(2 k theta_j) / (4 k^2 - 1));
* legendre-gauss grid: numpy's Gauss-Legendre rule;
* lobatto grid: Gauss-Lobatto-Legendre rule (Newton on (1-x^2) P'_{n-1});
* orthonormal associated Legendre functions P_l^m(cos theta) by the
  three-term recurrence in l, all orders at once (vectorised over m);
* vector tables: dP/dtheta and m P / sin(theta) from the ladder identities.

Layout returned: ``[mmax, lmax, nlat]`` (``[2, mmax, lmax, nlat]`` for the
vector tables), the torch-harmonics layout; nodes run north pole first.
"""
from __future__ import annotations

import math

import numpy as np
import torch

GRIDS = ("equiangular", "legendre-gauss", "lobatto")
NORMS = ("ortho", "four-pi", "schmidt")


def _check(grid: str, norm: str) -> None:
    if grid not in GRIDS:
        raise ValueError(f"Unknown quadrature mode {grid!r}; expected one of {GRIDS}")
    if norm not in NORMS:
        raise ValueError(f"Unknown normalization {norm!r}; expected one of {NORMS}")


def default_lmax(nlat: int, grid: str) -> int:
    return nlat - 1 if grid == "lobatto" else nlat


def default_mmax(nlon: int) -> int:
    return nlon // 2 + 1


def clenshaw_curtis(n: int):
    """Nodes x_j = -cos(pi j/(n-1)) (ascending) and Clenshaw-Curtis weights."""
    if n < 2:
        raise ValueError("equiangular grid needs nlat >= 2")
    N = n - 1
    theta = np.pi * np.arange(n) / N
    x = -np.cos(theta)
    if n == 2:
        return x, np.ones(2)
    w = np.ones(n)
    half = N // 2
    for k in range(1, half + 1):
        b = 1.0 if 2 * k == N else 2.0
        w -= b * np.cos(2.0 * k * theta) / (4.0 * k * k - 1.0)
    c = np.full(n, 2.0)
    c[0] = c[-1] = 1.0
    return x, c * w / N


def gauss_lobatto(n: int):
    if n < 2:
        raise ValueError("lobatto grid needs nlat >= 2")
    N = n - 1
    x = -np.cos(np.pi * np.arange(n) / N)
    for _ in range(200):
        p0, p1 = np.ones_like(x), x.copy()
        for k in range(2, N + 1):
            p0, p1 = p1, ((2.0 * k - 1.0) * x * p1 - (k - 1.0) * p0) / k
        step = (x * p1 - p0) / (n * p1)
        step[0] = step[-1] = 0.0
        x = x - step
        if np.max(np.abs(step)) < 1e-16:
            break
    p0, p1 = np.ones_like(x), x.copy()
    for k in range(2, N + 1):
        p0, p1 = p1, ((2.0 * k - 1.0) * x * p1 - (k - 1.0) * p0) / k
    return x, 2.0 / (N * n * p1 * p1)


def nodes_and_weights(nlat: int, grid: str):
    """(colatitudes north-first, quadrature weights)."""
    if grid == "equiangular":
        x, w = clenshaw_curtis(nlat)
    elif grid == "legendre-gauss":
        x, w = np.polynomial.legendre.leggauss(nlat)
    elif grid == "lobatto":
        x, w = gauss_lobatto(nlat)
    else:
        raise ValueError(f"Unknown quadrature mode {grid!r}")
    return np.flip(np.arccos(x)).copy(), np.asarray(w, np.float64)


def _legendre_rows(n_m: int, n_l: int, x: np.ndarray, seed: float, device=None):
    """Yield (l, row) with row[m, k] = P_l^m(x_k) (no Condon-Shortley phase,
    zero for m > l), for l = 0 .. n_l-1 and all m < n_m at once, as float64
    torch tensors on ``device`` (default: the host; row is only valid until
    the next step).

    The recurrence runs upwards in l for every order simultaneously, keeping
    only the two previous rows, so memory stays O(n_m * nlat); the row updates
    are multi-threaded torch operations."""
    dev = torch.device("cpu") if device is None else torch.device(device)
    f64 = dict(dtype=torch.float64, device=dev)
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float64)).to(dev)
    sin_t = torch.sqrt((1.0 + xt) * (1.0 - xt))
    K = xt.numel()
    mm = torch.arange(n_m, **f64)
    sect = torch.full((K,), float(seed), **f64)  # P_l^l at the current l
    prev2 = torch.zeros((n_m, K), **f64)
    prev1 = torch.zeros((n_m, K), **f64)
    row = torch.zeros((n_m, K), **f64)
    for l in range(n_l):
        if l > 0:
            sect = math.sqrt((2.0 * l + 1.0) / (2.0 * l)) * sin_t * sect
        row.zero_()
        if l >= 2:
            k = min(l - 1, n_m)
            m = mm[:k]
            a = torch.sqrt((4.0 * l * l - 1.0) / (l * l - m * m))
            b = torch.sqrt(((l - 1.0) ** 2 - m * m) * (2.0 * l + 1.0) / ((2.0 * l - 3.0) * (l * l - m * m)))
            torch.mul(prev1[:k], xt[None, :], out=row[:k])
            row[:k].mul_(a[:, None]).addcmul_(prev2[:k], b[:, None], value=-1.0)
        if l >= 1 and l - 1 < n_m:
            row[l - 1] = math.sqrt(2.0 * l + 1.0) * xt * prev1[l - 1]
        if l < n_m:
            row[l] = sect
        yield l, row
        prev2, prev1, row = prev1, row, prev2


def _norm_seed(norm: str, inverse: bool) -> float:
    f = 1.0 if norm == "ortho" else math.sqrt(4.0 * math.pi)
    f = 1.0 / f if inverse else f
    return f / math.sqrt(4.0 * math.pi)


def _schmidt(norm: str, inverse: bool, l: int) -> float:
    if norm != "schmidt":
        return 1.0
    s = math.sqrt(2.0 * l + 1.0)
    return s if inverse else 1.0 / s


def _torch_dtype(dtype):
    return torch.float32 if np.dtype(dtype) == np.float32 else torch.float64


def legendre(mmax: int, lmax: int, theta: np.ndarray, norm: str = "ortho",
             inverse: bool = False, csphase: bool = True, kscale=None,
             dtype=np.float64, device=None):
    """[mmax, lmax, nlat] normalised associated Legendre functions, each
    latitude optionally multiplied by ``kscale`` (the quadrature weights).
    A numpy array, or a torch tensor on ``device`` when one is given."""
    x = np.cos(theta)
    dev = torch.device("cpu") if device is None else torch.device(device)
    out = torch.zeros((mmax, lmax, x.size), dtype=_torch_dtype(dtype), device=dev)
    sign = torch.ones(mmax, dtype=torch.float64, device=dev)
    if csphase:
        sign[1::2] = -1.0
    ks = torch.ones(x.size, dtype=torch.float64) if kscale is None else torch.from_numpy(
        np.asarray(kscale, np.float64))
    f = sign[:, None] * ks.to(dev)[None, :]
    for l, row in _legendre_rows(mmax, lmax, x, _norm_seed(norm, inverse), device):
        out[:, l, :] = row * f * _schmidt(norm, inverse, l)
    return out if device is not None else out.numpy()


def dlegendre(mmax: int, lmax: int, theta: np.ndarray, norm: str = "ortho",
              inverse: bool = False, csphase: bool = True, kscale=None, lscale=None,
              dtype=np.float64, sign1: float = 1.0, device=None):
    """[2, mmax, lmax, nlat]: dP/dtheta and m P / sin(theta), optionally
    multiplied by ``kscale[k]`` and ``lscale[l]``; the second table is also
    multiplied by ``sign1``.  A numpy array, or a torch tensor on ``device``
    when one is given."""
    x = np.cos(theta)
    K = x.size
    dev = torch.device("cpu") if device is None else torch.device(device)
    f64 = dict(dtype=torch.float64, device=dev)
    out = torch.zeros((2, mmax, lmax, K), dtype=_torch_dtype(dtype), device=dev)
    m = torch.arange(mmax, **f64)
    sign = torch.ones(mmax, **f64)
    if csphase:
        sign[1::2] = -1.0
    ks = (torch.ones(K, dtype=torch.float64) if kscale is None
          else torch.from_numpy(np.asarray(kscale, np.float64))).to(dev)
    rows = _legendre_rows(mmax + 1, lmax + 1, x, _norm_seed(norm, inverse), device)
    _, first = next(rows)
    cur = first.clone()
    d0 = torch.empty((mmax, K), **f64)
    d1 = torch.empty((mmax, K), **f64)
    for l in range(lmax):
        _, nxt = next(rows)
        cs = _schmidt(norm, inverse, l)
        ns = _schmidt(norm, inverse, l + 1)
        # d0 = (sqrt((l+m)(l-m+1)) P^{m-1}_l - sqrt((l-m)(l+m+1)) P^{m+1}_l) / 2
        ca = 0.5 * cs * torch.sqrt(torch.clamp((l + m) * (l - m + 1.0), min=0.0))
        cb = 0.5 * cs * torch.sqrt(torch.clamp((l - m) * (l + m + 1.0), min=0.0))
        torch.mul(cur[1: mmax + 1], cb[:, None], out=d0)
        d0.neg_()
        d0[1:].addcmul_(cur[: mmax - 1], ca[1:, None])
        d0[0] = -math.sqrt(l * (l + 1.0)) * cs * cur[1]
        # d1 = F (sqrt((l-m+1)(l-m+2)) P^{m-1}_{l+1} + sqrt((l+m+1)(l+m+2)) P^{m+1}_{l+1})
        F = 0.5 * math.sqrt((2.0 * l + 1.0) / (2.0 * l + 3.0)) * ns
        ga = F * torch.sqrt(torch.clamp((l - m + 1.0) * (l - m + 2.0), min=0.0))
        gb = F * torch.sqrt((l + m + 1.0) * (l + m + 2.0))
        torch.mul(nxt[1: mmax + 1], gb[:, None], out=d1)
        d1[1:].addcmul_(nxt[: mmax - 1], ga[1:, None])
        d1[0] = 0.0
        keep = (m <= l).to(torch.float64)
        fs = sign * keep * (1.0 if lscale is None else float(lscale[l]))
        f = fs[:, None] * ks[None, :]
        out[0, :, l, :] = d0 * f
        out[1, :, l, :] = d1 * f * sign1
        cur.copy_(nxt)
    return out if device is not None else out.numpy()


def _try_torch_harmonics():
    """torch-harmonics when importable (``restated=True`` in the builders below
    skips it and always uses the float64 restatement)."""
    try:
        import torch_harmonics  # noqa: F401
        return torch_harmonics
    except Exception:
        return None


def _from_th(t, dtype, device):
    """A torch-harmonics table as numpy (``device`` None) or a tensor on ``device``."""
    if device is None:
        return t.double().numpy().astype(dtype)
    return t.to(device=device, dtype=_torch_dtype(dtype))


def _resolve(nlat, nlon, lmax, mmax, grid, norm):
    _check(grid, norm)
    lmax = lmax or default_lmax(nlat, grid)
    mmax = mmax or default_mmax(nlon)
    return lmax, mmax


def scalar_forward(nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                   dtype=np.float64, restated=False, device=None):
    """RealSHT ``weights`` [mmax, lmax, nlat] (float64) and (lmax, mmax)."""
    th = None if restated else _try_torch_harmonics()
    if th is not None:
        ref = th.RealSHT(nlat, nlon, lmax=lmax, mmax=mmax, grid=grid, norm=norm, csphase=csphase)
        return _from_th(ref.weights, dtype, device), ref.lmax, ref.mmax
    lmax, mmax = _resolve(nlat, nlon, lmax, mmax, grid, norm)
    theta, w = nodes_and_weights(nlat, grid)
    return legendre(mmax, lmax, theta, norm, False, csphase, kscale=w, dtype=dtype, device=device), lmax, mmax


def scalar_inverse(nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                   dtype=np.float64, restated=False, device=None):
    """InverseRealSHT ``pct`` [mmax, lmax, nlat]."""
    th = None if restated else _try_torch_harmonics()
    if th is not None:
        ref = th.InverseRealSHT(nlat, nlon, lmax=lmax, mmax=mmax, grid=grid, norm=norm, csphase=csphase)
        return _from_th(ref.pct, dtype, device), ref.lmax, ref.mmax
    lmax, mmax = _resolve(nlat, nlon, lmax, mmax, grid, norm)
    theta, _ = nodes_and_weights(nlat, grid)
    return legendre(mmax, lmax, theta, norm, True, csphase, dtype=dtype, device=device), lmax, mmax


def vector_forward(nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                   dtype=np.float64, restated=False, device=None):
    """RealVectorSHT ``weights`` [2, mmax, lmax, nlat]."""
    th = None if restated else _try_torch_harmonics()
    if th is not None:
        ref = th.RealVectorSHT(nlat, nlon, lmax=lmax, mmax=mmax, grid=grid, norm=norm, csphase=csphase)
        return _from_th(ref.weights, dtype, device), ref.lmax, ref.mmax
    lmax, mmax = _resolve(nlat, nlon, lmax, mmax, grid, norm)
    theta, w = nodes_and_weights(nlat, grid)
    ll = np.arange(lmax, dtype=np.float64)
    lscale = np.ones(lmax)
    lscale[1:] = 1.0 / (ll[1:] * (ll[1:] + 1.0))
    d = dlegendre(mmax, lmax, theta, norm, False, csphase, kscale=w, lscale=lscale, dtype=dtype, sign1=-1.0,
                  device=device)
    return d, lmax, mmax


def vector_inverse(nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                   dtype=np.float64, restated=False, device=None):
    """InverseRealVectorSHT ``dpct`` [2, mmax, lmax, nlat]."""
    th = None if restated else _try_torch_harmonics()
    if th is not None:
        ref = th.InverseRealVectorSHT(nlat, nlon, lmax=lmax, mmax=mmax, grid=grid, norm=norm, csphase=csphase)
        return _from_th(ref.dpct, dtype, device), ref.lmax, ref.mmax
    lmax, mmax = _resolve(nlat, nlon, lmax, mmax, grid, norm)
    theta, _ = nodes_and_weights(nlat, grid)
    return dlegendre(mmax, lmax, theta, norm, True, csphase, dtype=dtype, device=device), lmax, mmax


SEGMENT = 16  # degrees between recurrence checkpoints (matches the kernel)


def scalar_recurrence_tables(nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True,
                             inverse=False, segment=SEGMENT):
    """Inputs of the recurrence kernel, built in float64, returned as float32:

    * seeds [mmax, ceil(lmax/16), nlat, 2]: w_k * P_l^m(x_k) at l = m + 16c and
      m + 16c + 1 (normalisation, Schmidt factor, Condon-Shortley phase and
      quadrature weight included; zero outside l < lmax);
    * coef [mmax, lmax, 2]: (a_lm, b_lm) of P_l = a x P_{l-1} - b P_{l-2} for the
      normalised (and, for ``schmidt``, rescaled) functions, for l >= m + 2;
    * cos_theta [nlat].

    The same functions as ``scalar_forward``'s table (which is w_k P_l^m); with
    ``inverse``, those of ``scalar_inverse``'s ``pct`` (the inverse
    normalisation, no quadrature weight).  ``segment``: degrees between
    checkpoints (16 for the forward kernels, 8 for the inverse kernel)."""
    lmax, mmax = _resolve(nlat, nlon, lmax, mmax, grid, norm)
    theta, w = nodes_and_weights(nlat, grid)
    if inverse:
        w = np.ones_like(w)
    x = np.cos(theta)
    nseg = (lmax + segment - 1) // segment
    seeds = np.zeros((mmax, nseg, nlat, 2), dtype=np.float32)
    coef = np.zeros((mmax, lmax, 2), dtype=np.float32)
    sign = np.ones(mmax)
    if csphase:
        sign[1::2] = -1.0
    m_all = np.arange(mmax)
    for l, row in _legendre_rows(mmax, lmax, x, _norm_seed(norm, inverse)):
        row = row.numpy()
        f = _schmidt(norm, inverse, l)
        vals = row * (sign * f)[:, None] * w[None, :]          # [mmax, K]
        d = l - m_all
        sel = (d >= 0) & (d % segment < 2)
        ms = m_all[sel]
        seeds[ms, d[sel] // segment, :, d[sel] % segment] = vals[sel].astype(np.float32)
        if l >= 2:
            mm = m_all[(m_all <= l - 2)].astype(np.float64)
            a = np.sqrt((4.0 * l * l - 1.0) / (l * l - mm * mm))
            b = np.sqrt(((l - 1.0) ** 2 - mm * mm) * (2.0 * l + 1.0) / ((2.0 * l - 3.0) * (l * l - mm * mm)))
            a *= f / _schmidt(norm, inverse, l - 1)
            b *= f / _schmidt(norm, inverse, l - 2)
            k = mm.astype(np.int64)
            coef[k, l, 0] = a
            coef[k, l, 1] = b
    return seeds, coef, x.astype(np.float32)


def recurrence_seeds_symmetric(seeds, cos_theta, tol=1e-6) -> bool:
    """True when recurrence checkpoints obey the equatorial parity the
    ``HOLYSHT_FLAG_EQUATORIAL_PARITY`` kernels rely on: cos_theta mirrored
    (x_{K-1-k} = -x_k) and, for every checkpoint degree pair (l0, l0 + 1) of an
    order, the mirrored latitude's value equal to +/- this one's, the sign
    (-1)^(l+m') of the Legendre function's order m' (scalar seeds [..., 2]: orders
    m, signs (+, -); vector seeds [..., 4]: orders m -/+ 1, signs (-, +, -, +)).
    Checked to ``tol`` of the largest seed."""
    s = np.asarray(seeds, dtype=np.float32)
    x = np.asarray(cos_theta, dtype=np.float64)
    if x.size == 0 or np.abs(x + x[::-1]).max() > 1e-6:
        return False
    sign = np.array([1.0, -1.0] if s.shape[-1] == 2 else [-1.0, 1.0, -1.0, 1.0], dtype=np.float32)
    scale = max(float(np.abs(s).max()), 1e-30)
    err = 0.0
    for m in range(s.shape[0]):  # one order at a time: bounded temporaries
        d = s[m, :, ::-1, :] - sign * s[m]
        err = max(err, float(np.abs(d).max()) if d.size else 0.0)
    return err <= tol * scale


def compact_recurrence_seeds(seeds, lmax: int):
    """Checkpoints in the compact latitude-major layout of
    ``HOLYSHT_FLAG_SEEDS_COMPACT``: [nlat, nsegs, S] from [mmax, nseg, nlat, S],
    keeping for each order m < min(mmax, lmax) its ceil((lmax - m) / 16)
    segments, orders in turn.  A warp of the recurrence kernels owns 32
    consecutive segments, so one latitude's checkpoints are contiguous."""
    s = np.asarray(seeds)
    mlim = min(s.shape[0], lmax)
    parts = [s[m, : (lmax - m + SEGMENT - 1) // SEGMENT] for m in range(mlim)]
    flat = np.concatenate(parts, axis=0) if parts else np.zeros((0,) + s.shape[2:], s.dtype)
    return np.ascontiguousarray(flat.transpose(1, 0, 2))


def vector_recurrence_tables(nlat, nlon, lmax=None, mmax=None, grid="equiangular", norm="ortho", csphase=True):
    """Inputs of the vector recurrence kernel (float64 built, float32 returned).

    The vector tables of order m are ladder combinations of the Legendre
    functions of orders m - 1 and m + 1 (the same identities as
    :func:`dlegendre`).  With Q^{m'}_l(x_k) = w_k P_l^{m'}(x_k) (normalised,
    Schmidt factor included, no Condon-Shortley phase):

        W0[m, l, k] = alpha Q^{m-1}_l + beta Q^{m+1}_l
        W1[m, l, k] = gamma Q^{m-1}_{l+1} + delta Q^{m+1}_{l+1}

    which are ``vector_forward``'s tables (1/(l(l+1)) scaling, phase and the
    sign of the second table folded into alpha .. delta).  The kernel runs both
    recurrences upwards in l in float32, re-seeded every 16 degrees.

    * seeds [mmax, ceil(lmax/16), nlat, 4]: Q^{m-1} at l0, l0+1 and Q^{m+1} at
      l0, l0+1 for l0 = m + 16c (zero where the order does not exist);
    * coef [mmax, lmax, 8]: a, b of order m-1 and a, b of order m+1 for
      Q_{l+2} = a x Q_{l+1} - b Q_l, then alpha, beta, gamma, delta of degree l;
    * cos_theta [nlat]."""
    lmax, mmax = _resolve(nlat, nlon, lmax, mmax, grid, norm)
    theta, w = nodes_and_weights(nlat, grid)
    x = np.cos(theta)
    nseg = (lmax + SEGMENT - 1) // SEGMENT
    seeds = np.zeros((mmax, nseg, nlat, 4), dtype=np.float32)
    coef = np.zeros((mmax, lmax, 8), dtype=np.float32)
    m_all = np.arange(mmax)
    for l, row in _legendre_rows(mmax + 1, lmax + 1, x, _norm_seed(norm, False)):
        row = row.numpy()
        q = row * _schmidt(norm, False, l) * w[None, :]  # [mmax + 1, K]: Q^{m'}_l
        for off in (0, 1):  # checkpoint degrees l0 = l - off
            d = l - off - m_all
            sel = (d >= 0) & (d % SEGMENT == 0) & (l - off < lmax)
            ms = m_all[sel]
            c = d[sel] // SEGMENT
            lower = ms >= 1
            seeds[ms[lower], c[lower], :, off] = q[ms[lower] - 1].astype(np.float32)
            seeds[ms, c, :, 2 + off] = q[ms + 1].astype(np.float32)

    def rec(mp, lt):  # a, b of order mp at degree lt (lt >= mp + 1), Schmidt-rescaled
        mp = np.asarray(mp, np.float64)
        a = np.sqrt((4.0 * lt * lt - 1.0) / (lt * lt - mp * mp))
        b = np.sqrt(np.maximum((lt - 1.0) ** 2 - mp * mp, 0.0) * (2.0 * lt + 1.0)
                    / ((2.0 * lt - 3.0) * (lt * lt - mp * mp)))
        f = _schmidt(norm, False, lt)
        return a * f / _schmidt(norm, False, lt - 1), b * f / _schmidt(norm, False, lt - 2)

    sign = np.ones(mmax)
    if csphase:
        sign[1::2] = -1.0
    for l in range(lmax):
        ms = m_all[m_all <= l]
        mf = ms.astype(np.float64)
        lt = l + 2.0
        am, bm = rec(np.maximum(mf - 1.0, 0.0), lt)
        am[ms == 0] = 0.0
        bm[ms == 0] = 0.0
        ap, bp = rec(mf + 1.0, lt)
        s = sign[ms] * (1.0 / (l * (l + 1.0)) if l > 0 else 1.0)
        alpha = 0.5 * np.sqrt((l + mf) * (l - mf + 1.0))
        beta = -0.5 * np.sqrt(np.maximum((l - mf) * (l + mf + 1.0), 0.0))
        F = 0.5 * math.sqrt((2.0 * l + 1.0) / (2.0 * l + 3.0))
        gamma = F * np.sqrt(np.maximum((l - mf + 1.0) * (l - mf + 2.0), 0.0))
        delta = F * np.sqrt((l + mf + 1.0) * (l + mf + 2.0))
        z = ms == 0  # order 0: dP/dtheta = -sqrt(l(l+1)) P^1, m P / sin(theta) = 0
        alpha[z] = 0.0
        beta[z] = -math.sqrt(l * (l + 1.0))
        gamma[z] = 0.0
        delta[z] = 0.0
        coef[ms, l] = np.stack([am, bm, ap, bp, alpha * s, beta * s, -gamma * s, -delta * s], axis=1)
    return seeds, coef, x.astype(np.float32)
