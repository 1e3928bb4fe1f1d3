"""CPU tests of the oracle: pinned to mathematics and to the reference's own
CPU code path (golden fixtures made by tests/golden/make_golden.py)."""
import numpy as np
import pytest
from scipy.special import sph_legendre_p

from oracle import sht_oracle as orc

GOLDEN = ["eq12x24", "lg10x20_l8_m7", "eq9x17_odd", "lob8x16"]


def rel_l2(a, b):
    a = np.asarray(a, np.complex128)
    b = np.asarray(b, np.complex128)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


# ---------------------------------------------------------------- quadrature

@pytest.mark.parametrize("n", [2, 3, 5, 8, 17, 64])
def test_clenshaw_curtis_exactness(n):
    x, w = orc.quadrature(n, "equiangular")
    assert np.all(np.diff(x) > 0)
    for d in range(n):
        exact = 2.0 / (d + 1) if d % 2 == 0 else 0.0
        assert abs(np.sum(w * x**d) - exact) < 1e-13


@pytest.mark.parametrize("n", [3, 6, 11])
def test_lobatto_exactness(n):
    x, w = orc.quadrature(n, "lobatto")
    assert x[0] == -1.0 and x[-1] == 1.0
    for d in range(2 * n - 2):
        exact = 2.0 / (d + 1) if d % 2 == 0 else 0.0
        assert abs(np.sum(w * x**d) - exact) < 1e-13


def test_gauss_exactness():
    x, w = orc.quadrature(9, "legendre-gauss")
    for d in range(18):
        exact = 2.0 / (d + 1) if d % 2 == 0 else 0.0
        assert abs(np.sum(w * x**d) - exact) < 1e-13


# ---------------------------------------------------------------- Legendre

def test_orthonormal_legendre_matches_scipy():
    theta = np.linspace(0.05, np.pi - 0.05, 11)
    P = orc.legendre_table(12, 12, theta, norm="ortho", csphase=True)
    for m in range(12):
        for l in range(12):
            ref = np.ravel(sph_legendre_p(l, m, theta)) if l >= m else 0.0 * theta
            np.testing.assert_allclose(P[m, l], ref, atol=1e-13)


def test_csphase_flips_odd_orders():
    theta = np.linspace(0.1, 3.0, 5)
    a = orc.legendre_table(6, 6, theta, csphase=True)
    b = orc.legendre_table(6, 6, theta, csphase=False)
    np.testing.assert_array_equal(a[0::2], b[0::2])
    np.testing.assert_array_equal(a[1::2], -b[1::2])


def test_schmidt_and_fourpi_scaling():
    theta = np.linspace(0.1, 3.0, 5)
    o = orc.legendre_table(5, 5, theta, norm="ortho")
    f = orc.legendre_table(5, 5, theta, norm="four-pi")
    s = orc.legendre_table(5, 5, theta, norm="schmidt")
    np.testing.assert_allclose(f, o * np.sqrt(4 * np.pi), atol=1e-13)
    l = np.arange(5)[None, :, None]
    np.testing.assert_allclose(s, f / np.sqrt(2 * l + 1), atol=1e-13)
    fi = orc.legendre_table(5, 5, theta, norm="four-pi", inverse=True)
    np.testing.assert_allclose(fi, o / np.sqrt(4 * np.pi), atol=1e-13)


def test_discrete_orthonormality_gauss():
    # Gauss rule with n nodes is exact for degree 2n-1: sum_k w_k P_l^m P_l'^m = delta / (2 pi)
    nlat, L = 24, 12
    cost, w = orc.quadrature(nlat, "legendre-gauss")
    theta = np.flip(np.arccos(cost))
    P = orc.legendre_table(L, L, theta)
    for m in range(L):
        G = (P[m] * w) @ P[m].T * 2 * np.pi
        I = np.diag((np.arange(L) >= m).astype(float))
        np.testing.assert_allclose(G, I, atol=1e-12)


def test_vector_tables_are_derivatives():
    theta = np.linspace(0.2, 2.9, 7)
    D = orc.dlegendre_tables(7, 7, theta)
    h = 1e-6
    num = (orc.legendre_table(7, 7, theta + h) - orc.legendre_table(7, 7, theta - h)) / (2 * h)
    np.testing.assert_allclose(D[0], num, atol=1e-7)
    m = np.arange(7)[:, None, None]
    np.testing.assert_allclose(D[1], m * orc.legendre_table(7, 7, theta) / np.sin(theta), atol=1e-12)


def test_vector_tables_finite_at_poles():
    d = orc.vector_forward_tables(9, 16)
    assert np.all(np.isfinite(d))


# ---------------------------------------------------------------- transforms

def test_scalar_roundtrip_gauss():
    nlat, nlon = 16, 32
    W = orc.scalar_forward_table(nlat, nlon, grid="legendre-gauss")
    P = orc.scalar_inverse_table(nlat, nlon, grid="legendre-gauss")
    L, M = W.shape[1], W.shape[0]
    rng = np.random.default_rng(0)
    c = (rng.standard_normal((2, L, M)) + 1j * rng.standard_normal((2, L, M)))
    c *= (np.arange(M)[None, :] <= np.arange(L)[:, None])
    c[..., 0] = c[..., 0].real
    c[..., M - 1] = c[..., M - 1].real  # nyquist (M = nlon/2+1) is real
    x = orc.sht_inverse(c, P, nlon)
    c2 = orc.sht_forward(x, W)
    # the Nyquist column is not represented for l < nlat modes beyond the grid; compare the rest
    assert rel_l2(c2[..., : M - 1], c[..., : M - 1]) < 1e-12


def test_vector_roundtrip_gauss():
    nlat, nlon = 16, 32
    W = orc.vector_forward_tables(nlat, nlon, grid="legendre-gauss")
    D = orc.vector_inverse_tables(nlat, nlon, grid="legendre-gauss")
    L, M = W.shape[2], W.shape[1]
    rng = np.random.default_rng(1)
    c = (rng.standard_normal((2, 2, L, M)) + 1j * rng.standard_normal((2, 2, L, M)))
    c *= (np.arange(M)[None, :] <= np.arange(L)[:, None])
    c[..., 0, :] = 0.0  # l = 0 has no vector mode
    c[..., 0] = c[..., 0].real
    c = c[..., : M - 1]
    c = np.concatenate([c, np.zeros(c.shape[:-1] + (1,))], axis=-1)
    x = orc.vector_sht_inverse(c, D, nlon)
    c2 = orc.vector_sht_forward(x, W)
    assert rel_l2(c2[..., :-1], c[..., :-1]) < 1e-11


# ---------------------------------------------------------------- golden pins

@pytest.mark.parametrize("name", GOLDEN)
def test_oracle_matches_reference_cpu_path(golden_dir, name):
    g = np.load(golden_dir / f"{name}.npz")
    nlat, nlon = int(g["nlat"]), int(g["nlon"])
    kw = dict(lmax=int(g["lmax"]), mmax=int(g["mmax"]), grid=str(g["grid"]))
    W = orc.scalar_forward_table(nlat, nlon, **kw)
    P = orc.scalar_inverse_table(nlat, nlon, **kw)
    V = orc.vector_forward_tables(nlat, nlon, **kw)
    D = orc.vector_inverse_tables(nlat, nlon, **kw)
    assert rel_l2(orc.sht_forward(g["x"], W), g["sht"]) < 2e-6
    assert rel_l2(orc.vector_sht_forward(g["xv"], V), g["vsht"]) < 2e-6
    assert rel_l2(orc.sht_inverse(g["c"], P, nlon), g["isht"]) < 2e-6
    assert rel_l2(orc.vector_sht_inverse(g["cv"], D, nlon), g["ivsht"]) < 2e-6


def test_oracle_ops_match_reference_kats(golden_dir):
    g = np.load(golden_dir / "ops_tri.npz")
    wt = g["weight_t"].astype(np.float64)
    assert rel_l2(orc.legendre_forward(g["x"], wt), g["fwd"]) < 1e-6
    assert rel_l2(orc.legendre_inverse(g["c"], wt), g["inv"]) < 1e-6
    assert rel_l2(orc.legendre_forward(g["x"].real, wt), g["fwd_real"]) < 1e-6
    assert rel_l2(orc.legendre_inverse(g["c"].real, wt), g["inv_real"]) < 1e-6
    np.testing.assert_allclose(orc.prepare_irfft(g["c"], 20), g["prep_even"], atol=0)
    np.testing.assert_allclose(orc.prepare_irfft(g["c"], 19), g["prep_odd"], atol=0)


def test_cpu_baseline_matches_oracle():
    nlat, nlon = 12, 24
    W = orc.scalar_forward_table(nlat, nlon)
    V = orc.vector_forward_tables(nlat, nlon)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3, nlat, nlon)).astype(np.float32)
    xv = rng.standard_normal((3, 2, nlat, nlon)).astype(np.float32)
    assert rel_l2(orc.CpuForwardBaseline(W, vector=False)(x), orc.sht_forward(x, W)) < 1e-5
    assert rel_l2(orc.CpuForwardBaseline(V, vector=True)(xv), orc.vector_sht_forward(xv, V)) < 1e-5
