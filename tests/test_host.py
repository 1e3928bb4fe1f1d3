"""CPU tests of the host side: the C ABI library loads and exports every
declared symbol, the package's weight generator agrees with the oracle, the
modules construct with the reference's buffers, and the product path refuses
CPU tensors (there is no CPU fallback)."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import holysht_b200 as hs
from holysht_b200 import _lib, weights
from oracle import sht_oracle as orc

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^\s*(?:int|const char\*)\s+(holysht_\w+)\s*\(", text, re.M))
    return names


def test_header_declares_the_exports():
    assert _declared_symbols() == set(_lib.EXPORTS)


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    assert lib.holysht_version() >= 100
    assert lib.holysht_last_error() == b""


def test_invalid_arguments_are_rejected_without_gpu():
    lib = _lib.load()
    # negative extents and null pointers are caught before any CUDA call
    st = lib.holysht_fused_legendre_forward(None, None, None, -1, 4, 4, 4, None)
    assert st == _lib.HOLYSHT_ERR_INVALID
    assert b"negative" in lib.holysht_last_error()
    st = lib.holysht_fused_legendre_forward(None, None, None, 2, 4, 4, 4, None)
    assert st == _lib.HOLYSHT_ERR_INVALID
    st = lib.holysht_fused_legendre_forward_real(None, None, 0, None, 1, 1, 1, 1, 9, None)
    assert st == _lib.HOLYSHT_ERR_INVALID and b"backend_hint" in lib.holysht_last_error()
    d = _lib.ContractDesc()
    d.kind, d.direction, d.in_dtype, d.batch, d.nlat, d.lmax, d.mmax, d.out_cols = 1, 0, 0, 1, 4, 4, 4, 2
    assert lib.holysht_legendre_contract(ctypes.byref(d), None) == _lib.HOLYSHT_ERR_INVALID
    assert b"out_cols" in lib.holysht_last_error()
    d.out_cols, d.kind = 4, 7
    assert lib.holysht_legendre_contract(ctypes.byref(d), None) == _lib.HOLYSHT_ERR_INVALID
    # empty problems are a no-op success
    assert lib.holysht_fused_legendre_forward(None, None, None, 0, 4, 4, 4, None) == _lib.HOLYSHT_OK
    with pytest.raises(RuntimeError, match="invalid extents"):
        _lib.check(lib.holysht_sht_prepare_irfft(None, -1, 4, 4, 6, None))



def test_dense_workspace_size_overflow_is_rejected():
    """Extents whose workspace size would wrap in 64 bits are refused instead of
    yielding a small size that a smaller buffer would pass."""
    lib = _lib.load()
    n = ctypes.c_int64(0)
    big = 1 << 40
    st = lib.holysht_legendre_dense_tc_workspace(_lib.DIR_FORWARD, big, big, big, big, ctypes.byref(n))
    assert st == _lib.HOLYSHT_ERR_INVALID and b"overflow" in lib.holysht_last_error()
    st = lib.holysht_legendre_dense_tc_workspace(_lib.DIR_FORWARD, 65535, 1 << 31, 1 << 31, 1 << 31,
                                                 ctypes.byref(n))
    assert st == _lib.HOLYSHT_ERR_INVALID
    assert lib.holysht_legendre_dense_tc_workspace(_lib.DIR_FORWARD, 4, 64, 64, 65, ctypes.byref(n)) == 0
    assert n.value > 0

@pytest.mark.parametrize("grid", ["equiangular", "legendre-gauss", "lobatto"])
@pytest.mark.parametrize("norm", ["ortho", "schmidt", "four-pi"])
def test_package_tables_match_oracle(grid, norm):
    nlat, nlon = 11, 20
    for cs in (True, False):
        a, L, M = weights.scalar_forward(nlat, nlon, grid=grid, norm=norm, csphase=cs)
        np.testing.assert_allclose(a, orc.scalar_forward_table(nlat, nlon, grid=grid, norm=norm, csphase=cs), atol=1e-13)
        b, _, _ = weights.scalar_inverse(nlat, nlon, grid=grid, norm=norm, csphase=cs)
        np.testing.assert_allclose(b, orc.scalar_inverse_table(nlat, nlon, grid=grid, norm=norm, csphase=cs), atol=1e-13)
        c, _, _ = weights.vector_forward(nlat, nlon, grid=grid, norm=norm, csphase=cs)
        np.testing.assert_allclose(c, orc.vector_forward_tables(nlat, nlon, grid=grid, norm=norm, csphase=cs), atol=1e-13)
        d, _, _ = weights.vector_inverse(nlat, nlon, grid=grid, norm=norm, csphase=cs)
        np.testing.assert_allclose(d, orc.vector_inverse_tables(nlat, nlon, grid=grid, norm=norm, csphase=cs), atol=1e-13)
        assert (L, M) == (orc.default_lmax(nlat, grid), orc.default_mmax(nlon))


def test_package_tables_custom_lmax_mmax():
    a, L, M = weights.vector_forward(10, 20, lmax=6, mmax=4)
    assert a.shape == (2, 4, 6, 10) and (L, M) == (6, 4)
    np.testing.assert_allclose(a, orc.vector_forward_tables(10, 20, lmax=6, mmax=4), atol=1e-13)


def test_bad_grid_and_norm():
    with pytest.raises(ValueError):
        weights.scalar_forward(8, 16, grid="healpix")
    with pytest.raises(ValueError):
        weights.scalar_forward(8, 16, norm="bogus")


def test_module_buffers_and_shapes():
    m = hs.RealSHT(12, 24)
    assert (m.lmax, m.mmax) == (12, 13)
    assert m.weights.shape == (13, 12, 12) and m.weight_t.shape == (12, 12, 13)
    assert set(m.state_dict()) == {"weights", "weight_t"}
    v = hs.RealVectorSHT(12, 24, dtype="bf16")
    assert v.w0.dtype == torch.bfloat16 and v.w0_t.dtype == torch.float32
    assert set(v.state_dict()) == {"w0", "w1", "w0_t", "w1_t"}
    i = hs.InverseRealSHT(12, 24, lmax=8, mmax=6)
    assert i.pct.shape == (6, 8, 12) and i.pct_t.shape == (8, 12, 6)
    iv = hs.InverseRealVectorSHT(12, 24)
    assert set(iv.state_dict()) == {"d0", "d1", "d0_t", "d1_t"}
    torch.testing.assert_close(m.weight_t, m.weights.permute(1, 2, 0))


def test_aliases():
    assert hs.FusedRealSHT is hs.RealSHT
    assert hs.FusedInverseRealSHT is hs.InverseRealSHT
    assert hs.FusedRealVectorSHT is hs.RealVectorSHT
    assert hs.FusedInverseRealVectorSHT is hs.InverseRealVectorSHT
    assert hs.legendre_forward is hs.fused_legendre_forward
    assert hs.sht_inverse is hs.fused_sht_inverse


def test_cpu_tensors_fail_loudly():
    m = hs.RealSHT(8, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(2, 8, 16))
    with pytest.raises(RuntimeError, match="CUDA"):
        hs.fused_legendre_forward(torch.zeros(1, 8, 9, dtype=torch.complex64), m.weights)
    out = torch.empty(1, 8, 9, dtype=torch.complex64)
    with pytest.raises(RuntimeError, match="CUDA"):
        hs.ops.fused_legendre_forward(out, out, m.weight_t)


def test_missing_library_fails_loudly(tmp_path):
    """Without the native library the package raises; nothing falls back to a
    CPU or PyTorch implementation."""
    import subprocess
    import sys

    code = ("import torch, holysht_b200 as hs\n"
            "try:\n    hs._lib.load()\nexcept RuntimeError as e:\n    print('raised', e)\n")
    env = dict(__import__("os").environ, HOLYSHT_B200_LIBRARY=str(tmp_path / "absent.so"))
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("raised") and "not found" in r.stdout


def test_graphed_module_passthrough_on_cpu():
    inner = torch.nn.Identity()
    g = hs.GraphedModule(inner)
    x = torch.randn(3)
    assert g(x) is x


def test_tile_table_layout():
    L, K, M = 3, 5, 37
    w = torch.arange(L * K * M, dtype=torch.float32).reshape(L, K, M)
    t = hs.ops.tile_table(w)
    assert t.shape == (L, 2, K, 32) and t.is_contiguous()
    for l in range(L):
        for k in range(K):
            for m in range(M):
                assert t[l, m // 32, k, m % 32] == w[l, k, m]
    assert torch.all(t[:, 1, :, M - 32:] == 0)


def test_group_table_layout():
    L, K, M = 6, 5, 37
    w0, w1 = torch.randn(L, K, M), torch.randn(L, K, M)
    g = hs.ops.group_table((w0, w1), _lib.DIR_FORWARD)
    gc = hs.ops.group_table((w0, w1), _lib.DIR_FORWARD, conj=True)
    assert g.shape == (2, 2, K, 32, 4, 2)
    gi = hs.ops.group_table(w0, _lib.DIR_INVERSE)
    assert gi.shape == (2, 2, L, 32, 4, 1)
    go = hs.ops.group_table(w0, _lib.DIR_FORWARD, m_offset=2)
    for l in range(L):
        for k in range(K):
            for m in range(M):
                # vector pairs are stored as (W0 + W1, W0 - W1), the form the kernel
                # contracts; entries above the diagonal (l < m) are zero whatever
                # the input holds there
                t = float(m <= l)
                assert g[l // 4, m // 32, k, m % 32, l % 4, 0] == t * (w0[l, k, m] + w1[l, k, m])
                assert g[l // 4, m // 32, k, m % 32, l % 4, 1] == t * (w0[l, k, m] - w1[l, k, m])
                assert gc[l // 4, m // 32, k, m % 32, l % 4, 0] == t * (w0[l, k, m] - w1[l, k, m])
                assert gi[k // 4, m // 32, l, m % 32, k % 4, 0] == t * w0[l, k, m]
                # an order slice starting at global order 2: column m is order m + 2
                assert go[l // 4, m // 32, k, m % 32, l % 4, 0] == float(m + 2 <= l) * w0[l, k, m]
    assert torch.all(g[1, :, :, :, 2:, :] == 0)  # rows beyond lmax are zero


def test_group_table8_layout():
    L, K, M = 11, 5, 37
    w0, w1 = torch.randn(L, K, M), torch.randn(L, K, M)
    g = hs.ops.group_table8((w0, w1), _lib.DIR_FORWARD)
    assert g.shape == (2, 2, K, 4, 32, 4)
    gi = hs.ops.group_table8(w0, _lib.DIR_INVERSE)
    assert gi.shape == (1, 2, L, 2, 32, 4)
    for l in range(L):
        for k in range(K):
            for m in range(M):
                t = float(m <= l)
                r = l % 8
                # vector: quad r // 2 holds (row 2q: W0+W1, W0-W1, row 2q+1: W0+W1, W0-W1)
                q, e = r // 2, 2 * (r % 2)
                assert g[l // 8, m // 32, k, q, m % 32, e] == t * (w0[l, k, m] + w1[l, k, m])
                assert g[l // 8, m // 32, k, q, m % 32, e + 1] == t * (w0[l, k, m] - w1[l, k, m])
                # scalar inverse: rows are k, quad k // 4 of the group holds rows 4q .. 4q+3
                rk = k % 8
                assert gi[k // 8, m // 32, l, rk // 4, m % 32, rk % 4] == t * w0[l, k, m]
    # rows 11 .. 15 of the last group are zero: row 11 in quad 1, rows 12 .. 15 in quads 2, 3
    assert torch.all(g[1, :, :, 1, :, 2:] == 0) and torch.all(g[1, :, :, 2:, :, :] == 0)


def test_group_table8_conjugate_and_scalar_forward():
    L, K, M = 9, 3, 33
    w0, w1 = torch.randn(L, K, M), torch.randn(L, K, M)
    gc = hs.ops.group_table8((w0, w1), _lib.DIR_INVERSE, conj=True)  # rows are k
    assert gc.shape == (1, 2, L, 4, 32, 4)
    gs = hs.ops.group_table8(w0, _lib.DIR_FORWARD)
    assert gs.shape == (2, 2, K, 2, 32, 4)
    for l in range(L):
        for k in range(K):
            for m in range(M):
                t = float(m <= l)
                q, e = k // 2, 2 * (k % 2)
                assert gc[0, m // 32, l, q, m % 32, e] == t * (w0[l, k, m] - w1[l, k, m])
                assert gc[0, m // 32, l, q, m % 32, e + 1] == t * (w0[l, k, m] + w1[l, k, m])
                r = l % 8
                assert gs[l // 8, m // 32, k, r // 4, m % 32, r % 4] == t * w0[l, k, m]


def _snake_loads(steps, ks, G, chunk):
    loads = [0] * G
    for i, s in enumerate(steps):
        rnd, pos = divmod(i, G)
        c = G - 1 - pos if rnd & 1 else pos
        per = (s + ks - 1) // ks
        loads[c] += (per + chunk - 1) // chunk + 2
    return loads


def test_stream_launch_plan_metric_shapes():
    """The streaming kernel's launch plan (host-only, planned for 148 SMs)."""
    plan = hs.ops.stream_launch_plan
    V, S_, F, I = _lib.KIND_VECTOR, _lib.KIND_SCALAR, _lib.DIR_FORWARD, _lib.DIR_INVERSE
    # 512x1024 b4: forward 72 tiles of 64 rows x 32 orders, split in clusters of 2 (144 CTAs)
    assert plan(V, F, batch=4, nlat=512, lmax=512, mmax=513, sm_count=148) == {"ks": 2, "clusters": 72, "items": 72}
    assert plan(S_, F, batch=4, nlat=512, lmax=512, mmax=513, sm_count=148) == {"ks": 2, "clusters": 72, "items": 72}
    # inverse: 8 row tiles x 16 order tiles with reductions 512 - 32 j, 74 clusters of 2 in snake order
    assert plan(V, I, batch=4, nlat=512, lmax=512, mmax=513, sm_count=148) == {"ks": 2, "clusters": 74, "items": 128}
    # 256x512 (C1/C2): 20 tiles, split 4
    assert plan(V, F, batch=4, nlat=256, lmax=256, mmax=257, sm_count=148) == {"ks": 4, "clusters": 20, "items": 20}
    # batch groups multiply the items; an explicit split is kept
    assert plan(S_, F, batch=64, nlat=512, lmax=512, mmax=513, sm_count=148)["items"] == 72 * 8
    assert plan(V, F, batch=4, nlat=512, lmax=512, mmax=513, ksplit=4, sm_count=148)["ks"] == 4


def test_stream_snake_assignment_balances_the_inverse():
    # item reductions of the 512x1024 inverse, longest first (8 row tiles per order tile)
    steps = [512 - 32 * j for j in range(16) for _ in range(8)]
    loads = _snake_loads(steps, 2, 74, 4)
    mean = sum(loads) / len(loads)
    assert max(loads) <= 1.1 * mean
    # one item per cluster instead leaves the longest tile alone: almost 2x the mean
    assert max(_snake_loads(steps, 1, 128, 4)) >= 1.8 * (sum(_snake_loads(steps, 1, 128, 4)) / 128)


def test_stream_launch_plan_rejects_bad_arguments():
    with pytest.raises(RuntimeError, match="SCALAR and VECTOR"):
        hs.ops.stream_launch_plan(_lib.KIND_REAL, _lib.DIR_FORWARD, batch=1, nlat=8, lmax=8, mmax=8, sm_count=148)
    with pytest.raises(RuntimeError, match="ksplit"):
        hs.ops.stream_launch_plan(_lib.KIND_VECTOR, _lib.DIR_FORWARD, batch=1, nlat=8, lmax=8, mmax=8, ksplit=3,
                                  sm_count=148)


@pytest.mark.parametrize("nlat,grid,norm,cs", [(24, "equiangular", "ortho", True),
                                               (33, "legendre-gauss", "schmidt", False),
                                               (40, "lobatto", "four-pi", True)])
def test_vector_recurrence_tables_reproduce_the_vector_tables(nlat, grid, norm, cs):
    """The vector recurrence kernel's inputs, evaluated with its own scheme
    (two recurrences re-seeded every 16 degrees, ladder combination per degree)
    in float64, give RealVectorSHT's tables."""
    from holysht_b200 import weights as W

    nlon = 2 * nlat
    seeds, coef, x = W.vector_recurrence_tables(nlat, nlon, grid=grid, norm=norm, csphase=cs)
    ref, L, M = W.vector_forward(nlat, nlon, grid=grid, norm=norm, csphase=cs)
    got = np.zeros_like(ref)
    x64 = x.astype(np.float64)
    for m in range(min(M, L)):
        for l in range(m, L):
            d = l - m
            if d % W.SEGMENT == 0:
                qm0, qm1, qp0, qp1 = (seeds[m, d // W.SEGMENT, :, i].astype(np.float64) for i in range(4))
            am, bm, ap, bp, al, be, ga, de = coef[m, l].astype(np.float64)
            got[0, m, l] = al * qm0 + be * qp0
            got[1, m, l] = ga * qm1 + de * qp1
            qm0, qm1 = qm1, am * x64 * qm1 - bm * qm0
            qp0, qp1 = qp1, ap * x64 * qp1 - bp * qp0
    assert np.abs(got - ref).max() <= 1e-6 * np.abs(ref).max()


def test_reference_backend_flags_map_onto_the_paths(monkeypatch):
    """HOLYSHT_FORCE_BACKEND of the reference picks the tensor-core path (tc_*) or the
    streaming kernel (fma/tma); its autotune flags are ignored with a warning."""
    import holysht_b200 as hs_mod

    m = hs.RealSHT(16, 32)
    monkeypatch.delenv("HOLYSHT_DENSE_TC", raising=False)
    monkeypatch.setenv("HOLYSHT_FORCE_BACKEND", "tc_tf32")
    assert hs_mod._dense_tc_eligible(m, 1, _lib.DIR_FORWARD)
    monkeypatch.setenv("HOLYSHT_FORCE_BACKEND", "tma")
    assert not hs_mod._dense_tc_eligible(m, 4096, _lib.DIR_FORWARD)
    monkeypatch.setenv("HOLYSHT_FORCE_BACKEND", "auto")
    assert hs_mod._dense_tc_eligible(m, 4096, _lib.DIR_FORWARD)
    monkeypatch.setenv("HOLYSHT_AUTOTUNE", "1")
    hs_mod._REF_FLAGS_WARNED.discard("HOLYSHT_AUTOTUNE")
    with pytest.warns(UserWarning, match="HOLYSHT_AUTOTUNE"):
        hs_mod._dense_tc_eligible(m, 1, _lib.DIR_FORWARD)


def test_compact_recurrence_seeds_order_and_symmetry():
    """The compact checkpoint layout keeps each order's existing segments, orders
    in turn, latitude-major; the grids this package builds pass the equatorial
    symmetry check and a perturbed one does not."""
    nlat, nlon, L = 21, 40, 19
    seeds, coef, ct = weights.scalar_recurrence_tables(nlat, nlon, lmax=L, mmax=15)
    comp = weights.compact_recurrence_seeds(seeds, L)
    per = [(L - m + 15) // 16 for m in range(15)]
    assert comp.shape == (nlat, sum(per), 2)
    i = 0
    for m, n in enumerate(per):
        for c in range(n):
            np.testing.assert_array_equal(comp[:, i], seeds[m, c])
            i += 1
    assert weights.recurrence_seeds_symmetric(seeds, ct)
    bad = seeds.copy()
    bad[3, 0, 2, 0] += 1e-3 * np.abs(seeds).max()
    assert not weights.recurrence_seeds_symmetric(bad, ct)
    vs, _, vct = weights.vector_recurrence_tables(nlat, nlon, grid="legendre-gauss")
    assert weights.recurrence_seeds_symmetric(vs, vct)


def test_recurrence_flags_are_checked_without_gpu():
    lib = _lib.load()
    st = lib.holysht_legendre_forward_recurrence_ex(None, None, 0, 0, None, None, None, 1, 4, 4, 4,
                                                    ctypes.c_float(1.0), 1 << 10, None)
    assert st == _lib.HOLYSHT_ERR_INVALID and b"flag" in lib.holysht_last_error()
    st = lib.holysht_legendre_vector_forward_recurrence_ex(None, None, 0, 0, 0, None, None, None, 1, 4, 4, 4,
                                                           ctypes.c_float(1.0), _lib.FLAG_SEEDS_COMPACT, None)
    assert st == _lib.HOLYSHT_ERR_INVALID and b"null" in lib.holysht_last_error()


def test_rfft_entries_check_arguments_without_gpu():
    lib = _lib.load()
    v = ctypes.c_int64(0)
    assert lib.holysht_rfft_workspace(0, 64, ctypes.byref(v)) == _lib.HOLYSHT_ERR_INVALID
    assert lib.holysht_rfft_workspace(4, 64, None) == _lib.HOLYSHT_ERR_INVALID
    d = _lib.ContractDesc()
    assert lib.holysht_rfft_contract(None, 4, 64, None, None, 0, ctypes.byref(d), None) == _lib.HOLYSHT_ERR_INVALID
    assert b"null" in lib.holysht_last_error()


def _fold_scalar(spec, seeds, coef, x, L, M, par):
    """The scalar segment kernels' algebra in float64 loops: per order and
    16-degree segment, the recurrence from the checkpoints over (northern, with
    ``par``) latitudes, contracted with X_k +/- X_{K-1-k} by the parity of the
    degree's offset in the segment."""
    B, K, _ = spec.shape
    out = np.zeros((B, L, M), complex)
    for m in range(min(M, L)):
        for c in range((L - m + 15) // 16):
            lseg = m + 16 * c
            for k in range((K + 1) // 2 if par else K):
                km = K - 1 - k
                xm = spec[:, km, m] if (par and km != k) else 0
                e, o = spec[:, k, m] + xm, (spec[:, k, m] - xm) if par else spec[:, k, m]
                p2, p1 = seeds[m, c, k]
                for q in range(16):
                    l = lseg + q
                    if q == 0:
                        pl = p2
                    elif q == 1:
                        pl = p1
                    else:
                        a, b = coef[m, l] if l < L else (0.0, 0.0)
                        pl = a * x[k] * p1 - b * p2
                        p2, p1 = p1, pl
                    if l < L:
                        out[:, l, m] += pl * (o if q & 1 else e)
    return out


def _fold_vector(spec, seeds, coef, x, L, M, par):
    """The vector segment kernels' algebra: both recurrences, the ladder
    combinations, S = sum (W0+W1) u and D = sum (W0-W1) v with the mirror terms
    -s (W0-W1) u' and -s (W0+W1) v' under ``par``, sph = (S+D)/2, tor = i(S-D)/2."""
    B, _, K, _ = spec.shape
    out = np.zeros((B, 2, L, M), complex)
    for m in range(min(M, L)):
        for c in range((L - m + 15) // 16):
            lseg = m + 16 * c
            S = np.zeros((16, B), complex)
            D = np.zeros((16, B), complex)
            for k in range((K + 1) // 2 if par else K):
                km = K - 1 - k
                u, v = spec[:, 0, k, m] + 1j * spec[:, 1, k, m], spec[:, 0, k, m] - 1j * spec[:, 1, k, m]
                mir = par and km != k
                um = spec[:, 0, km, m] + 1j * spec[:, 1, km, m] if mir else 0
                vm = spec[:, 0, km, m] - 1j * spec[:, 1, km, m] if mir else 0
                qm0, qm1, qp0, qp1 = seeds[m, c, k]
                for q in range(16):
                    l = lseg + q
                    cf = coef[m, l] if l < L else np.zeros(8)
                    w0 = cf[4] * qm0 + cf[5] * qp0
                    w1 = cf[6] * qm1 + cf[7] * qp1
                    s = 1 if q & 1 else -1  # -(-1)^(l+m), l - m = 16c + q
                    S[q] += (w0 + w1) * u + (s * (w0 - w1) * um if par else 0)
                    D[q] += (w0 - w1) * v + (s * (w0 + w1) * vm if par else 0)
                    qm0, qm1 = qm1, cf[0] * x[k] * qm1 - cf[1] * qm0
                    qp0, qp1 = qp1, cf[2] * x[k] * qp1 - cf[3] * qp0
            for q in range(16):
                if lseg + q < L:
                    out[:, 0, lseg + q, m] = 0.5 * (S[q] + D[q])
                    out[:, 1, lseg + q, m] = 0.5j * (S[q] - D[q])
    return out


@pytest.mark.parametrize("nlat,nlon,grid", [(12, 24, "equiangular"), (11, 22, "legendre-gauss")])
def test_recurrence_fold_algebra_matches_oracle(nlat, nlon, grid):
    """The segment kernels' algebra (checkpoints, recurrences, equatorial fold,
    vector ladder and u/v form), run in float64 on the package's checkpoint
    tables, reproduces the oracle's contraction with and without the fold, for
    even and odd nlat (the tables are float32, hence 1e-6)."""
    rng = np.random.default_rng(nlat)
    seeds, coef, x = (a.astype(np.float64) for a in weights.scalar_recurrence_tables(nlat, nlon, grid=grid))
    M, L = coef.shape[0], coef.shape[1]
    spec = rng.standard_normal((2, nlat, M)) + 1j * rng.standard_normal((2, nlat, M))
    ref = orc.legendre_forward(spec, orc.scalar_forward_table(nlat, nlon, grid=grid).transpose(1, 2, 0))
    for par in (False, True):
        got = _fold_scalar(spec, seeds, coef, x, L, M, par)
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6
    seeds, coef, x = (a.astype(np.float64) for a in weights.vector_recurrence_tables(nlat, nlon, grid=grid))
    spec = rng.standard_normal((2, 2, nlat, M)) + 1j * rng.standard_normal((2, 2, nlat, M))
    w = orc.vector_forward_tables(nlat, nlon, grid=grid)
    ref = orc.vector_legendre_forward(spec, w[0].transpose(1, 2, 0), w[1].transpose(1, 2, 0))
    for par in (False, True):
        got = _fold_vector(spec, seeds, coef, x, L, M, par)
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6


@pytest.mark.parametrize("grid,norm,cs", [("equiangular", "ortho", True), ("legendre-gauss", "schmidt", False),
                                          ("equiangular", "four-pi", True)])
def test_inverse_recurrence_tables_reproduce_the_inverse_table(grid, norm, cs):
    """The inverse kernel's inputs (8-degree checkpoints in the inverse
    normalisation, no quadrature weight, and the recurrence coefficients),
    advanced in float64 by P_l = a_l x P_{l-1} - b_l P_{l-2} from each
    checkpoint, reproduce InverseRealSHT's pct table; the synthesis from them
    matches the oracle's inverse contraction."""
    nlat, nlon = 13, 26
    seeds, coef, x = (a.astype(np.float64) for a in
                      weights.scalar_recurrence_tables(nlat, nlon, grid=grid, norm=norm, csphase=cs,
                                                       inverse=True, segment=8))
    pct = orc.scalar_inverse_table(nlat, nlon, grid=grid, norm=norm, csphase=cs)
    M, L = coef.shape[0], coef.shape[1]
    assert seeds.shape == (M, (L + 7) // 8, nlat, 2)
    got = np.zeros_like(pct)
    for m in range(M):
        for c in range((L - m + 7) // 8):
            l0 = m + 8 * c
            p0, p1 = seeds[m, c, :, 0], seeds[m, c, :, 1]
            got[m, l0] = p0
            if l0 + 1 < L:
                got[m, l0 + 1] = p1
            for l in range(l0 + 2, min(l0 + 8, L)):
                p0, p1 = p1, coef[m, l, 0] * x * p1 - coef[m, l, 1] * p0
                got[m, l] = p1
    scale = np.abs(pct).max()
    np.testing.assert_allclose(got, pct, rtol=0, atol=1e-6 * scale)
    rng = np.random.default_rng(3)
    spec = rng.standard_normal((2, L, M)) + 1j * rng.standard_normal((2, L, M))
    ref = orc.legendre_inverse(spec, pct.transpose(1, 2, 0))
    syn = orc.legendre_inverse(spec, got.transpose(1, 2, 0))
    assert np.linalg.norm(syn - ref) / np.linalg.norm(ref) < 1e-6


def test_inverse_recurrence_arguments_are_checked_without_gpu():
    """The inverse recurrence entry rejects bad flags, extents, strides and
    misaligned pointers before touching the device (the addresses below are
    never dereferenced)."""
    lib = _lib.load()
    f = lib.holysht_legendre_inverse_recurrence
    B, K, L, M = 2, 8, 8, 8
    good, odd = 0x10000, 0x10004
    one = ctypes.c_float(1.0)

    def call(out=good, spec=good, seeds=good, flags=0, obs=K * M, ors=M, cols=M, sbs=L * M, srs=M, nlon=16):
        return f(out, obs, ors, cols, spec, sbs, srs, seeds, good, good, B, K, L, M, one, flags, nlon, None)

    assert call(flags=1 << 12) == _lib.HOLYSHT_ERR_INVALID and b"flag" in lib.holysht_last_error()
    assert call(cols=M - 1) == _lib.HOLYSHT_ERR_INVALID and b"out_cols" in lib.holysht_last_error()
    assert call(srs=M - 1) == _lib.HOLYSHT_ERR_INVALID and b"strides" in lib.holysht_last_error()
    assert call(flags=_lib.FLAG_IRFFT_PREP, nlon=8) == _lib.HOLYSHT_ERR_INVALID
    assert b"irfft" in lib.holysht_last_error()
    assert call(seeds=odd) == _lib.HOLYSHT_ERR_INVALID and b"seeds" in lib.holysht_last_error()
    assert call(spec=odd) == _lib.HOLYSHT_ERR_INVALID and b"aligned" in lib.holysht_last_error()
    assert call(out=odd) == _lib.HOLYSHT_ERR_INVALID and b"aligned" in lib.holysht_last_error()
    assert call(out=None) == _lib.HOLYSHT_ERR_INVALID and b"null" in lib.holysht_last_error()


def test_forward_recurrence_entries_reject_misaligned_spectra_without_gpu():
    """Both forward recurrence entries refuse a spectrum or output that is not
    8-byte aligned (the addresses are never dereferenced)."""
    lib = _lib.load()
    good, odd = 0x10000, 0x10004
    one = ctypes.c_float(1.0)
    for spec, out in ((odd, good), (good, odd)):
        st = lib.holysht_legendre_forward_recurrence_ex(out, spec, 64, 8, good, good, good, 1, 8, 8, 8, one, 0,
                                                        None)
        assert st == _lib.HOLYSHT_ERR_INVALID and b"aligned" in lib.holysht_last_error()
        st = lib.holysht_legendre_vector_forward_recurrence_ex(out, spec, 128, 64, 8, good, good, good, 1, 8, 8, 8,
                                                               one, 0, None)
        assert st == _lib.HOLYSHT_ERR_INVALID and b"aligned" in lib.holysht_last_error()
