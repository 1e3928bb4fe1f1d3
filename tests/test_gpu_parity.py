"""GPU parity of the sm_100a kernels against the float64 oracle and the
reference's own CPU outputs (golden fixtures).  Every call goes through the
C ABI of libholysht_b200.so.

Tolerances (FP32 paths): relative L2 <= 1e-6 and max-abs <= 1e-5 * max|ref|
against the float64 oracle on the same float32 tables; against the golden
fixtures (themselves FP32 results of the reference's CPU path) 1e-5.
BF16-input paths: 1e-6 against FP32-on-the-bf16-rounded-spectrum (the
contraction itself is exact FP32), and 1e-2 against unrounded FP32.
"""
import numpy as np
import pytest
import torch

import holysht_b200 as hs
from holysht_b200 import _lib, ops
from oracle import sht_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = ["eq12x24", "lg10x20_l8_m7", "eq9x17_odd", "lob8x16"]
FP32_REL = 1e-6
FP32_MAXABS = 1e-5
GOLD_REL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.complex128)
    b = np.asarray(b, np.complex128)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a))


def assert_fp32_close(got, ref, rel=FP32_REL, maxabs=FP32_MAXABS):
    got = got.detach().cpu().numpy() if torch.is_tensor(got) else got
    r = rel_l2(got, ref)
    scale = np.max(np.abs(ref)) if np.size(ref) else 0.0
    err = np.max(np.abs(np.asarray(got, np.complex128) - ref)) if np.size(ref) else 0.0
    assert r <= rel, f"relative L2 {r:.3e} > {rel:.1e}"
    assert err <= maxabs * max(scale, 1e-30), f"max-abs {err:.3e} > {maxabs:.1e} * {scale:.3e}"


def tri_table(rng, L, K, M):
    w = rng.standard_normal((L, K, M)).astype(np.float32)
    w *= (np.arange(M)[None, None, :] <= np.arange(L)[:, None, None])
    return w


def cplx(rng, shape):
    return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)


SHAPES = [  # (B, K, L, M)
    (1, 1, 1, 1),
    (3, 7, 5, 5),
    (2, 16, 16, 17),
    (5, 33, 40, 37),
    (9, 64, 48, 65),
    (4, 70, 96, 33),
    (17, 20, 12, 70),
]


# ------------------------------------------------------------- operator level

@pytest.mark.parametrize("B,K,L,M", SHAPES)
def test_op_scalar_forward_inverse(B, K, L, M):
    rng = np.random.default_rng(B * 1000 + K)
    w = tri_table(rng, L, K, M)
    x = cplx(rng, (B, K, M))
    c = cplx(rng, (B, L, M))
    wt = torch.from_numpy(w).to(DEV)
    out = torch.full((B, L, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    ops.fused_legendre_forward(out, torch.from_numpy(x).to(DEV), wt)
    ref = orc.legendre_forward(x.astype(np.complex128), w.astype(np.float64))
    assert_fp32_close(out, ref)
    # exact zeros above the diagonal
    upper = np.arange(M)[None, :] > np.arange(L)[:, None]
    assert np.all(out.cpu().numpy()[:, upper] == 0)
    inv = torch.full((B, K, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    ops.fused_legendre_inverse(inv, torch.from_numpy(c).to(DEV), wt)
    assert_fp32_close(inv, orc.legendre_inverse(c.astype(np.complex128), w.astype(np.float64)))


@pytest.mark.parametrize("B,K,L,M", SHAPES)
def test_op_vector_forward_inverse(B, K, L, M):
    rng = np.random.default_rng(B * 7 + M)
    w0, w1 = tri_table(rng, L, K, M), tri_table(rng, L, K, M)
    x = cplx(rng, (B, 2, K, M))
    c = cplx(rng, (B, 2, L, M))
    t0, t1 = torch.from_numpy(w0).to(DEV), torch.from_numpy(w1).to(DEV)
    out = torch.full((B, 2, L, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    ops.fused_vector_legendre_forward(out, torch.from_numpy(x).to(DEV), t0, t1)
    W0, W1 = w0.astype(np.float64), w1.astype(np.float64)
    assert_fp32_close(out, orc.vector_legendre_forward(x.astype(np.complex128), W0, W1))
    inv = torch.full((B, 2, K, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    ops.fused_vector_legendre_inverse(inv, torch.from_numpy(c).to(DEV), t0, t1)
    assert_fp32_close(inv, orc.vector_legendre_inverse(c.astype(np.complex128), W0, W1))


@pytest.mark.parametrize("B,K,L,M", SHAPES)
def test_op_real_forward_inverse(B, K, L, M):
    rng = np.random.default_rng(B + 3 * K)
    w = tri_table(rng, L, K, M)
    x = rng.standard_normal((B, K, M)).astype(np.float32)
    c = rng.standard_normal((B, L, M)).astype(np.float32)
    wt = torch.from_numpy(w).to(DEV)
    out = torch.full((B, L, M), np.nan, dtype=torch.float32, device=DEV)
    ops.fused_legendre_forward_real(out, torch.from_numpy(x).to(DEV), wt)
    assert_fp32_close(out, orc.legendre_forward(x.astype(np.float64), w.astype(np.float64)))
    xb = torch.from_numpy(x).to(DEV).bfloat16()
    outb = torch.empty((B, L, M), dtype=torch.float32, device=DEV)
    ops.fused_legendre_forward_real_ex(outb, xb, wt, 4)
    xr = xb.float().cpu().numpy().astype(np.float64)
    assert_fp32_close(outb, orc.legendre_forward(xr, w.astype(np.float64)))
    inv = torch.full((B, K, M), np.nan, dtype=torch.float32, device=DEV)
    ops.fused_legendre_inverse_real(inv, torch.from_numpy(c).to(DEV), wt)
    assert_fp32_close(inv, orc.legendre_inverse(c.astype(np.float64), w.astype(np.float64)))


@pytest.mark.parametrize("ks", [1, 2, 4, 8])
def test_cluster_split_is_exact_across_sizes(ks):
    rng = np.random.default_rng(ks)
    B, K, L, M = 4, 200, 100, 101
    w0, w1 = tri_table(rng, L, K, M), tri_table(rng, L, K, M)
    x = cplx(rng, (B, 2, K, M))
    t0, t1 = torch.from_numpy(w0).to(DEV), torch.from_numpy(w1).to(DEV)
    xin = torch.from_numpy(x).to(DEV)
    out = torch.empty((B, 2, L, M), dtype=torch.complex64, device=DEV)
    ops.legendre_contract(kind=_lib.KIND_VECTOR, direction=_lib.DIR_FORWARD, input=xin, output=out,
                          w0=t0, w1=t1, batch=B, nlat=K, lmax=L, mmax=M,
                          in_strides=(2 * K * M, K * M, M), out_strides=(2 * L * M, L * M, M),
                          out_cols=M, ksplit=ks)
    ref = orc.vector_legendre_forward(x.astype(np.complex128), w0.astype(np.float64), w1.astype(np.float64))
    assert_fp32_close(out, ref)
    # deterministic: a second launch is bit-identical
    out2 = torch.empty_like(out)
    ops.legendre_contract(kind=_lib.KIND_VECTOR, direction=_lib.DIR_FORWARD, input=xin, output=out2,
                          w0=t0, w1=t1, batch=B, nlat=K, lmax=L, mmax=M,
                          in_strides=(2 * K * M, K * M, M), out_strides=(2 * L * M, L * M, M),
                          out_cols=M, ksplit=ks)
    assert torch.equal(out, out2)


def test_conjugate_vector_map_is_the_adjoint():
    rng = np.random.default_rng(11)
    B, K, L, M = 2, 24, 20, 21
    w0, w1 = tri_table(rng, L, K, M), tri_table(rng, L, K, M)
    g = cplx(rng, (B, 2, L, M))
    t0, t1 = torch.from_numpy(w0).to(DEV), torch.from_numpy(w1).to(DEV)
    out = torch.empty((B, 2, K, M), dtype=torch.complex64, device=DEV)
    ops.legendre_contract(kind=_lib.KIND_VECTOR, direction=_lib.DIR_INVERSE, input=torch.from_numpy(g).to(DEV),
                          output=out, w0=t0, w1=t1, batch=B, nlat=K, lmax=L, mmax=M,
                          in_strides=(2 * L * M, L * M, M), out_strides=(2 * K * M, K * M, M),
                          out_cols=M, flags=_lib.FLAG_CONJ_W1)
    ref = orc.vector_legendre_inverse(g.astype(np.complex128), w0.astype(np.float64), w1.astype(np.float64), conj_w1=True)
    assert_fp32_close(out, ref)


def test_pack_recompose_known_answers():
    B, K, M = 2, 3, 4
    xr = torch.arange(B * 2 * K * M * 2, dtype=torch.float32).reshape(B, 2, K, M, 2)
    x = torch.view_as_complex(xr.contiguous()).to(DEV)
    s0, s1 = hs._stack_vector_forward_real_inputs(x)
    f = lambda c, r: xr[:, c, :, :, r].reshape(-1, K, M)
    torch.testing.assert_close(s0.cpu(), torch.cat([f(0, 0), f(0, 1), f(1, 0), f(1, 1)]), rtol=0, atol=0)
    torch.testing.assert_close(s1.cpu(), torch.cat([f(1, 1), f(1, 0), f(0, 1), f(0, 0)]), rtol=0, atol=0)
    L = 3
    o0 = torch.arange(4 * B * L * M, dtype=torch.float32).reshape(4 * B, L, M)
    o1 = 1000 + torch.arange(4 * B * L * M, dtype=torch.float32).reshape(4 * B, L, M)
    out = hs._recompose_vector_forward_real_outputs(o0.to(DEV), o1.to(DEV), batch_size=B, lmax=L, mmax=M)
    r00, r01, r10, r11 = o0.split(B)
    s11, s10, s01, s00 = o1.split(B)
    exp = torch.empty(B, 2, L, M, 2)
    exp[:, 0, ..., 0], exp[:, 0, ..., 1] = r00 - s11, r01 + s10
    exp[:, 1, ..., 0], exp[:, 1, ..., 1] = -s01 - r10, s00 - r11
    torch.testing.assert_close(out.cpu(), torch.view_as_complex(exp), rtol=0, atol=0)


def test_prepare_irfft_matches_reference(golden_dir):
    g = np.load(golden_dir / "ops_tri.npz")
    c = torch.from_numpy(g["c"]).to(DEV)
    for nlon, key in ((20, "prep_even"), (19, "prep_odd")):
        got = hs._prepare_irfft_input(c, nlon, c.size(-1))
        np.testing.assert_array_equal(got.cpu().numpy(), g[key])


def test_op_kats_match_reference(golden_dir):
    g = np.load(golden_dir / "ops_tri.npz")
    wt = torch.from_numpy(g["weight_t"]).to(DEV)
    weights = wt.permute(2, 0, 1).contiguous()
    x = torch.from_numpy(g["x"]).to(DEV)
    c = torch.from_numpy(g["c"]).to(DEV)
    assert rel_l2(hs.fused_legendre_forward(x, weights).cpu(), g["fwd"]) < GOLD_REL
    assert rel_l2(hs.fused_legendre_inverse(c, weights).cpu(), g["inv"]) < GOLD_REL
    assert rel_l2(hs.fused_legendre_forward_real(x.real.contiguous(), wt).cpu(), g["fwd_real"]) < GOLD_REL
    assert rel_l2(hs.fused_legendre_inverse_real(c.real.contiguous(), wt).cpu(), g["inv_real"]) < GOLD_REL


def test_op_argument_errors():
    w = torch.zeros(4, 5, 6, device=DEV)
    x = torch.zeros(2, 5, 6, dtype=torch.complex64, device=DEV)
    with pytest.raises(RuntimeError, match="output must be"):
        ops.fused_legendre_forward(torch.empty(2, 4, 7, dtype=torch.complex64, device=DEV), x, w)
    with pytest.raises(RuntimeError, match="nlat"):
        ops.fused_legendre_forward(torch.empty(2, 4, 6, dtype=torch.complex64, device=DEV),
                                   torch.zeros(2, 3, 6, dtype=torch.complex64, device=DEV), w)
    with pytest.raises(RuntimeError, match="contiguous"):
        ops.fused_legendre_forward(torch.empty(2, 4, 6, dtype=torch.complex64, device=DEV),
                                   torch.zeros(2, 6, 5, dtype=torch.complex64, device=DEV).transpose(1, 2), w)
    with pytest.raises(RuntimeError, match="float32"):
        ops.fused_legendre_forward(torch.empty(2, 4, 6, dtype=torch.complex64, device=DEV), x, w.double())


# ------------------------------------------------------------- module level

@pytest.mark.parametrize("name", GOLDEN)
def test_modules_match_reference_golden(golden_dir, name):
    g = np.load(golden_dir / f"{name}.npz")
    nlat, nlon = int(g["nlat"]), int(g["nlon"])
    kw = dict(lmax=int(g["lmax"]), mmax=int(g["mmax"]), grid=str(g["grid"]))
    sht = hs.RealSHT(nlat, nlon, **kw).to(DEV)
    vsht = hs.RealVectorSHT(nlat, nlon, **kw).to(DEV)
    isht = hs.InverseRealSHT(nlat, nlon, **kw).to(DEV)
    ivsht = hs.InverseRealVectorSHT(nlat, nlon, **kw).to(DEV)

    x = torch.from_numpy(g["x"]).to(DEV).requires_grad_(True)
    coef = sht(x)
    (coef.real.square().sum() + coef.imag.square().sum()).backward()
    assert rel_l2(coef.detach().cpu(), g["sht"]) < GOLD_REL
    assert rel_l2(x.grad.cpu(), g["grad_sht"]) < GOLD_REL

    xv = torch.from_numpy(g["xv"]).to(DEV).requires_grad_(True)
    vc = vsht(xv)
    (vc.real.square().sum() + vc.imag.square().sum()).backward()
    assert rel_l2(vc.detach().cpu(), g["vsht"]) < GOLD_REL
    assert rel_l2(xv.grad.cpu(), g["grad_vsht"]) < GOLD_REL

    c = torch.from_numpy(g["c"]).to(DEV).requires_grad_(True)
    y = isht(c)
    torch.tanh(y).sum().backward()
    assert rel_l2(y.detach().cpu(), g["isht"]) < GOLD_REL
    assert rel_l2(c.grad.cpu(), g["grad_isht"]) < GOLD_REL

    cv = torch.from_numpy(g["cv"]).to(DEV).requires_grad_(True)
    yv = ivsht(cv)
    torch.tanh(yv).sum().backward()
    assert rel_l2(yv.detach().cpu(), g["ivsht"]) < GOLD_REL
    assert rel_l2(cv.grad.cpu(), g["grad_ivsht"]) < GOLD_REL


def _module_oracle_scalar(m, x):
    w = m.weight_t.permute(2, 0, 1).double().cpu().numpy()
    return orc.sht_forward(x, w)


def _module_oracle_vector(m, x):
    w = np.stack([m.w0_t.permute(2, 0, 1).double().cpu().numpy(), m.w1_t.permute(2, 0, 1).double().cpu().numpy()])
    return orc.vector_sht_forward(x, w)


@pytest.mark.parametrize("grid", ["equiangular", "legendre-gauss"])
def test_scalar_module_c1_shape(grid):
    # C1 shape: (4, 256, 512), lmax 256, mmax 257, seed 0
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 256, 512)).astype(np.float32)
    m = hs.RealSHT(256, 512, grid=grid).to(DEV)
    out = m(torch.from_numpy(x).to(DEV))
    assert out.shape == (4, 256, 257) and out.dtype == torch.complex64
    assert_fp32_close(out, _module_oracle_scalar(m, x.astype(np.float64)))
    upper = np.arange(257)[None, :] > np.arange(256)[:, None]
    assert np.all(out.cpu().numpy()[:, upper] == 0)


def test_vector_module_c2_shape_band_limited():
    # C2: band-limited field synthesised from N(0,1)*(l+1)^-1.5 coefficients, seed 1
    nlat, nlon = 256, 512
    rng = np.random.default_rng(1)
    L, M = 256, 257
    scale = (np.arange(L, dtype=np.float64) + 1.0) ** -1.5
    tri = np.arange(M)[None, :] <= np.arange(L)[:, None]
    c = (rng.standard_normal((4, 2, L, M)) + 1j * rng.standard_normal((4, 2, L, M))) * scale[:, None] * tri
    isv = hs.InverseRealVectorSHT(nlat, nlon).to(DEV)
    x = isv(torch.from_numpy(c.astype(np.complex64)).to(DEV))
    m = hs.RealVectorSHT(nlat, nlon).to(DEV)
    out = m(x)
    assert out.shape == (4, 2, L, M)
    assert_fp32_close(out, _module_oracle_vector(m, x.cpu().numpy().astype(np.float64)))


def test_metric_shapes_match_oracle():
    # the benchmark configuration: 512 x 1024, batch 4, lmax 512, mmax 513
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 512, 1024)).astype(np.float32)
    m = hs.RealSHT(512, 1024).to(DEV)
    assert_fp32_close(m(torch.from_numpy(x).to(DEV)), _module_oracle_scalar(m, x.astype(np.float64)))
    del m
    rng = np.random.default_rng(1)
    xv = rng.standard_normal((4, 2, 512, 1024)).astype(np.float32)
    v = hs.RealVectorSHT(512, 1024).to(DEV)
    assert_fp32_close(v(torch.from_numpy(xv).to(DEV)), _module_oracle_vector(v, xv.astype(np.float64)))


def test_bf16_module_paths():
    rng = np.random.default_rng(2)
    x = torch.from_numpy(rng.standard_normal((2, 3, 64, 128)).astype(np.float32)).bfloat16().float().to(DEV)
    m32 = hs.RealSHT(64, 128, grid="legendre-gauss").to(DEV)
    m16 = hs.RealSHT(64, 128, grid="legendre-gauss", dtype="bf16").to(DEV)
    m16.weight_t.copy_(m32.weight_t)
    o32, o16 = m32(x), m16(x)
    assert rel_l2(o16.cpu(), o32.cpu()) < 1e-2
    # the bf16 path is FP32 on the bf16-rounded spectrum
    # the reference rounds the 2*pi-scaled spectrum (torch-ext/holysht/__init__.py:1291-1295)
    spec = 2 * torch.pi * torch.fft.rfft(x, dim=-1, norm="forward")
    spec = torch.complex(spec.real.bfloat16().float(), spec.imag.bfloat16().float())
    w = m32.weight_t.permute(2, 0, 1).double().cpu().numpy()
    ref = np.einsum("...km,mlk->...lm", spec.cpu().numpy()[..., : m32.mmax].astype(np.complex128), w)
    assert_fp32_close(o16, ref)


def test_noncontiguous_and_leading_dims():
    rng = np.random.default_rng(5)
    base = torch.from_numpy(rng.standard_normal((3, 32, 2, 64)).astype(np.float32)).to(DEV)
    x = base.permute(0, 2, 1, 3)  # (3, 2, 32, 64) non-contiguous
    v = hs.RealVectorSHT(32, 64).to(DEV)
    out = v(x)
    assert_fp32_close(out, _module_oracle_vector(v, x.cpu().numpy().astype(np.float64)))
    m = hs.RealSHT(32, 64).to(DEV)
    out = m(x)  # (3, 2) leading dims
    assert out.shape == (3, 2, 32, 33)
    assert_fp32_close(out, _module_oracle_scalar(m, x.cpu().numpy().astype(np.float64)))


def test_roundtrip_gauss_metric_size():
    # size-independent property at the benchmark size: analysis o synthesis = identity
    # on band-limited coefficients (Gauss quadrature is exact here)
    nlat, nlon = 512, 1024
    rng = np.random.default_rng(3)
    isht = hs.InverseRealSHT(nlat, nlon, grid="legendre-gauss").to(DEV)
    sht = hs.RealSHT(nlat, nlon, grid="legendre-gauss").to(DEV)
    L, M = sht.lmax, sht.mmax
    tri = np.arange(M)[None, :] <= np.arange(L)[:, None]
    c = (rng.standard_normal((2, L, M)) + 1j * rng.standard_normal((2, L, M))) * tri
    c[..., 0] = c[..., 0].real
    c[..., M - 1] = 0
    ct = torch.from_numpy(c.astype(np.complex64)).to(DEV)
    back = sht(isht(ct))
    assert rel_l2(back.cpu().numpy(), c) < 2e-5


def test_training_roundtrip_gradients_match_float64_autograd():
    # C4-style: inverse -> tanh -> forward -> sum|coef|^2, gradients vs float64 torch autograd
    nlat, nlon, B = 24, 48, 3
    rng = np.random.default_rng(3)
    isht = hs.InverseRealSHT(nlat, nlon).to(DEV)
    sht = hs.RealSHT(nlat, nlon).to(DEV)
    L, M = sht.lmax, sht.mmax
    tri = np.arange(M)[None, :] <= np.arange(L)[:, None]
    scale = (np.arange(L) + 1.0)[:, None] ** -2
    c = ((rng.standard_normal((B, L, M)) + 1j * rng.standard_normal((B, L, M))) * scale * tri).astype(np.complex64)
    ct = torch.from_numpy(c).to(DEV).requires_grad_(True)
    coef = sht(torch.tanh(isht(ct)))
    (coef.real.square().sum() + coef.imag.square().sum()).backward()

    P = isht.pct.double().cpu().to(torch.complex128)
    W = sht.weight_t.permute(2, 0, 1).double().cpu().to(torch.complex128)
    c64 = torch.from_numpy(c.astype(np.complex128)).requires_grad_(True)
    y = torch.einsum("blm,mlk->bkm", c64, P)
    full = torch.zeros(B, nlat, nlon // 2 + 1, dtype=torch.complex128)
    full[..., :M] = y
    full[..., 0] = full[..., 0].real.to(full.dtype)
    full[..., nlon // 2] = full[..., nlon // 2].real.to(full.dtype)
    xs = torch.fft.irfft(full, n=nlon, dim=-1, norm="forward")
    X = 2 * torch.pi * torch.fft.rfft(torch.tanh(xs), dim=-1, norm="forward")[..., :M]
    ref_coef = torch.einsum("bkm,mlk->blm", X, W)
    (ref_coef.real.square().sum() + ref_coef.imag.square().sum()).backward()
    assert_fp32_close(coef.detach(), ref_coef.detach().numpy(), rel=2e-6, maxabs=2e-5)
    assert_fp32_close(ct.grad, c64.grad.numpy(), rel=2e-5, maxabs=1e-4)


def test_graphed_module_matches_eager():
    m = hs.RealVectorSHT(64, 128).to(DEV)
    g = hs.GraphedModule(m)
    x = torch.randn(2, 2, 64, 128, device=DEV)
    ref = m(x)
    torch.testing.assert_close(g(x), ref, rtol=0, atol=0)
    x2 = torch.randn_like(x)
    torch.testing.assert_close(g(x2), m(x2), rtol=0, atol=0)


# ------------------------------------------------------------- tensor-core dense path

TC_SHAPES = [  # (B, K, L, M, W)
    (4, 32, 128, 129, 129),
    (128, 64, 200, 201, 260),
    (100, 36, 130, 65, 65),
    (200, 512, 300, 301, 301),
]


@pytest.mark.parametrize("B,K,L,M,W", TC_SHAPES)
def test_dense_tensor_core_forward_matches_oracle(B, K, L, M, W):
    rng = np.random.default_rng(B + K)
    w = tri_table(rng, L, K, M)
    spec = cplx(rng, (B, K, W))
    tab = torch.from_numpy(np.ascontiguousarray(w.transpose(2, 0, 1))).to(DEV)  # [M, L, K]
    out = torch.full((B, L, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    ops.legendre_dense_tc(_lib.DIR_FORWARD, out, torch.from_numpy(spec).to(DEV), tab, nlat=K, lmax=L, mmax=M,
                          scale=1.5)
    ref = 1.5 * orc.legendre_forward(spec[..., :M].astype(np.complex128), w.astype(np.float64))
    assert_fp32_close(out, ref)
    upper = np.arange(M)[None, :] > np.arange(L)[:, None]
    assert np.all(out.cpu().numpy()[:, upper] == 0)
    assert ops.tc_error_word() == 0


@pytest.mark.parametrize("B,K,L,M,nlon", [(4, 30, 128, 129, 256), (130, 64, 200, 101, 220), (200, 300, 512, 257, 512)])
def test_dense_tensor_core_inverse_matches_oracle(B, K, L, M, nlon):
    rng = np.random.default_rng(B + L)
    w = tri_table(rng, L, K, M)
    c = cplx(rng, (B, L, M)) * (np.arange(M)[None, None, :] <= np.arange(L)[None, :, None])
    W = nlon // 2 + 1
    tab = torch.from_numpy(np.ascontiguousarray(w.transpose(2, 1, 0))).to(DEV)  # [M, K, L]
    out = torch.full((B, K, W), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    ops.legendre_dense_tc(_lib.DIR_INVERSE, out, torch.from_numpy(c.astype(np.complex64)).to(DEV), tab, nlat=K,
                          lmax=L, mmax=M, flags=_lib.FLAG_IRFFT_PREP, nlon=nlon)
    y = orc.legendre_inverse(c.astype(np.complex128), w.astype(np.float64))
    ref = orc.prepare_irfft(y, nlon)
    assert_fp32_close(out, ref)
    assert ops.tc_error_word() == 0


def test_scalar_modules_use_tensor_cores_for_large_batches(monkeypatch):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((2, 80, 64, 128)).astype(np.float32)  # 160 slices >= 128
    m = hs.RealSHT(64, 128).to(DEV)
    xt = torch.from_numpy(x).to(DEV)
    got = m(xt)
    assert_fp32_close(got, _module_oracle_scalar(m, x.astype(np.float64)))
    # inverse + training round trip on tensor cores vs the SIMT kernels
    inv = hs.InverseRealSHT(64, 128).to(DEV)

    def roundtrip():
        c = got.detach().clone().requires_grad_(True)
        coef = m(torch.tanh(inv(c)))
        (coef.real.square().sum() + coef.imag.square().sum()).backward()
        return coef.detach(), c.grad

    coef_tc, grad_tc = roundtrip()
    monkeypatch.setenv("HOLYSHT_DENSE_TC", "0")
    simt = m(xt)
    coef_simt, grad_simt = roundtrip()
    assert_fp32_close(got, simt.cpu().numpy().astype(np.complex128), rel=1e-6, maxabs=1e-5)
    assert_fp32_close(coef_tc, coef_simt.cpu().numpy().astype(np.complex128), rel=2e-6, maxabs=2e-5)
    assert_fp32_close(grad_tc, grad_simt.cpu().numpy().astype(np.complex128), rel=2e-6, maxabs=2e-5)


# ------------------------------------------------------------- recurrence variant

@pytest.mark.parametrize("nlat,nlon,grid,norm,cs", [
    (512, 1024, "equiangular", "ortho", True),
    (96, 192, "legendre-gauss", "schmidt", False),
    (33, 64, "lobatto", "four-pi", True),
    (256, 512, "equiangular", "ortho", True),
])
def test_recurrence_variant_matches_oracle(nlat, nlon, grid, norm, cs):
    rng = np.random.default_rng(nlat)
    x = rng.standard_normal((5, nlat, nlon)).astype(np.float32)  # 5 batches: two batch groups
    m = hs.RealSHT(nlat, nlon, grid=grid, norm=norm, csphase=cs, variant="recurrence").to(DEV)
    out = m(torch.from_numpy(x).to(DEV))
    assert_fp32_close(out, _module_oracle_scalar(m, x.astype(np.float64)))
    upper = np.arange(m.mmax)[None, :] > np.arange(m.lmax)[:, None]
    assert np.all(out.cpu().numpy()[:, upper] == 0)


@pytest.mark.parametrize("nlat,nlon,grid,norm,cs", [
    (512, 1024, "equiangular", "ortho", True),
    (96, 192, "legendre-gauss", "schmidt", False),
    (33, 64, "lobatto", "four-pi", True),
    (130, 256, "equiangular", "ortho", True),
])
def test_vector_recurrence_variant_matches_oracle(nlat, nlon, grid, norm, cs):
    rng = np.random.default_rng(nlat + 1)
    x = rng.standard_normal((5, 2, nlat, nlon)).astype(np.float32)  # 5 batches: two batch groups
    m = hs.RealVectorSHT(nlat, nlon, grid=grid, norm=norm, csphase=cs, variant="recurrence").to(DEV)
    out = m(torch.from_numpy(x).to(DEV))
    assert_fp32_close(out, _module_oracle_vector(m, x.astype(np.float64)))
    upper = np.arange(m.mmax)[None, :] > np.arange(m.lmax)[:, None]
    assert np.all(out.cpu().numpy()[:, :, upper] == 0)
    # the table variant of the same transform
    t = hs.RealVectorSHT(nlat, nlon, grid=grid, norm=norm, csphase=cs).to(DEV)
    ref = t(torch.from_numpy(x).to(DEV)).cpu().numpy().astype(np.complex128)
    got = out.cpu().numpy().astype(np.complex128)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-6


@pytest.mark.parametrize("vector", [False, True])
@pytest.mark.parametrize("nlat,nlon,grid", [(47, 96, "equiangular"), (64, 128, "legendre-gauss")])
def test_recurrence_ops_every_fold_and_block_shape(vector, nlat, nlon, grid, monkeypatch):
    """The recurrence ops with and without the equatorial fold, for every
    degree-block and latitude-chunk shape of the segment kernels, odd and even
    nlat, 6 batches (a partial batch group), against the float64 oracle."""
    rng = np.random.default_rng(nlat + 7 * vector)
    B = 6
    if vector:
        seeds, coef, ct = hs.weights.vector_recurrence_tables(nlat, nlon, grid=grid)
        mod = hs.RealVectorSHT(nlat, nlon, grid=grid)
    else:
        seeds, coef, ct = hs.weights.scalar_recurrence_tables(nlat, nlon, grid=grid)
        mod = hs.RealSHT(nlat, nlon, grid=grid)
    assert hs.weights.recurrence_seeds_symmetric(seeds, ct)
    M, _, K, _ = seeds.shape
    L = coef.shape[1]
    shape = (B, 2, K, M + 3) if vector else (B, K, M + 3)  # row stride wider than mmax
    spec = (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)
    if vector:
        w0 = mod.w0_t.cpu().numpy().astype(np.float64)
        w1 = mod.w1_t.cpu().numpy().astype(np.float64)
        ref = orc.vector_legendre_forward(spec[..., :M].astype(np.complex128), w0, w1)
    else:
        ref = orc.legendre_forward(spec[..., :M].astype(np.complex128),
                                      mod.weight_t.cpu().numpy().astype(np.float64))
    layouts = [torch.from_numpy(seeds).to(DEV),
               torch.from_numpy(hs.weights.compact_recurrence_seeds(seeds, L)).to(DEV)]
    cf, x = (torch.from_numpy(a).to(DEV) for a in (coef, ct))
    sp = torch.from_numpy(spec).to(DEV)
    shapes = [("8", "4"), ("16", "2"), ("16", "8"), ("8", "8")]
    for db, nkc in shapes:
        monkeypatch.setenv("HSB_REC_DB", db)
        monkeypatch.setenv("HSB_REC_NKC", nkc)
        for parity in (False, True):
            for sd in layouts:
                out = torch.full((B, 2, L, M) if vector else (B, L, M), float("nan"), dtype=torch.complex64,
                                 device=DEV)
                if vector:
                    ops.legendre_vector_forward_recurrence(out, sp, sd, cf, x, 1.0, parity=parity)
                else:
                    ops.legendre_forward_recurrence(out, sp, sd, cf, x, 1.0, parity=parity)
                assert_fp32_close(out, ref)


@pytest.mark.parametrize("vector", [False, True])
def test_cached_forward_runs_rfft_and_contraction_in_one_call(vector):
    """From the second call on, a no-grad FP32 forward runs cuFFT's R2C and the
    Legendre kernel in one library call (holysht_rfft_contract); it gives the
    first call's result (torch's rfft + the contraction) and the oracle's, and a
    non-contiguous input of the same shape takes torch's rfft instead."""
    rng = np.random.default_rng(11 + vector)
    nlat, nlon = 96, 192
    shape = (3, 2, nlat, nlon) if vector else (3, nlat, nlon)
    x = rng.standard_normal(shape).astype(np.float32)
    m = (hs.RealVectorSHT if vector else hs.RealSHT)(nlat, nlon).to(DEV)
    xt = torch.from_numpy(x).to(DEV)
    with torch.no_grad():
        first = m(xt)
        fast = next(iter(m.__dict__["_fast_forward"].values()))
        assert fast.fft_work is not None, "the library could not open cuFFT"
        second = m(xt)
        wide = torch.zeros(shape[:-1] + (2 * nlon,), device=DEV)
        wide[..., :nlon] = xt
        third = m(wide[..., :nlon])  # same shape, rows not contiguous
    assert not wide[..., :nlon].is_contiguous()
    assert rel_l2(second.cpu().numpy(), first.cpu().numpy()) <= 1e-7
    assert rel_l2(third.cpu().numpy(), first.cpu().numpy()) <= 1e-7
    ref = (_module_oracle_vector if vector else _module_oracle_scalar)(m, x.astype(np.float64))
    assert_fp32_close(second, ref)


@pytest.mark.parametrize("nlat,nlon,grid,norm,cs,lmax,mmax", [
    (512, 1024, "equiangular", "ortho", True, None, None),
    (96, 192, "legendre-gauss", "schmidt", False, None, None),
    (33, 64, "lobatto", "four-pi", True, None, None),
    (47, 96, "equiangular", "ortho", True, 40, 30),
])
def test_inverse_recurrence_variant_matches_oracle(nlat, nlon, grid, norm, cs, lmax, mmax):
    """InverseRealSHT(variant="recurrence"): the synthesis from functions
    generated in registers (one thread per order and latitude) against the
    float64 oracle and the table variant, 5 batches (two batch groups), odd
    nlat and truncated lmax / mmax (zero columns up to nlon/2+1); the op with
    and without the equatorial fold; gradients through the table backward."""
    rng = np.random.default_rng(nlat + 3)
    m = hs.InverseRealSHT(nlat, nlon, lmax=lmax, mmax=mmax, grid=grid, norm=norm, csphase=cs,
                          variant="recurrence").to(DEV)
    t = hs.InverseRealSHT(nlat, nlon, lmax=lmax, mmax=mmax, grid=grid, norm=norm, csphase=cs).to(DEV)
    L, M = m.lmax, m.mmax
    c = (rng.standard_normal((5, L, M)) + 1j * rng.standard_normal((5, L, M))).astype(np.complex64)
    c *= (np.arange(M)[None, :] <= np.arange(L)[:, None])
    ct = torch.from_numpy(c).to(DEV)
    got = m(ct)
    ref = orc.sht_inverse(c.astype(np.complex128), m.pct.double().cpu().numpy(), nlon)
    assert_fp32_close(got, ref)
    assert rel_l2(got.detach().cpu().numpy(), t(ct).detach().cpu().numpy()) <= 1e-6
    seeds, coef, cth = m.recurrence_tables()
    W = nlon // 2 + 1
    ref_spec = np.einsum("blm,mlk->bkm", c.astype(np.complex128), m.pct.double().cpu().numpy())
    for parity in (False, True):
        spec = torch.full((5, nlat, W), float("nan"), dtype=torch.complex64, device=DEV)
        ops.legendre_inverse_recurrence(spec, ct, seeds, coef, cth, 1.0, parity=parity)
        s = spec.cpu().numpy()
        assert np.all(s[..., M:] == 0)
        assert_fp32_close(s[..., :M], ref_spec)
    cg = ct.clone().requires_grad_(True)
    cg2 = ct.clone().requires_grad_(True)
    (m(cg) ** 2).sum().backward()
    (t(cg2) ** 2).sum().backward()
    assert rel_l2(cg.grad.cpu().numpy(), cg2.grad.cpu().numpy()) <= 1e-6
