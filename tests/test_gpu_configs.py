"""GPU parity at the full sizes of the benchmark configurations.

C3  RealSHT(dtype="bf16") 512x1024 Legendre-Gauss, x (4, 16, 512, 1024), seed 2
C4  training round trip 512x1024: InverseRealSHT -> tanh -> RealSHT -> sum|coef|^2
    -> backward on spectral (8, 32, 512, 513), seed 3; and the vector pair on (8, 2, 512, 513)
C5  RealSHT 1024x2048 on (16, 64, 1024, 2048) (the tcgen05 dense path, K = L = 1024)
    and RealVectorSHT 1024x2048 on (16, 2, 1024, 2048), seed 4

The GPU runs the whole workload; the float64 check runs on a sample that is
exact for its part of the output: chosen orders m (every order is an
independent contraction) and chosen slices (every slice is an independent
transform, and the loss of the round trip is a sum over slices, so the
gradient of one slice depends on that slice only).  The check uses the
modules' own float32 tables in float64 (numpy / torch autograd on the CPU).

Tolerances: FP32 outputs relative L2 <= 1e-6 and max-abs <= 1e-5 * max|ref|
BF16 inputs: <= 1e-6 against FP32 on the
bf16-rounded spectrum, <= 1e-2 against FP32 on the unrounded input.  The C4
round trip chains four contractions and two FFTs in FP32, so its coefficients
and gradients are held to 2e-6 / 2e-5 relative L2 (measured errors are
printed in the assertion messages).
"""
import numpy as np
import pytest
import torch

import holysht_b200 as hs

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rel(a, b):
    a = np.asarray(a, np.complex128)
    b = np.asarray(b, np.complex128)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _check(got, ref, rel, maxabs, what):
    r = _rel(got, ref)
    err = float(np.max(np.abs(np.asarray(got, np.complex128) - ref)))
    scale = float(np.max(np.abs(ref)))
    assert r <= rel, f"{what}: relative L2 {r:.3e} > {rel:.1e}"
    assert err <= maxabs * scale, f"{what}: max-abs {err:.3e} > {maxabs:.1e} * {scale:.3e}"


def _spectrum64(x, M):
    """2*pi * rfft(x, norm="forward")[..., :M] in float64 (the reference's spectrum)."""
    return 2.0 * np.pi * np.fft.rfft(np.asarray(x, np.float64), axis=-1, norm="forward")[..., :M]


def _orders(M):
    cand = [0, 1, 2, 31, 32, 33, M // 4, M // 2 - 1, M // 2, M - 33, M - 2, M - 1]
    return sorted({m for m in cand if 0 <= m < M})


def _scalar_ref(X, W, ms):
    """X [s, K, M] spectrum, W [M, L, K] table -> [s, L, len(ms)]."""
    return np.stack([X[:, :, m] @ W[m].astype(np.float64).T for m in ms], axis=-1)


def _vector_ref(X, W0, W1, ms):
    """X [s, 2, K, M] -> [s, 2, L, len(ms)] (sph = W0 c0 + i W1 c1, tor = i W1 c0 - W0 c1)."""
    out = []
    for m in ms:
        w0 = W0[m].astype(np.float64).T
        w1 = W1[m].astype(np.float64).T
        c0, c1 = X[:, 0, :, m], X[:, 1, :, m]
        out.append(np.stack([c0 @ w0 + 1j * (c1 @ w1), 1j * (c0 @ w1) - c1 @ w0], axis=1))
    return np.stack(out, axis=-1)


# ----------------------------------------------------------------------- C3

def test_c3_bf16_legendre_gauss_full_size():
    nlat, nlon = 512, 1024
    rng = np.random.default_rng(2)
    x16 = torch.from_numpy(rng.standard_normal((4, 16, nlat, nlon)).astype(np.float32)).bfloat16()
    x = x16.float().to(DEV)
    m16 = hs.RealSHT(nlat, nlon, grid="legendre-gauss", dtype="bf16").to(DEV)
    m32 = hs.RealSHT(nlat, nlon, grid="legendre-gauss").to(DEV)
    with torch.no_grad():
        o16 = m16(x)
        o32 = m32(x)
    assert o16.shape == (4, 16, 512, 513)
    # against unrounded FP32 (the same module maths without the bf16 spectrum rounding)
    r = (torch.linalg.vector_norm(o16 - o32) / torch.linalg.vector_norm(o32)).item()
    assert r <= 1e-2, f"bf16 vs fp32 relative L2 {r:.3e}"
    # FP32 on the bf16-rounded spectrum: the reference rounds 2*pi*rfft(x, norm="forward")
    # (torch-ext/holysht/__init__.py:1291-1295), then contracts in FP32
    M = m32.mmax
    slices = [0, 17, 63]
    # the same cuFFT call as the module (one plan over all 64 slices): a spectrum
    # value one ulp away can round to the neighbouring bf16 value
    spec = (2 * torch.pi * torch.fft.rfft(x, dim=-1, norm="forward")).reshape(64, nlat, -1)[slices, :, :M]
    spec = torch.complex(spec.real.bfloat16().float(), spec.imag.bfloat16().float()).cpu().numpy()
    W = m32.weights.cpu().numpy()
    ms = _orders(M)
    ref = _scalar_ref(spec.astype(np.complex128), W, ms)
    got = o16.reshape(64, 512, M)[slices][..., ms].cpu().numpy()
    _check(got, ref, 1e-6, 1e-5, "C3 bf16 module vs FP32 on the rounded spectrum")


# ----------------------------------------------------------------------- C4

def _c4_coefficients(shape, L, M, seed):
    rng = np.random.default_rng(seed)
    scale = (np.arange(L, dtype=np.float64) + 1.0)[:, None] ** -2
    tri = np.arange(M)[None, :] <= np.arange(L)[:, None]
    c = (rng.standard_normal(shape, dtype=np.float32) + 1j * rng.standard_normal(shape, dtype=np.float32))
    return (c * (scale * tri)).astype(np.complex64)


def _irfft64(y, nlon):
    K, M = y.shape[-2], y.shape[-1]
    full = torch.zeros(y.shape[:-1] + (nlon // 2 + 1,), dtype=torch.complex128)
    full[..., :M] = y
    full[..., 0] = full[..., 0].real.to(full.dtype)
    if nlon % 2 == 0:
        full[..., nlon // 2] = full[..., nlon // 2].real.to(full.dtype)
    return torch.fft.irfft(full, n=nlon, dim=-1, norm="forward")


def test_c4_scalar_training_round_trip_full_size():
    nlat, nlon, L, M = 512, 1024, 512, 513
    c = _c4_coefficients((8, 32, L, M), L, M, 3)
    inv = hs.InverseRealSHT(nlat, nlon).to(DEV)
    fwd = hs.RealSHT(nlat, nlon).to(DEV)
    ct = torch.from_numpy(c).to(DEV).requires_grad_(True)
    coef = fwd(torch.tanh(inv(ct)))
    (coef.real.square().sum() + coef.imag.square().sum()).backward()
    torch.cuda.synchronize()

    flat = [0, 137, 255]
    P = inv.pct.double().cpu().to(torch.complex128)      # [M, L, K]
    W = fwd.weights.double().cpu().to(torch.complex128)  # [M, L, K]
    c64 = torch.from_numpy(c.reshape(256, L, M)[flat].astype(np.complex128)).requires_grad_(True)
    y = torch.einsum("blm,mlk->bkm", c64, P)
    X = 2 * torch.pi * torch.fft.rfft(torch.tanh(_irfft64(y, nlon)), dim=-1, norm="forward")[..., :M]
    ref = torch.einsum("bkm,mlk->blm", X, W)
    (ref.real.square().sum() + ref.imag.square().sum()).backward()
    got = coef.detach().reshape(256, L, M)[flat].cpu().numpy()
    grad = ct.grad.reshape(256, L, M)[flat].cpu().numpy()
    _check(got, ref.detach().numpy(), 2e-6, 2e-5, "C4 scalar coefficients")
    _check(grad, c64.grad.numpy(), 2e-5, 1e-4, "C4 scalar gradient")


def test_c4_vector_training_round_trip_full_size():
    nlat, nlon, L, M = 512, 1024, 512, 513
    c = _c4_coefficients((8, 2, L, M), L, M, 3)
    inv = hs.InverseRealVectorSHT(nlat, nlon).to(DEV)
    fwd = hs.RealVectorSHT(nlat, nlon).to(DEV)
    ct = torch.from_numpy(c).to(DEV).requires_grad_(True)
    coef = fwd(torch.tanh(inv(ct)))
    (coef.real.square().sum() + coef.imag.square().sum()).backward()
    torch.cuda.synchronize()

    sel = [0, 5]
    D0 = inv.d0.double().cpu().to(torch.complex128)
    D1 = inv.d1.double().cpu().to(torch.complex128)
    W0 = fwd.w0.double().cpu().to(torch.complex128)
    W1 = fwd.w1.double().cpu().to(torch.complex128)
    c64 = torch.from_numpy(c[sel].astype(np.complex128)).requires_grad_(True)
    fi = lambda a, d: torch.einsum("blm,mlk->bkm", a, d)  # noqa: E731
    ff = lambda a, w: torch.einsum("bkm,mlk->blm", a, w)  # noqa: E731
    sph, tor = c64[:, 0], c64[:, 1]
    y = torch.stack([fi(sph, D0) + 1j * fi(tor, D1), 1j * fi(sph, D1) - fi(tor, D0)], dim=1)
    X = 2 * torch.pi * torch.fft.rfft(torch.tanh(_irfft64(y, nlon)), dim=-1, norm="forward")[..., :M]
    ref = torch.stack([ff(X[:, 0], W0) + 1j * ff(X[:, 1], W1), 1j * ff(X[:, 0], W1) - ff(X[:, 1], W0)], dim=1)
    (ref.real.square().sum() + ref.imag.square().sum()).backward()
    got = coef.detach()[sel].cpu().numpy()
    grad = ct.grad[sel].cpu().numpy()
    _check(got, ref.detach().numpy(), 2e-6, 2e-5, "C4 vector coefficients")
    _check(grad, c64.grad.numpy(), 2e-5, 1e-4, "C4 vector gradient")


# ----------------------------------------------------------------------- C5

def test_c5_scalar_tensor_core_full_size():
    nlat, nlon = 1024, 2048
    m = hs.RealSHT(nlat, nlon).to(DEV)
    L, M = m.lmax, m.mmax
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(16, 64, nlat, nlon, device=DEV, generator=g)
    with torch.no_grad():
        out = m(x)  # 1024 slices: the tcgen05 dense path (K = L = 1024)
    torch.cuda.synchronize()
    assert out.shape == (16, 64, L, M)
    slices = [0, 1, 517, 1023]
    xs = x.reshape(1024, nlat, nlon)[slices].cpu().numpy()
    ms = _orders(M) + [511, 1023]
    ms = sorted(set(ms))
    ref = _scalar_ref(_spectrum64(xs, M), m.weights.cpu().numpy(), ms)
    got = out.reshape(1024, L, M)[slices][..., ms].cpu().numpy()
    _check(got, ref, 1e-6, 1e-5, "C5 scalar sampled orders")
    # exact zeros above the diagonal on a full slice
    upper = torch.arange(M, device=DEV)[None, :] > torch.arange(L, device=DEV)[:, None]
    assert out.reshape(1024, L, M)[5][upper].abs().max().item() == 0.0
    del out, x
    torch.cuda.empty_cache()


def test_c5_vector_full_size():
    nlat, nlon = 1024, 2048
    m = hs.RealVectorSHT(nlat, nlon).to(DEV)
    L, M = m.lmax, m.mmax
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(16, 2, nlat, nlon, device=DEV, generator=g)
    with torch.no_grad():
        out = m(x)
    torch.cuda.synchronize()
    assert out.shape == (16, 2, L, M)
    sel = [0, 9, 15]
    xs = x[sel].cpu().numpy()
    ms = sorted(set(_orders(M) + [511, 1023]))
    ref = _vector_ref(_spectrum64(xs, M), m.w0.cpu().numpy(), m.w1.cpu().numpy(), ms)
    got = out[sel][..., ms].cpu().numpy()
    _check(got, ref, 1e-6, 1e-5, "C5 vector sampled orders")
    upper = torch.arange(M, device=DEV)[None, :] > torch.arange(L, device=DEV)[:, None]
    assert out[3][:, upper].abs().max().item() == 0.0
    del out, x
    torch.cuda.empty_cache()


@pytest.mark.parametrize("builder", ["scalar_forward", "scalar_inverse", "vector_forward", "vector_inverse"])
def test_tables_built_on_the_gpu_match_the_host(builder):
    """The float64 table recurrence run on the GPU (used to build large sharded
    tables quickly) gives the host's tables."""
    from holysht_b200 import weights as W

    fn = getattr(W, builder)
    for grid in ("equiangular", "legendre-gauss"):
        host, L, M = fn(48, 96, grid=grid, restated=True)
        dev, L2, M2 = fn(48, 96, grid=grid, restated=True, device=DEV)
        assert (L, M) == (L2, M2) and dev.device.type == "cuda"
        d = dev.cpu().numpy()
        assert np.max(np.abs(d - host)) <= 1e-13 * np.max(np.abs(host))
