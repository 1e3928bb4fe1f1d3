"""GPU parity of the streaming kernel (table layout HOLYSHT_TABLE_GROUPED8)
against the float64 oracle, through the C ABI.

Tolerance (FP32): relative L2 <= 1e-6 and max-abs <= 1e-5 * max|ref| on the
same float32 tables; exact zeros above the diagonal and in padding columns;
bit-identical repeat launches; the device error word stays clear.
"""
import math

import numpy as np
import pytest
import torch

from holysht_b200 import _lib, ops
from oracle import sht_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP32_REL = 1e-6
FP32_MAXABS = 1e-5


def assert_fp32_close(got, ref):
    got = got.detach().cpu().numpy().astype(np.complex128)
    ref = np.asarray(ref, np.complex128)
    nr = np.linalg.norm(ref)
    rel = np.linalg.norm(got - ref) / nr if nr > 0 else np.linalg.norm(got)
    assert rel <= FP32_REL, f"relative L2 {rel:.3e}"
    assert np.abs(got - ref).max() <= FP32_MAXABS * max(np.abs(ref).max(), 1e-30)


def tri_table(rng, L, K, M, m_offset=0):
    w = rng.standard_normal((L, K, M)).astype(np.float32)
    w *= (np.arange(M)[None, None, :] + m_offset <= np.arange(L)[:, None, None])
    return w


def cplx(rng, shape):
    return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)


def run(kind, direction, x, out, table, B, K, L, M, W_in, W_out, ks=0, scale=1.0, flags=0, nlon=0, m_offset=0):
    P = 2 if kind == _lib.KIND_VECTOR else 1
    Rin = K if direction == _lib.DIR_FORWARD else L
    Rout = L if direction == _lib.DIR_FORWARD else K
    ops.legendre_contract(kind=kind, direction=direction, input=x, output=out, w0=table, batch=B, nlat=K,
                          lmax=L, mmax=M, in_strides=(P * Rin * W_in, Rin * W_in, W_in),
                          out_strides=(P * Rout * W_out, Rout * W_out, W_out), out_cols=W_out, scale=scale,
                          flags=flags, nlon=nlon, ksplit=ks, grouped8=True, m_offset=m_offset)


SHAPES = [  # (B, K, L, M)
    (1, 1, 1, 1),
    (3, 7, 5, 5),
    (2, 16, 16, 17),
    (5, 33, 40, 37),
    (9, 64, 48, 65),
    (4, 70, 96, 33),
    (17, 20, 12, 70),
    (4, 130, 129, 129),
]


@pytest.mark.parametrize("B,K,L,M", SHAPES)
@pytest.mark.parametrize("ks", [0, 1, 2])
def test_stream_scalar_forward_inverse(B, K, L, M, ks):
    rng = np.random.default_rng(B * 131 + K + ks)
    w = tri_table(rng, L, K, M)
    wt = torch.from_numpy(w).to(DEV)
    W = M + 3  # spectrum rows wider than the table (an rfft with more columns)
    x = cplx(rng, (B, K, W))
    out = torch.full((B, L, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    run(_lib.KIND_SCALAR, _lib.DIR_FORWARD, torch.from_numpy(x).to(DEV), out,
        ops.group_table8(wt, _lib.DIR_FORWARD), B, K, L, M, W, M, ks=ks, scale=0.5)
    ref = 0.5 * orc.legendre_forward(x[..., :M].astype(np.complex128), w.astype(np.float64))
    assert_fp32_close(out, ref)
    upper = np.arange(M)[None, :] > np.arange(L)[:, None]
    assert np.all(out.cpu().numpy()[:, upper] == 0)

    c = cplx(rng, (B, L, M))
    inv = torch.full((B, K, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    run(_lib.KIND_SCALAR, _lib.DIR_INVERSE, torch.from_numpy(c).to(DEV), inv,
        ops.group_table8(wt, _lib.DIR_INVERSE), B, K, L, M, M, M, ks=ks)
    assert_fp32_close(inv, orc.legendre_inverse(c.astype(np.complex128), w.astype(np.float64)))
    assert ops.stream_error_word() == 0


@pytest.mark.parametrize("B,K,L,M", SHAPES)
@pytest.mark.parametrize("ks", [0, 2, 4])
def test_stream_vector_forward_inverse(B, K, L, M, ks):
    rng = np.random.default_rng(B * 17 + M + ks)
    w0, w1 = tri_table(rng, L, K, M), tri_table(rng, L, K, M)
    t0, t1 = torch.from_numpy(w0).to(DEV), torch.from_numpy(w1).to(DEV)
    W0, W1 = w0.astype(np.float64), w1.astype(np.float64)
    x = cplx(rng, (B, 2, K, M))
    out = torch.full((B, 2, L, M), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    run(_lib.KIND_VECTOR, _lib.DIR_FORWARD, torch.from_numpy(x).to(DEV), out,
        ops.group_table8((t0, t1), _lib.DIR_FORWARD), B, K, L, M, M, M, ks=ks)
    assert_fp32_close(out, orc.vector_legendre_forward(x.astype(np.complex128), W0, W1))

    # inverse with the conjugate map (table built from (W0, -W1)) and irfft preparation
    c = cplx(rng, (B, 2, L, M))
    nlon = 2 * M + 2
    Wout = nlon // 2 + 1
    inv = torch.full((B, 2, K, Wout), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    run(_lib.KIND_VECTOR, _lib.DIR_INVERSE, torch.from_numpy(c).to(DEV), inv,
        ops.group_table8((t0, t1), _lib.DIR_INVERSE, conj=True), B, K, L, M, M, Wout, ks=ks,
        flags=_lib.FLAG_IRFFT_PREP, nlon=nlon)
    ref = np.zeros((B, 2, K, Wout), np.complex128)
    ref[..., :M] = orc.vector_legendre_inverse(c.astype(np.complex128), W0, W1, conj_w1=True)
    ref[..., 0] = ref[..., 0].real
    got = inv.cpu().numpy()
    assert np.all(got[..., M:] == 0) and np.all(got[..., 0].imag == 0)
    assert_fp32_close(inv, ref)
    assert ops.stream_error_word() == 0


def test_stream_order_slice_keeps_the_global_triangle():
    rng = np.random.default_rng(5)
    B, K, L, M, off = 3, 40, 100, 96, 32
    w = tri_table(rng, L, K, M)              # full table
    ws = np.ascontiguousarray(w[:, :, off:off + 48])  # orders 32 .. 79
    x = cplx(rng, (B, K, 48))
    out = torch.full((B, L, 48), complex(np.nan, np.nan), dtype=torch.complex64, device=DEV)
    run(_lib.KIND_SCALAR, _lib.DIR_FORWARD, torch.from_numpy(x).to(DEV), out,
        ops.group_table8(torch.from_numpy(ws).to(DEV), _lib.DIR_FORWARD, m_offset=off), B, K, L, 48, 48, 48,
        m_offset=off)
    assert_fp32_close(out, orc.legendre_forward(x.astype(np.complex128), ws.astype(np.float64)))
    got = out.cpu().numpy()
    upper = (np.arange(48)[None, :] + off) > np.arange(L)[:, None]
    assert np.all(got[:, upper] == 0)


@pytest.mark.parametrize("ks", [1, 2, 4, 8])
def test_stream_split_is_deterministic_and_matches(ks):
    rng = np.random.default_rng(ks + 40)
    B, K, L, M = 4, 256, 160, 161
    w0, w1 = tri_table(rng, L, K, M), tri_table(rng, L, K, M)
    t0, t1 = torch.from_numpy(w0).to(DEV), torch.from_numpy(w1).to(DEV)
    tab = ops.group_table8((t0, t1), _lib.DIR_FORWARD)
    x = torch.from_numpy(cplx(rng, (B, 2, K, M))).to(DEV)
    outs = []
    for _ in range(2):
        o = torch.empty((B, 2, L, M), dtype=torch.complex64, device=DEV)
        run(_lib.KIND_VECTOR, _lib.DIR_FORWARD, x, o, tab, B, K, L, M, M, M, ks=ks)
        outs.append(o)
    assert torch.equal(outs[0], outs[1])
    ref = orc.vector_legendre_forward(x.cpu().numpy().astype(np.complex128), w0.astype(np.float64),
                                      w1.astype(np.float64))
    assert_fp32_close(outs[0], ref)


def test_stream_metric_size_matches_grouped_kernel():
    """512 x 1024 vector forward, batch 4: the streaming kernel against the
    4-row kernel on the same (W0 + W1, W0 - W1) tables (both FP32, different
    summation orders)."""
    import holysht_b200 as hs

    m = hs.RealVectorSHT(512, 1024).to(DEV)
    B = 4
    x = torch.randn((B, 2, 512, 1024), device=DEV, generator=torch.Generator(DEV).manual_seed(3))
    spec = torch.fft.rfft(x, dim=-1)
    L, M, W = m.lmax, m.mmax, spec.size(-1)
    out4 = torch.empty((B, 2, L, M), dtype=torch.complex64, device=DEV)
    ops.legendre_contract(kind=_lib.KIND_VECTOR, direction=_lib.DIR_FORWARD, input=spec, output=out4,
                          w0=m.table(_lib.DIR_FORWARD, "grouped")[0], batch=B, nlat=512, lmax=L, mmax=M,
                          in_strides=(2 * 512 * W, 512 * W, W), out_strides=(2 * L * M, L * M, M), out_cols=M,
                          scale=2 * math.pi / 1024, grouped=True)
    tab8 = ops.group_table8((m.w0_t, m.w1_t), _lib.DIR_FORWARD)
    out8 = torch.empty_like(out4)
    run(_lib.KIND_VECTOR, _lib.DIR_FORWARD, spec, out8, tab8, B, 512, L, M, W, M, scale=2 * math.pi / 1024)
    a = out8.cpu().numpy().astype(np.complex128)
    b = out4.cpu().numpy().astype(np.complex128)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) <= 1e-6
    assert ops.stream_error_word() == 0


def test_stream_rejects_flags_it_does_not_take():
    B, K, L, M = 1, 8, 8, 8
    t = torch.zeros((L, K, M), device=DEV)
    x = torch.zeros((B, 2, K, M), dtype=torch.complex64, device=DEV)
    out = torch.zeros((B, 2, L, M), dtype=torch.complex64, device=DEV)
    with pytest.raises(RuntimeError, match="GROUPED8"):
        run(_lib.KIND_VECTOR, _lib.DIR_FORWARD, x, out, ops.group_table8((t, t), _lib.DIR_FORWARD), B, K, L, M,
            M, M, flags=_lib.FLAG_CONJ_W1)


def test_stream_clusters_with_several_items_match():
    """Persistent clusters: the 512 x 1024 inverse has 128 items for 74 clusters
    (snake order, two items per cluster), and a forced split of 8 leaves 18
    clusters for 72 forward items; both against the 4-row kernel."""
    import holysht_b200 as hs

    B, K, L, M = 4, 512, 512, 513
    g = torch.Generator(DEV).manual_seed(7)
    m = hs.RealVectorSHT(K, 2 * K).to(DEV)
    assert ops.stream_launch_plan(_lib.KIND_VECTOR, _lib.DIR_INVERSE, batch=B, nlat=K, lmax=L, mmax=M)["clusters"] < 128
    c = torch.complex(torch.randn((B, 2, L, M), device=DEV, generator=g), torch.randn((B, 2, L, M), device=DEV, generator=g))
    c = c * (torch.arange(M, device=DEV)[None, :] <= torch.arange(L, device=DEV)[:, None])
    t8 = ops.group_table8((m.w0_t, m.w1_t), _lib.DIR_INVERSE, conj=True)
    t4 = ops.group_table((m.w0_t, m.w1_t), _lib.DIR_INVERSE, conj=True)
    for ks in (0, 8):
        o8 = torch.empty((B, 2, K, M), dtype=torch.complex64, device=DEV)
        o4 = torch.empty_like(o8)
        run(_lib.KIND_VECTOR, _lib.DIR_INVERSE, c, o8, t8, B, K, L, M, M, M, ks=ks)
        ops.legendre_contract(kind=_lib.KIND_VECTOR, direction=_lib.DIR_INVERSE, input=c, output=o4, w0=t4, batch=B,
                              nlat=K, lmax=L, mmax=M, in_strides=(2 * L * M, L * M, M), out_strides=(2 * K * M, K * M, M),
                              out_cols=M, grouped=True)
        a, b = o8.cpu().numpy().astype(np.complex128), o4.cpu().numpy().astype(np.complex128)
        assert np.linalg.norm(a - b) / np.linalg.norm(b) <= 1e-6, ks
    x = torch.randn((B, 2, K, 2 * K), device=DEV, generator=g)
    spec = torch.fft.rfft(x, dim=-1)
    W = spec.size(-1)
    f8 = ops.group_table8((m.w0_t, m.w1_t), _lib.DIR_FORWARD)
    outs = []
    for ks in (0, 8):
        o = torch.empty((B, 2, L, M), dtype=torch.complex64, device=DEV)
        run(_lib.KIND_VECTOR, _lib.DIR_FORWARD, spec, o, f8, B, K, L, M, W, M, ks=ks)
        outs.append(o.cpu().numpy().astype(np.complex128))
    assert np.linalg.norm(outs[0] - outs[1]) / np.linalg.norm(outs[1]) <= 1e-6
    assert ops.stream_error_word() == 0


def test_module_fast_path_matches_the_general_path():
    """Repeated no-grad forwards run a cached launch (rfft + one prepared
    contraction); results equal the general path, per input shape, and the
    cache is dropped when the tables change (state dict) or move (.to())."""
    import holysht_b200 as hs

    g = torch.Generator(DEV).manual_seed(11)
    for cls, shape in ((hs.RealVectorSHT, (3, 2, 32, 64)), (hs.RealSHT, (2, 5, 32, 64))):
        m = cls(32, 64).to(DEV)
        x = torch.randn(shape, device=DEV, generator=g)
        x2 = torch.randn((1,) + shape[1:], device=DEV, generator=g)
        with torch.no_grad():
            first = m(x)
            again = m(x)             # cached launch
            other = m(x2)            # a second shape
        assert "_fast_forward" in m.__dict__ and len(m.__dict__["_fast_forward"]) == 2
        general = m(x.clone().requires_grad_(True)).detach()  # autograd path
        assert torch.equal(first, again) and torch.equal(first, general)
        assert other.shape == (1,) + first.shape[1:]
        # new tables through the state dict: the cached launch must not survive
        sd = {k: v * 2 for k, v in m.state_dict().items()}
        m.load_state_dict(sd)
        with torch.no_grad():
            doubled = m(x)
        assert torch.allclose(doubled, 2 * first, rtol=1e-5, atol=1e-6)
        m.to(DEV)
        assert "_fast_forward" not in m.__dict__
        with torch.no_grad():
            assert torch.allclose(m(x), doubled)


def test_prepared_launch_checks_tensors_and_is_thread_safe():
    """A prepared contraction rejects tensors whose shape or strides differ
    from the ones it was built for, and one module's cached forward driven
    from several threads at once gives each caller its own result."""
    import threading

    import holysht_b200 as hs

    m = hs.RealVectorSHT(32, 64).to(DEV)
    g = torch.Generator(DEV).manual_seed(5)
    xs = [torch.randn((3, 2, 32, 64), device=DEV, generator=g) for _ in range(4)]
    with torch.no_grad():
        expected = [m(x) for x in xs]
    fast = m.__dict__["_fast_forward"][(xs[0].shape, xs[0].dtype, xs[0].device)]
    spec = torch.fft.rfft(xs[0], dim=-1)
    with pytest.raises(RuntimeError, match="do not match"):
        fast.plan.launch(spec[:2], torch.empty((2, 2, m.lmax, m.mmax), dtype=torch.complex64, device=DEV))
    with pytest.raises(RuntimeError, match="do not match"):
        fast.plan.launch(spec, torch.empty((3, 2, m.mmax, m.lmax), dtype=torch.complex64, device=DEV).transpose(-1, -2))

    got = [[] for _ in xs]
    errors = []

    def worker(i):
        try:
            with torch.no_grad():
                for _ in range(25):
                    got[i].append(m(xs[i]))
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(xs))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    for i, outs in enumerate(got):
        assert len(outs) == 25 and all(torch.equal(o, expected[i]) for o in outs)
    assert ops.stream_error_word() == 0


@pytest.mark.parametrize("kind", [_lib.KIND_SCALAR, _lib.KIND_VECTOR])
def test_stream_rounds_the_spectrum_to_bf16(kind):
    """HOLYSHT_FLAG_ROUND_BF16: the staged (already scaled) spectrum is rounded to
    bfloat16 and contracted in FP32: FP32-exact against the float64 oracle on the
    rounded spectrum."""
    rng = np.random.default_rng(21 + kind)
    B, K, L, M = 5, 70, 64, 65
    P = 2 if kind == _lib.KIND_VECTOR else 1
    w0, w1 = tri_table(rng, L, K, M), tri_table(rng, L, K, M)
    x = cplx(rng, (B, P, K, M)) if P == 2 else cplx(rng, (B, K, M))
    xr = torch.from_numpy(x).view(torch.float32).bfloat16().float().view(torch.complex64).numpy()
    if P == 2:
        tab = ops.group_table8((torch.from_numpy(w0).to(DEV), torch.from_numpy(w1).to(DEV)), _lib.DIR_FORWARD)
        ref = orc.vector_legendre_forward(xr.astype(np.complex128), w0.astype(np.float64), w1.astype(np.float64))
        out = torch.empty((B, 2, L, M), dtype=torch.complex64, device=DEV)
    else:
        tab = ops.group_table8(torch.from_numpy(w0).to(DEV), _lib.DIR_FORWARD)
        ref = orc.legendre_forward(xr.astype(np.complex128), w0.astype(np.float64))
        out = torch.empty((B, L, M), dtype=torch.complex64, device=DEV)
    run(kind, _lib.DIR_FORWARD, torch.from_numpy(x).to(DEV), out, tab, B, K, L, M, M, M, flags=_lib.FLAG_ROUND_BF16)
    assert_fp32_close(out, ref)
    assert ops.stream_error_word() == 0


def test_empty_batches_are_no_ops():
    """Zero batches through the reference-named operators, the streaming entry
    and the modules: empty outputs, no error, nothing launched that reads."""
    import holysht_b200 as hs

    K, L, M = 16, 12, 13
    w = torch.zeros((L, K, M), device=DEV)
    ops.fused_legendre_forward(torch.empty((0, L, M), dtype=torch.complex64, device=DEV),
                               torch.empty((0, K, M), dtype=torch.complex64, device=DEV), w)
    ops.fused_vector_legendre_inverse(torch.empty((0, 2, K, M), dtype=torch.complex64, device=DEV),
                                      torch.empty((0, 2, L, M), dtype=torch.complex64, device=DEV), w, w)
    run(_lib.KIND_VECTOR, _lib.DIR_FORWARD, torch.empty((0, 2, K, M), dtype=torch.complex64, device=DEV),
        torch.empty((0, 2, L, M), dtype=torch.complex64, device=DEV), ops.group_table8((w, w), _lib.DIR_FORWARD),
        0, K, L, M, M, M)
    for cls, shape in ((hs.RealSHT, (0, 16, 32)), (hs.RealVectorSHT, (0, 2, 16, 32))):
        m = cls(16, 32).to(DEV)
        with torch.no_grad():
            for _ in range(2):  # the general path, then the cached launch
                out = m(torch.empty(shape, device=DEV))
                assert out.shape == shape[:-2] + (m.lmax, m.mmax) and out.numel() == 0
    inv = hs.InverseRealVectorSHT(16, 32).to(DEV)
    y = inv(torch.empty((0, 2, inv.lmax, inv.mmax), dtype=torch.complex64, device=DEV))
    assert y.shape == (0, 2, 16, 32)
    torch.cuda.synchronize()
    assert ops.stream_error_word() == 0


def test_host_stream_pipeline_matches_module_calls():
    """holysht_b200.pipeline.HostStream: pinned host batches in, pinned host
    results out, copies overlapped with the transforms; every result equals the
    module's own output for that batch."""
    import holysht_b200 as hs
    from holysht_b200.pipeline import HostStream

    dev = torch.device("cuda")
    m = hs.RealVectorSHT(64, 128).to(dev)
    ins = [torch.randn(3, 2, 64, 128).pin_memory() for _ in range(5)]
    outs = [torch.empty(3, 2, 64, 65, dtype=torch.complex64).pin_memory() for _ in range(5)]
    HostStream(m, dev).run(ins, outs)
    for i, o in zip(ins, outs):
        torch.testing.assert_close(o, m(i.to(dev)).cpu(), rtol=0, atol=0)
    with pytest.raises(ValueError, match="pinned"):
        HostStream(m, dev).run([torch.randn(3, 2, 64, 128)], [outs[0]])


@pytest.mark.parametrize("vector", [False, True])
@pytest.mark.parametrize("nlat,nlon,grid", [(33, 64, "equiangular"), (48, 96, "legendre-gauss"),
                                            (31, 64, "lobatto"), (512, 1024, "equiangular")])
def test_parity_folded_forward_matches_oracle(monkeypatch, vector, nlat, nlon, grid):
    """The equatorial-parity layout (northern half of the table, rows k and
    K-1-k read together; odd nlat has an equator row paired with itself)
    against the float64 oracle, for both kinds and every grid family."""
    import holysht_b200 as hs

    monkeypatch.delenv("HOLYSHT_PARITY", raising=False)  # the forward default
    dev = torch.device("cuda")
    rng = np.random.default_rng(nlat + 7 * vector)
    shape = (5, 2, nlat, nlon) if vector else (5, nlat, nlon)
    x = rng.standard_normal(shape).astype(np.float32)
    m = (hs.RealVectorSHT if vector else hs.RealSHT)(nlat, nlon, grid=grid).to(dev)
    assert m.table(_lib.DIR_FORWARD)[2] == "parity"
    with torch.no_grad():
        got = m(torch.from_numpy(x).to(dev)).cpu().numpy()
    if vector:
        w = np.stack([m.w0.double().cpu().numpy(), m.w1.double().cpu().numpy()])
        ref = orc.vector_sht_forward(x.astype(np.float64), w)
    else:
        ref = orc.sht_forward(x.astype(np.float64), m.weights.double().cpu().numpy())
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel <= 1e-6, rel
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
    upper = np.arange(m.mmax)[None, :] > np.arange(m.lmax)[:, None]
    assert np.all(got[..., upper] == 0)


def test_parity_layout_is_skipped_for_asymmetric_tables():
    """Tables without the equatorial symmetry (e.g. loaded from elsewhere)
    fall back to the full layout."""
    import holysht_b200 as hs

    m = hs.RealSHT(16, 32).to("cuda")
    assert m.table(_lib.DIR_FORWARD)[2] == "parity"
    with torch.no_grad():
        m.weight_t[:, 0, :] += 1.0
        m.weights.copy_(m.weight_t.permute(2, 0, 1))
    m._drop_grouped()
    assert m.table(_lib.DIR_FORWARD)[2] == "grouped8"


@pytest.mark.parametrize("nlat,nlon,grid", [(33, 64, "equiangular"), (48, 96, "legendre-gauss"),
                                            (31, 64, "lobatto"), (512, 1024, "equiangular")])
def test_parity_folded_scalar_inverse_matches_oracle(monkeypatch, nlat, nlon, grid):
    """The scalar inverse on the parity fold (northern output rows, their mirrors
    written from the even/odd-degree sums; irfft preparation and zero columns on
    both halves) against the float64 oracle, and the RealSHT gradient that runs
    the same folded inverse."""
    import holysht_b200 as hs

    monkeypatch.setenv("HOLYSHT_PARITY_INV", "1")
    dev = torch.device("cuda")
    rng = np.random.default_rng(nlat + 3)
    inv = hs.InverseRealSHT(nlat, nlon, grid=grid).to(dev)
    assert inv.table(_lib.DIR_INVERSE)[2] == "parity"
    L, M = inv.lmax, inv.mmax
    tri = np.arange(M)[None, :] <= np.arange(L)[:, None]
    c = ((rng.standard_normal((5, L, M)) + 1j * rng.standard_normal((5, L, M))) * tri).astype(np.complex64)
    with torch.no_grad():
        got = inv(torch.from_numpy(c).to(dev)).cpu().numpy()
    ref = orc.sht_inverse(c.astype(np.complex128), inv.pct.double().cpu().numpy(), nlon)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel <= 1e-6, rel
    # gradient of the forward transform through the folded inverse direction
    fwd = hs.RealSHT(nlat, nlon, grid=grid).to(dev)
    x = torch.from_numpy(rng.standard_normal((3, nlat, nlon)).astype(np.float32)).to(dev).requires_grad_(True)
    coef = fwd(x)
    (coef.real.square().sum() + coef.imag.square().sum()).backward()
    xd = x.detach().double().cpu().requires_grad_(True)
    W = fwd.weights.double().cpu().to(torch.complex128)
    X = 2 * torch.pi * torch.fft.rfft(xd, dim=-1, norm="forward")[..., :M]
    r = torch.einsum("bkm,mlk->blm", X, W)
    (r.real.square().sum() + r.imag.square().sum()).backward()
    g, gr = x.grad.cpu().numpy(), xd.grad.numpy()
    assert np.linalg.norm(g - gr) / np.linalg.norm(gr) <= 2e-6
