"""Split-TF32 tensor-core GEMM (tcgen05 + TMEM, TMA-fed) against the oracle.

The f32 bound is the reference's scaled form |x - y| <= 2e-6 * sum|a b|
(small_matmul_tests.rs:153-186); the kernel's representation error per product
stays below ~1.7e-6 |a b| (hi = truncated tf32, lo = x - hi read as tf32).
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def tc_handle(kx, torch_cuda):
    h = kx.handle(0)
    h.set_f32_variant(3)    # KX_F32_3XTF32_1SM: the one-SM kernel at every size
    yield h
    h.set_f32_variant(0)


@pytest.fixture
def pair_handle(kx, torch_cuda):
    h = kx.handle(0)
    h.set_f32_variant(2)    # KX_F32_3XTF32: CTA pairs where the product is large enough
    yield h
    h.set_f32_variant(0)


def _view(kx, torch, arr, dims, strides, origin=0):
    buf = torch.from_numpy(np.ascontiguousarray(arr).reshape(-1)).cuda()
    return kx.TensorView(buf, list(dims), list(strides), origin)


def _check(got, a, b):
    exp, ab = oracle.gemm_dot2(a, b)
    g = got.astype(np.float64)
    assert np.isfinite(g).all()
    ratio = np.abs(g - exp) / np.maximum(ab, 1e-300)
    assert (np.abs(g - exp) <= 2e-6 * ab + 1e-30).all(), float(ratio.max())
    return float(ratio.max())


@pytest.mark.parametrize("m,k,n", [(128, 64, 256), (300, 1000, 260), (1, 64, 256), (520, 48, 1028)])
@pytest.mark.parametrize("b_layout", ["row", "col"])
def test_tc_2d_layouts(kx, torch_cuda, tc_handle, m, k, n, b_layout):
    rng = np.random.default_rng(m * 7 + k)
    pad = 8
    abuf = rng.uniform(-1, 1, (m, k + pad)).astype(np.float32)
    va = oracle.View(abuf, (m, k), (k + pad, 1))
    if b_layout == "row":
        bbuf = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        vb = oracle.View(bbuf, (k, n), (n, 1))
    else:
        bbuf = rng.uniform(-1, 1, (n, k)).astype(np.float32)     # B = bbuf^T, unit stride along k
        vb = oracle.View(bbuf, (k, n), (1, k))
    got = kx.matmul(_view(kx, torch_cuda, abuf, (m, k), (k + pad, 1)),
                    _view(kx, torch_cuda, bbuf, vb.dims, vb.strides)).cpu().numpy()
    assert tc_handle.last_kernel.startswith("tc_3xtf32"), tc_handle.last_kernel
    tc_handle.synchronize()
    _check(got, va, vb)


@pytest.mark.parametrize("m,k,n,width", [(512, 96, 8192, "128x224"), (520, 1040, 1000, "128x128"),
                                         (4096, 64, 8192, "128x256"), (1024, 200, 128, "128x128")])
@pytest.mark.parametrize("b_layout", ["row", "col"])
def test_tc_tile_widths(kx, torch_cuda, tc_handle, m, k, n, width, b_layout):
    """Each tile width the wave model picks (224: packs into whole waves, 128:
    narrow products, 256: the rest), ragged last column tiles included,
    against the compensated oracle."""
    rng = np.random.default_rng(m + n + k)
    abuf = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    if b_layout == "row":
        bbuf = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        vb = oracle.View(bbuf, (k, n), (n, 1))
    else:
        bbuf = rng.uniform(-1, 1, (n, k)).astype(np.float32)
        vb = oracle.View(bbuf, (k, n), (1, k))
    got = kx.matmul(_view(kx, torch_cuda, abuf, (m, k), (k, 1)),
                    _view(kx, torch_cuda, bbuf, vb.dims, vb.strides)).cpu().numpy()
    assert width in tc_handle.last_kernel, tc_handle.last_kernel
    tc_handle.synchronize()
    rows = np.r_[0:3, m // 2, m - 2:m]
    _check(got[rows], oracle.View(abuf[rows].copy(), (len(rows), k), (k, 1)), vb)


def test_tc_batched_and_broadcast(kx, torch_cuda, tc_handle):
    torch = torch_cuda
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (4, 256, 96)).astype(np.float32)
    b = rng.uniform(-1, 1, (4, 96, 512)).astype(np.float32)
    bb = rng.uniform(-1, 1, (1, 96, 512)).astype(np.float32)
    for bm in (b, bb):
        got = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(bm).cuda()).cpu().numpy()
        assert tc_handle.last_kernel.startswith("tc_3xtf32")
        for i in range(4):
            _check(got[i], oracle.View.of(a[i]), oracle.View.of(bm[min(i, bm.shape[0] - 1)]))
    # attention-shaped: Q [2,4,256,128] x K^T (K [2,4,256,128] viewed transposed): batch axes merge
    q = rng.uniform(-1, 1, (2, 4, 256, 128)).astype(np.float32)
    kk = rng.uniform(-1, 1, (2, 4, 256, 128)).astype(np.float32)
    s = kx.matmul(torch.from_numpy(q).cuda(), torch.from_numpy(kk).cuda().transpose(2, 3)).cpu().numpy()
    assert tc_handle.last_kernel.startswith("tc_3xtf32_128x") and tc_handle.last_kernel.endswith("_bk")
    for i, j in [(0, 0), (1, 3)]:
        _check(s[i, j], oracle.View.of(q[i, j]), oracle.View(kk[i, j], (128, 256), (1, 128)))
    tc_handle.synchronize()


@pytest.mark.parametrize("m,n,width", [(128, 256, "128x128"), (512, 8192, "128x224"), (4096, 8192, "128x256")])
def test_tc_nonfinite_keeps_ieee_propagation(kx, torch_cuda, tc_handle, m, n, width):
    """An inf in A must give inf (not NaN from inf * 0 in a cross term)."""
    torch = torch_cuda
    a = np.full((m, 64), 0.5, dtype=np.float32)
    b = np.ones((64, n), dtype=np.float32)
    a[3, 7] = np.inf
    a[5, 2] = np.nan
    got = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert width in tc_handle.last_kernel, tc_handle.last_kernel
    tc_handle.set_f32_variant(1)
    ref = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    assert np.isinf(got[3]).all() and np.isnan(got[5]).all()
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin], ref[fin])


def test_auto_selects_tensor_cores_for_large_products(kx, torch_cuda):
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    a = torch.rand(2048, 512, device="cuda") * 2 - 1
    b = torch.rand(512, 2048, device="cuda") * 2 - 1
    c = kx.matmul(a, b)
    assert h.last_kernel.startswith("tc_3xtf32"), h.last_kernel
    exp, ab = oracle.gemm_dot2(oracle.View.of(a.cpu().numpy()[:64]), oracle.View.of(b.cpu().numpy()))
    assert (np.abs(c[:64].cpu().numpy().astype(np.float64) - exp) <= 2e-6 * ab).all()
    h.set_f32_variant(1)
    kx.matmul(a, b)
    assert h.last_kernel.startswith("simt"), h.last_kernel
    h.set_f32_variant(0)
    h.synchronize()


@pytest.mark.parametrize("b_layout", ["row", "col"])
@pytest.mark.parametrize("m,k,n", [(2304, 200, 4352), (4096, 1040, 2400)])
def test_tc_pair_kernel(kx, torch_cuda, pair_handle, b_layout, m, k, n):
    """CTA-pair kernel (tcgen05 cta_group::2, 256 x 256 tiles): ragged k, m and
    n edges, both B layouts, row samples from both CTAs of a pair."""
    rng = np.random.default_rng(m + k + n)
    pad = 4
    abuf = rng.uniform(-1, 1, (m, k + pad)).astype(np.float32)
    if b_layout == "row":
        bbuf = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        vb = oracle.View(bbuf, (k, n), (n, 1))
    else:
        bbuf = rng.uniform(-1, 1, (n, k)).astype(np.float32)
        vb = oracle.View(bbuf, (k, n), (1, k))
    got = kx.matmul(_view(kx, torch_cuda, abuf, (m, k), (k + pad, 1)),
                    _view(kx, torch_cuda, bbuf, vb.dims, vb.strides)).cpu().numpy()
    assert pair_handle.last_kernel.startswith("tc_3xtf32_pair"), pair_handle.last_kernel
    pair_handle.synchronize()
    rows = np.array([0, 1, 127, 128, 129, 255, 256, 383, m // 2, m - 129, m - 1])
    _check(got[rows], oracle.View(np.ascontiguousarray(abuf[rows, :k]), (len(rows), k), (k, 1)), vb)


def test_tc_pair_batched_and_nonfinite(kx, torch_cuda, pair_handle):
    torch = torch_cuda
    rng = np.random.default_rng(8)
    a = rng.uniform(-1, 1, (3, 1024, 96)).astype(np.float32)
    b = rng.uniform(-1, 1, (3, 96, 1536)).astype(np.float32)
    got = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert pair_handle.last_kernel.startswith("tc_3xtf32_pair"), pair_handle.last_kernel
    for i in range(3):
        rows = np.array([0, 200, 511, 700, 1023])
        _check(got[i][rows], oracle.View(np.ascontiguousarray(a[i][rows]), (5, 96), (96, 1)), oracle.View.of(b[i]))
    # an inf in the peer CTA's rows and a NaN in the leader's: IEEE propagation as the FFMA path
    a2 = np.full((2048, 64), 0.5, dtype=np.float32)
    b2 = np.ones((64, 8192), dtype=np.float32)
    a2[130, 7] = np.inf
    a2[3, 2] = np.nan
    got = kx.matmul(torch.from_numpy(a2).cuda(), torch.from_numpy(b2).cuda()).cpu().numpy()
    assert pair_handle.last_kernel.startswith("tc_3xtf32_pair"), pair_handle.last_kernel
    assert np.isinf(got[130]).all() and np.isnan(got[3]).all()
    fin = np.isfinite(got)
    assert np.array_equal(got[fin], np.full(fin.sum(), 32.0, dtype=np.float32))
    pair_handle.synchronize()


def test_tc_short_k_output_paths(kx, torch_cuda):
    """The short-K kernel stores C through a tensor map in 32 x 32 boxes
    (clipped at ragged edges, batched scores) and with plain stores for
    single-row products; every output element is checked against f64 with
    the f32 bound."""
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    rng = np.random.default_rng(23)
    a = rng.uniform(-1, 1, (4100, 300)).astype(np.float32)
    b = rng.uniform(-1, 1, (300, 2052)).astype(np.float32)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c = torch.empty(4100, 2052, device="cuda")
    kx.matmul_into(da, db, c)
    assert h.last_kernel == "tc_3xtf32_short_128x128_bmn", h.last_kernel
    got = c.cpu().numpy().astype(np.float64)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    bound = 2e-6 * (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)) + 1e-30
    assert (np.abs(got - exact) <= bound).all()
    # single-row products (600 batches of 1 x 128 x 128): no row stride for a
    # tensor map -> plain stores
    a1 = rng.uniform(-1, 1, (600, 1, 128)).astype(np.float32)
    b1 = rng.uniform(-1, 1, (600, 128, 128)).astype(np.float32)
    c1 = kx.matmul(torch.from_numpy(a1).cuda(), torch.from_numpy(b1).cuda()).cpu().numpy().astype(np.float64)
    assert h.last_kernel == "tc_3xtf32_short_128x128_bmn", h.last_kernel
    a64, b64 = a1.astype(np.float64), b1.astype(np.float64)
    assert (np.abs(c1 - a64 @ b64) <= 2e-6 * (np.abs(a64) @ np.abs(b64)) + 1e-30).all()
    q = rng.standard_normal((4, 8, 512, 128)).astype(np.float32)     # 512 tiles
    k = rng.standard_normal((4, 8, 512, 128)).astype(np.float32)
    s = kx.matmul(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda().transpose(2, 3)).cpu().numpy()
    assert h.last_kernel == "tc_3xtf32_short_128x128_bk", h.last_kernel
    q64, k64 = q.astype(np.float64), k.astype(np.float64)
    exact = np.einsum("bhik,bhjk->bhij", q64, k64)
    bound = 2e-6 * np.einsum("bhik,bhjk->bhij", np.abs(q64), np.abs(k64)) + 1e-30
    assert (np.abs(s - exact) <= bound).all()
    h.synchronize()


@pytest.mark.parametrize("m,n,nb", [(2048 + 45, 2304 + 36, 1), (2048 + 100, 2304 + 92, 1), (2048 + 70, 2304 + 124, 1),
                                    (2048 + 1, 2304 + 4, 1), (333, 300, 40)])
def test_tc_short_k_box_edges_every_position(kx, torch_cuda, m, n, nb):
    """The staged 32 x 32 box stores with the matrix edge inside each of the
    four row quarters and each of the four 32-column blocks of a 128 x 128
    tile (partially clipped boxes there, wholly clipped ones beyond), and a
    batched product whose last rows of every batch end inside a box (the
    tensor map's batch dimension clips them); every element against f64."""
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    rng = np.random.default_rng(m * 7 + n)
    a = rng.uniform(-1, 1, (nb, m, 96)).astype(np.float32)
    b = rng.uniform(-1, 1, (nb, 96, n)).astype(np.float32)
    c = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy().astype(np.float64)
    assert h.last_kernel == "tc_3xtf32_short_128x128_bmn", h.last_kernel
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    bound = 2e-6 * (np.abs(a64) @ np.abs(b64)) + 1e-30
    assert (np.abs(c - a64 @ b64) <= bound).all()
    h.synchronize()


@pytest.mark.parametrize("m,k,n", [(512, 512, 512), (256, 1024, 256), (128, 4096, 128), (1024, 512, 1024),
                                   (200, 768, 132)])
def test_small_products_split_k_on_the_tensor_cores(kx, torch_cuda, m, k, n):
    """Products with too few tiles to fill the SMs split K over the tensor-core
    kernel (the K slices described as a batch) and sum the slices in order:
    every output against the compensated oracle with the f32 bound."""
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    from kernix_b200 import rng
    v = rng.uniform(131, m * k + k * n, -1, 1)
    a_np, b_np = v[:m * k].reshape(m, k), v[m * k:].reshape(k, n)
    c = kx.matmul(torch.from_numpy(a_np).cuda(), torch.from_numpy(b_np).cuda()).cpu().numpy()
    assert h.last_kernel == "tc_3xtf32_splitk", h.last_kernel
    want, absum = oracle.gemm_dot2(oracle.View.of(a_np), oracle.View.of(b_np))
    assert (np.abs(c.astype(np.float64) - want) <= 2e-6 * absum + 1e-30).all()


def test_split_k_back_to_back_and_guarded_output(kx, torch_cuda):
    """K-sliced tensor-core products back to back with new data on the same
    handle (the shared slice workspace reused) match the oracle, and a product
    into an output inside a larger buffer is bitwise the same with the guard
    elements on both sides untouched."""
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    rs = np.random.default_rng(11)
    m = k = n = 512
    for trial in range(3):
        a = rs.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rs.uniform(-1, 1, (k, n)).astype(np.float32)
        da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        c = kx.matmul(da, db)
        assert h.last_kernel == "tc_3xtf32_splitk", h.last_kernel
        want, absum = oracle.gemm_dot2(oracle.View.of(a.astype(np.float64)), oracle.View.of(b.astype(np.float64)))
        assert (np.abs(c.cpu().numpy().astype(np.float64) - want) <= 2e-6 * absum + 1e-30).all()
        buf = torch.full((m * n + 8,), -7.0, device="cuda")
        kx.matmul_into(da, db, kx.TensorView(buf, (m, n), (n, 1), 4))
        assert h.last_kernel == "tc_3xtf32_splitk"
        assert (buf[:4] == -7.0).all() and (buf[4 + m * n:] == -7.0).all()
        assert torch.equal(buf[4:4 + m * n].reshape(m, n), c)


def test_split_k_nonfinite_and_uneven_k(kx, torch_cuda):
    """inf and NaN in A propagate through the split slices as through one
    f32 accumulation; a K the slices cannot divide evenly keeps the SIMT
    split-K kernel."""
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    rs = np.random.default_rng(3)
    a = rs.uniform(-1, 1, (512, 512)).astype(np.float32)
    b = rs.uniform(-1, 1, (512, 512)).astype(np.float32)
    a[7, 300] = np.inf
    a[9, 10] = np.nan
    c = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert h.last_kernel == "tc_3xtf32_splitk"
    assert np.isnan(c[9]).all()
    assert np.array_equal(np.isinf(c[7]), b[300] != 0) and not np.isnan(c[7][b[300] != 0]).any()
    fin = np.ones(512, bool)
    fin[[7, 9]] = False
    assert np.isfinite(c[fin]).all()
    a2 = rs.uniform(-1, 1, (512, 520)).astype(np.float32)
    b2 = rs.uniform(-1, 1, (520, 512)).astype(np.float32)
    c2 = kx.matmul(torch.from_numpy(a2).cuda(), torch.from_numpy(b2).cuda()).cpu().numpy()
    assert h.last_kernel.startswith("simt"), h.last_kernel
    want, absum = oracle.gemm_dot2(oracle.View.of(a2), oracle.View.of(b2))
    assert (np.abs(c2.astype(np.float64) - want) <= 2e-6 * absum + 1e-30).all()


def test_tc_short_k_persistent(kx, torch_cuda):
    """K <= 1024 over many tiles: the persistent kernel (TMEM double-buffered,
    epilogue overlapping the next tile) -- attention scores Q K^T with a
    transposed K view, a ragged row-major case and inf/NaN propagation."""
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f32_variant(0)
    rng = np.random.default_rng(17)
    q = rng.standard_normal((4, 8, 512, 128)).astype(np.float32)
    k = rng.standard_normal((4, 8, 512, 128)).astype(np.float32)
    s = kx.matmul(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda().transpose(2, 3)).cpu().numpy()
    assert h.last_kernel == "tc_3xtf32_short_128x128_bk", h.last_kernel
    for bi, hi in [(0, 0), (3, 7), (2, 5)]:
        rows = np.array([0, 127, 128, 300, 511])
        _check(s[bi, hi][rows], oracle.View(np.ascontiguousarray(q[bi, hi][rows]), (5, 128), (128, 1)),
               oracle.View(k[bi, hi], (128, 512), (1, 128)))
    a = rng.uniform(-1, 1, (4100, 300)).astype(np.float32)
    b = rng.uniform(-1, 1, (300, 2052)).astype(np.float32)   # row pitch 8208 B: TMA-aligned
    c = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert h.last_kernel == "tc_3xtf32_short_128x128_bmn", h.last_kernel
    rows = np.array([0, 1, 2047, 4095, 4096, 4099])
    _check(c[rows], oracle.View(np.ascontiguousarray(a[rows]), (len(rows), 300), (300, 1)), oracle.View.of(b))
    a[5, 7] = np.inf
    a[4097, 3] = np.nan
    c = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert h.last_kernel == "tc_3xtf32_short_128x128_bmn", h.last_kernel
    assert np.isnan(c[4097]).all()
    assert np.array_equal(np.isinf(c[5]), b[7] != 0) and not np.isnan(c[5][b[7] != 0]).any()
    fin = np.isfinite(c).all(axis=1)
    assert fin[:5].all() and fin[6:4097].all()
    h.synchronize()


def test_expired_waits_report_timeout_and_leave_the_handle_usable(kx, torch_cuda):
    """The bounded-wait path: a diagnostic launch of the one-SM kernel issues no
    copies and bounds its waits by 1 ms, so every wait expires.  The kernel
    stops, frees its tensor memory and sets the status word; synchronize reports
    DeviceTimeout once; the next products on the same handle are correct."""
    from kernix_b200 import rng
    torch = torch_cuda
    h = kx.handle(0)
    m, k, n = 256, 2048, 384                    # K > 1024: not the short-K kernel
    a = rng.uniform(71, m * k, -1.0, 1.0).reshape(m, k)
    b = rng.uniform(72, k * n, -1.0, 1.0).reshape(k, n)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    out = torch.full((m, n), 7.0, device="cuda")
    h.set_f32_variant(3)                         # one-SM split-TF32 tiles
    try:
        h.synchronize()
        h.diag_expire_next_gemm(1_000_000)
        kx.matmul_into(da, db, out)
        assert h.last_kernel.startswith("tc_3xtf32_128x")
        with pytest.raises(kx.DeviceTimeout):
            h.synchronize()
        h.synchronize()                          # reported once, then cleared
        got = kx.matmul(da, db)
        assert h.last_kernel.startswith("tc_3xtf32_128x")
        h.synchronize()
    finally:
        h.set_f32_variant(0)
    want, absum = oracle.gemm_dot2(oracle.View.of(a), oracle.View.of(b))
    assert (np.abs(got.cpu().numpy().astype(np.float64) - want) <= 2e-6 * absum).all()
    with pytest.raises(kx.InvalidParameter):
        h.diag_expire_next_gemm(10)               # below 1 ms
