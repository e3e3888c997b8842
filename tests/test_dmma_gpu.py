"""f64 on the FP64 tensor pipe (mma.sync m16n8k4 .f64) against the oracle.

Every case forces the DMMA kernel (kx_set_f64_variant(KX_F64_DMMA)) so the
reference's f64 contracts are checked on it directly: exact integer/dyadic
results (ops_tests.rs:239-320, small_matmul_tests.rs:59-106), the scaled bound
|x - y| <= 1e-13 sum|a b| (small_matmul_tests.rs:153-186), batched geometry
(batched_matmul_tests.rs:5-48) and IEEE propagation of inf/NaN like the DFMA
kernel.
"""
import numpy as np
import pytest

import oracle
from golden import golden as G

pytestmark = pytest.mark.gpu


@pytest.fixture
def dmma(kx, torch_cuda):
    h = kx.handle(0)
    h.set_f64_variant(2)    # KX_F64_DMMA
    yield h
    h.set_f64_variant(0)


def to_dev(arr, torch):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def _views(kx, torch, rng, m, k, n, a_kc, b_kc):
    """A and B with unit stride along k (``*_kc``) or along m / n, each from a
    padded buffer so rows are not dense."""
    if a_kc:
        abuf = rng.standard_normal((m, k + 3))
        va = oracle.View(abuf, (m, k), (k + 3, 1))
    else:
        abuf = rng.standard_normal((k, m + 5))
        va = oracle.View(abuf, (m, k), (1, m + 5))
    if b_kc:
        bbuf = rng.standard_normal((n, k + 1))
        vb = oracle.View(bbuf, (k, n), (1, k + 1))
    else:
        bbuf = rng.standard_normal((k, n + 2))
        vb = oracle.View(bbuf, (k, n), (n + 2, 1))
    ta = kx.TensorView(to_dev(abuf.reshape(-1), torch), va.dims, va.strides, 0)
    tb = kx.TensorView(to_dev(bbuf.reshape(-1), torch), vb.dims, vb.strides, 0)
    return va, vb, ta, tb


@pytest.mark.parametrize("a_kc", [True, False])
@pytest.mark.parametrize("b_kc", [True, False])
@pytest.mark.parametrize("m,k,n", [(130, 37, 129), (1, 16, 1), (257, 64, 96), (64, 300, 255)])
def test_dmma_layouts_against_compensated_oracle(kx, torch_cuda, dmma, a_kc, b_kc, m, k, n):
    rng = np.random.default_rng(m * 1000 + k * 10 + n)
    va, vb, ta, tb = _views(kx, torch_cuda, rng, m, k, n, a_kc, b_kc)
    got = kx.matmul(ta, tb).cpu().numpy()
    assert dmma.last_kernel == "dmma_128x128", dmma.last_kernel
    exp, ab = oracle.gemm_dot2(va, vb)
    assert (np.abs(got - exp) <= 1e-13 * ab + 1e-300).all()


def test_dmma_even_sizes_take_16_byte_copies(kx, torch_cuda, dmma):
    """Even extents and aligned rows: the paired-copy loader, c2's layout
    (row-major A, B the transposed view of a row-major matrix)."""
    torch = torch_cuda
    rng = np.random.default_rng(2)
    a = rng.standard_normal((384, 256))
    bt = rng.standard_normal((320, 256))
    got = kx.matmul(to_dev(a, torch), to_dev(bt, torch).t()).cpu().numpy()
    assert dmma.last_kernel == "dmma_128x128"
    exp, ab = oracle.gemm_dot2(oracle.View.of(a), oracle.View(bt, (256, 320), (1, 256)))
    assert (np.abs(got - exp) <= 1e-13 * ab).all()


@pytest.mark.parametrize("case", ["exact_integers", "dyadic"])
def test_dmma_exact_results(kx, torch_cuda, dmma, case):
    """Integer and dyadic products are exact in f64 whatever the summation
    order (ops_tests.rs:239-320, small_matmul_tests.rs:59-106)."""
    torch = torch_cuda
    rng = np.random.default_rng(7)
    if case == "exact_integers":
        a = rng.integers(-50, 50, (150, 70)).astype(np.float64)
        b = rng.integers(-50, 50, (70, 140)).astype(np.float64)
    else:
        a = rng.integers(-64, 64, (131, 66)).astype(np.float64) / 64.0
        b = rng.integers(-64, 64, (66, 133)).astype(np.float64) / 32.0
    got = kx.matmul(to_dev(a, torch), to_dev(b, torch)).cpu().numpy()
    assert np.array_equal(got, a @ b)


@pytest.mark.parametrize("shape", [s for s in G.EXECUTION_SHAPES if min(s) > 0])
def test_dmma_execution_boundaries_exact(kx, torch_cuda, dmma, shape):
    m, k, n = shape
    a, b = G.execution_pair(m, k, n)
    got = kx.matmul(to_dev(a, torch_cuda), to_dev(b, torch_cuda)).cpu().numpy()
    assert np.array_equal(got, a @ b)


@pytest.mark.parametrize("scale", [1e-100, 1.0, 1e100])
def test_dmma_scaled_error_bounds(kx, dmma, scale):
    a, b = G.scaled_pair(scale, np.float64)
    out = np.full(31 * 32, np.nan)
    assert kx.try_dense_matmul(a.reshape(-1), b.reshape(-1), out, 31, 63, 32)
    exp, ab = oracle.gemm_dot2(oracle.View.of(a), oracle.View.of(b), threads=1)
    got = out.reshape(31, 32)
    assert np.isfinite(got).all()
    assert (np.abs(got - exp) <= 1e-13 * ab).all()


def test_dmma_batched_and_broadcast(kx, torch_cuda, dmma):
    torch = torch_cuda
    rng = np.random.default_rng(11)
    a = rng.standard_normal((3, 2, 70, 40))
    b = rng.standard_normal((2, 40, 90))        # broadcast over the leading batch
    got = kx.matmul(to_dev(a, torch), to_dev(b, torch)).cpu().numpy()
    assert dmma.last_kernel == "dmma_128x128"
    for i in range(3):
        for j in range(2):
            exp, ab = oracle.gemm_dot2(oracle.View.of(a[i, j]), oracle.View.of(b[j]))
            assert (np.abs(got[i, j] - exp) <= 1e-13 * ab).all()


def test_dmma_nonfinite_propagation_matches_dfma(kx, torch_cuda, dmma):
    torch = torch_cuda
    a = np.full((40, 24), 0.5)
    b = np.ones((24, 36))
    a[3, 7] = np.inf
    a[5, 2] = np.nan
    b[4, 30] = -np.inf
    got = kx.matmul(to_dev(a, torch), to_dev(b, torch)).cpu().numpy()
    dmma.set_f64_variant(1)
    ref = kx.matmul(to_dev(a, torch), to_dev(b, torch)).cpu().numpy()
    assert dmma.last_kernel.startswith("simt")
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    inf = np.isinf(ref)
    assert np.array_equal(np.sign(got[inf]), np.sign(ref[inf]))
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin], ref[fin])   # dyadic sums: exact in any order


def test_auto_selects_dmma_for_large_f64(kx, torch_cuda):
    torch = torch_cuda
    h = kx.handle(0)
    h.set_f64_variant(0)
    a = torch.randn(1536, 256, dtype=torch.float64, device="cuda")
    b = torch.randn(256, 1280, dtype=torch.float64, device="cuda")
    c = kx.matmul(a, b)
    assert h.last_kernel == "dmma_128x128", h.last_kernel
    exp, ab = oracle.gemm_dot2(oracle.View.of(a.cpu().numpy()[:40]), oracle.View.of(b.cpu().numpy()))
    assert (np.abs(c[:40].cpu().numpy() - exp) <= 1e-13 * ab).all()
