"""Device GEMM parity against the oracle on the reference's own test cases.

Every case here mirrors a Kernix test (cited) and calls through the C ABI
(kernix_b200 -> libkernix_b200.so).  Integer/dyadic cases must be exact;
the rest use the reference's tolerances.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from golden import golden as G

pytestmark = pytest.mark.gpu
KATS = json.loads((Path(__file__).parent / "golden" / "kats.json").read_text())


@pytest.fixture(scope="module")
def dev(torch_cuda):
    return torch_cuda.device("cuda:0")


def to_dev(arr, torch):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def view(kx, torch, buf, dims, strides, origin=0):
    return kx.TensorView(to_dev(np.ascontiguousarray(buf).reshape(-1), torch), list(dims), list(strides), origin)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("case", KATS["matmul_int"], ids=lambda c: c["cite"].split()[-1])
def test_known_answers(kx, torch_cuda, case, dtype):
    def mk(spec):
        if "storage" in spec:
            return view(kx, torch_cuda, np.asarray(spec["storage"], dtype), spec["dims"], spec["strides"],
                        spec["origin"])
        return to_dev(np.asarray(spec["values"], dtype).reshape(spec["dims"]), torch_cuda)
    out = kx.matmul(mk(case["a"]), mk(case["b"]))
    assert list(out.shape) == case["out_dims"]
    assert out.cpu().numpy().reshape(-1).tolist() == case["out"]


def test_errors_through_device_api(kx, torch_cuda):
    a = torch_cuda.zeros(2, 3, device="cuda")
    b = torch_cuda.zeros(4, 2, device="cuda")
    with pytest.raises(kx.ContractDimensionMismatch) as e:
        kx.matmul(a, b)
    assert (e.value.left, e.value.right) == (3, 4)
    with pytest.raises(kx.InvalidRank):
        kx.matmul(torch_cuda.zeros((), device="cuda"), a)
    with pytest.raises(kx.BroadcastIncompatible):
        kx.matmul(torch_cuda.zeros(2, 3, 4, device="cuda"), torch_cuda.zeros(3, 4, 5, device="cuda"))
    out = torch_cuda.zeros(3, 3, device="cuda")
    with pytest.raises(kx.LayoutError):
        kx.matmul_into(torch_cuda.zeros(3, 2, device="cuda"), torch_cuda.zeros(2, 3, device="cuda"), out.t())
    with pytest.raises(kx.OverlappingOutput):
        x = torch_cuda.zeros(3, 3, device="cuda")
        kx.matmul_into(x, torch_cuda.zeros(3, 3, device="cuda"), x)


@pytest.mark.parametrize("pair", KATS["batched_shapes"]["pairs"], ids=str)
def test_batched_geometry(kx, torch_cuda, pair):
    """batched_matmul_tests.rs:5-48 (f64 2e-13, f32 3e-6 relative to 1+|y|)."""
    a_dims, b_dims, out_dims = pair
    a = G.batched_values(a_dims, "left")
    b = G.batched_values(b_dims, "right")
    exp = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
    got = kx.matmul(to_dev(a, torch_cuda), to_dev(b, torch_cuda)).cpu().numpy()
    assert list(got.shape) == out_dims
    assert (np.abs(got - exp) < 2e-13 * (1 + np.abs(exp))).all()
    af, bf = a.astype(np.float32), b.astype(np.float32)
    expf = oracle.matmul_reference(oracle.View.of(af), oracle.View.of(bf))
    gotf = kx.matmul(to_dev(af, torch_cuda), to_dev(bf, torch_cuda)).cpu().numpy()
    assert (np.abs(gotf.astype(np.float64) - expf) < 3e-6 * (1 + np.abs(expf))).all()


def test_strided_batches_swapped_and_reversed(kx, torch_cuda):
    """batched_matmul_tests.rs:49-65: swap_axes(1,2) then reverse_axis(2) of a [2,3,4] tensor."""
    base = np.arange(24, dtype=np.float64) / 17.0
    # [2,3,4] C-order strides (12,4,1) -> swap(1,2): dims [2,4,3] strides (12,1,4)
    # -> reverse axis 2 (len 3): stride -4, origin += 2*4
    va = oracle.View(base, (2, 4, 3), (12, 1, -4), 8)
    b = np.full((3, 2), 0.7)
    exp = oracle.matmul_reference(va, oracle.View.of(b))
    dv = view(kx, torch_cuda, base, (2, 4, 3), (12, 1, -4), 8)
    # The reference's matmul sends this view to its ordered fallback, so it
    # equals matmul_reference exactly; the device's ordered mode does the same.
    assert np.array_equal(kx.matmul_reference(dv, to_dev(b, torch_cuda)).cpu().numpy(), exp)
    got = kx.matmul(dv, to_dev(b, torch_cuda)).cpu().numpy()
    assert (np.abs(got - exp) < 2e-13 * (1 + np.abs(exp))).all()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_ordered_mode_is_bitwise_matmul_reference(kx, torch_cuda, dtype):
    """execution_tests.rs:23-32 / native_kernel_tests.rs:51-69: the ordered
    path equals matmul_reference bit for bit, for any layout and batch."""
    rng = np.random.default_rng(3)
    cases = [
        ((7, 11), (11, 5)), ((65, 67), (67, 69)), ((17, 31), (31, 19)), ((3, 1, 9, 40), (5, 40, 12)),
        ((40,), (40, 9)), ((9, 40), (40,)), ((40,), (40,)), ((129, 300), (300, 131)),
    ]
    for a_dims, b_dims in cases:
        a = rng.uniform(-1, 1, a_dims).astype(dtype)
        b = rng.uniform(-1, 1, b_dims).astype(dtype)
        exp = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
        got = kx.matmul_reference(to_dev(a, torch_cuda), to_dev(b, torch_cuda)).cpu().numpy()
        assert np.array_equal(got, exp), (a_dims, b_dims)
    # transpose (a.T) times reversed rows, through views
    a = rng.uniform(-1, 1, (33, 21)).astype(dtype)
    b = rng.uniform(-1, 1, (33, 14)).astype(dtype)
    va, vb = oracle.View(a, (21, 33), (1, 21), 0), oracle.View(b, (33, 14), (-14, 1), 32 * 14)
    exp = oracle.matmul_reference(va, vb)
    got = kx.matmul_reference(view(kx, torch_cuda, a, (21, 33), (1, 21)),
                              view(kx, torch_cuda, b, (33, 14), (-14, 1), 32 * 14)).cpu().numpy()
    assert np.array_equal(got, exp)
    assert not kx.handle(0).ordered_matmul


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_dyadic_boundary_grid_through_dense_hook(kx, dtype):
    """small_matmul_tests.rs:59-106: exact, unaligned slices, NaN guards, reused output."""
    for m in G.DYADIC_M:
        for k in G.DYADIC_K:
            for n in G.DYADIC_N:
                av, bv = G.dyadic_pair(m, k, n, dtype)
                a, b = av[1:], bv[1:]
                out = np.full(m * n + 2, np.nan, dtype=dtype)
                exact = (a.astype(np.float64).reshape(m, k) @ b.astype(np.float64).reshape(k, n)).reshape(-1)
                for _ in range(2):
                    assert kx.try_dense_matmul(a, b, out[1:1 + m * n], m, k, n)
                    assert np.array_equal(out[1:1 + m * n].astype(np.float64), exact), (m, k, n)
                    assert np.isnan(out[0]) and np.isnan(out[-1])


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("shape", G.GAPPED_SHAPES)
def test_gapped_strides_through_strided_hook(kx, shape, dtype):
    """native_kernel_tests.rs:243-294: exact, NaN guard cells."""
    m, k, n = shape
    a, (ars, acs), ao, b, (brs, bcs), bo = G.gapped_strides(m, k, n, dtype)
    ma = kx.MatrixInput(a, [m, k], [ars, acs], ao)
    mb = kx.MatrixInput(b, [k, n], [brs, bcs], bo)
    out = np.full(m * n + 2, np.nan, dtype=dtype)
    assert kx.try_strided_matmul(ma, mb, out[1:1 + m * n])
    exact = oracle.View(a, (m, k), (ars, acs), ao).to_array().astype(np.float64) @ \
        oracle.View(b, (k, n), (brs, bcs), bo).to_array().astype(np.float64)
    assert np.array_equal(out[1:1 + m * n].astype(np.float64), exact.reshape(-1))
    assert np.isnan(out[0]) and np.isnan(out[-1])


def test_strided_hook_singleton_and_declines(kx):
    """native_kernel_tests.rs:17-28."""
    a = kx.MatrixInput(np.array([1.0]), [1, 1], [-(1 << 63), -(1 << 63)], 0)
    b = kx.MatrixInput(np.array([2.0]), [1, 1], [0, 0], 0)
    out = np.zeros(1)
    assert kx.try_strided_matmul(a, b, out) and out[0] == 2.0
    out = np.full(4, 7.0)
    assert not kx.try_dense_matmul(np.ones(1), np.full(1, 2.0), out, 2, 2, 2)
    assert (out == 7.0).all()


def test_tails_transposes_reversals_and_zero_dims(kx, torch_cuda):
    """native_kernel_tests.rs:29-49 (1e-13 (1 + |y|))."""
    for (m, k, n) in [(17, 31, 19), (1, 1, 1), (4, 0, 3), (0, 7, 3), (3, 7, 0)]:
        a, b = G.tensor_native(m, k), G.tensor_native(k, n)
        exp = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
        got = kx.matmul(to_dev(a, torch_cuda), to_dev(b, torch_cuda)).cpu().numpy()
        assert got.shape == exp.shape
        assert (np.abs(got - exp) < 1e-13 * (1 + np.abs(exp))).all()
    a, b = G.tensor_native(9, 7), G.tensor_native(9, 5)
    # a.transpose(): dims [7,9] strides (1,7); b.reverse_axis(0): dims [9,5] strides (-5,1) origin 40
    va, vb = oracle.View(a, (7, 9), (1, 7), 0), oracle.View(b, (9, 5), (-5, 1), 40)
    exp = oracle.matmul_reference(va, vb)
    got = kx.matmul(view(kx, torch_cuda, a, (7, 9), (1, 7), 0),
                    view(kx, torch_cuda, b, (9, 5), (-5, 1), 40)).cpu().numpy()
    assert (np.abs(got - exp) < 1e-13 * (1 + np.abs(exp))).all()


@pytest.mark.parametrize("shape", G.F64_BOUNDARY_SHAPES)
def test_f64_boundaries_and_reused_output(kx, torch_cuda, shape):
    """native_kernel_tests.rs:71-108: 1e-12 (1 + |y|), matmul_into keeps the pointer, bitwise equal."""
    m, k, n = shape
    a, b = G.tensor_native(m, k), G.tensor_native(k, n)
    exp = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
    da, db = to_dev(a, torch_cuda), to_dev(b, torch_cuda)
    got = kx.matmul(da, db)
    reused = torch_cuda.full((m, n), float("nan"), dtype=torch_cuda.float64, device="cuda")
    ptr = reused.data_ptr()
    for _ in range(2):
        kx.matmul_into(da, db, reused)
        assert reused.data_ptr() == ptr
        assert torch_cuda.equal(reused, got)
    g = got.cpu().numpy()
    assert (np.abs(g - exp) < 1e-12 * (1 + np.abs(exp))).all()


@pytest.mark.parametrize("shape", G.F32_BOUNDARY_SHAPES)
def test_f32_matches_f64_oracle(kx, torch_cuda, shape):
    """native_kernel_tests.rs:139-181: |x - y| < 1e-5 (1 + |y|)."""
    m, k, n = shape
    a, b = G.f32_boundary_pair(m, k, n)
    got = kx.matmul(to_dev(a, torch_cuda), to_dev(b, torch_cuda)).cpu().numpy().astype(np.float64)
    exp = a.astype(np.float64) @ b.astype(np.float64)
    assert (np.abs(got - exp) < 1e-5 * (1 + np.abs(exp))).all()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_broadcast_batches_exact_integers(kx, torch_cuda, dtype):
    """native_kernel_tests.rs:110-137,183-199."""
    a = ((np.arange(2 * 64 * 65) % 7) - 3).astype(dtype).reshape(2, 64, 65)
    b = ((np.arange(65 * 67) % 11) - 5).astype(dtype).reshape(1, 65, 67)
    exp = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
    got = kx.matmul(to_dev(a, torch_cuda), to_dev(b, torch_cuda)).cpu().numpy()
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("batch", [1, 4, 16, 64])
def test_small_broadcast_batches(kx, torch_cuda, batch):
    """small_matmul_tests.rs:108-135: exact dyadic small batches."""
    a = ((np.arange(batch * 17 * 32) % 13) / 8.0).reshape(batch, 17, 32)
    b = ((np.arange(32 * 16) % 17) / 16.0).reshape(1, 32, 16)
    exp = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
    got = kx.matmul(to_dev(a, torch_cuda), to_dev(b, torch_cuda)).cpu().numpy()
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("dtype,scales,budget", [(np.float64, [1e-100, 1.0, 1e100], 1e-13),
                                                 (np.float32, [1e-10, 1.0, 1e10], 2e-6)])
def test_scaled_error_bounds(kx, dtype, scales, budget):
    """small_matmul_tests.rs:153-186: |x - y| <= budget * sum |a b|."""
    for scale in scales:
        a, b = G.scaled_pair(scale, dtype)
        out = np.full(31 * 32, np.nan, dtype=dtype)
        assert kx.try_dense_matmul(a.reshape(-1), b.reshape(-1), out, 31, 63, 32)
        got = out.reshape(31, 32).astype(np.float64)
        exp, ab = oracle.gemm_dot2(oracle.View.of(a), oracle.View.of(b), threads=1)
        assert np.isfinite(got).all()
        assert (np.abs(got - exp) <= budget * ab).all(), scale


@pytest.mark.parametrize("shape", G.EXECUTION_SHAPES)
def test_execution_boundaries_exact(kx, torch_cuda, shape):
    """execution_tests.rs:80-120: exact in both dtypes."""
    m, k, n = shape
    a, b = G.execution_pair(m, k, n)
    exact = a @ b if m and n else np.zeros((m, n))
    for dtype in (np.float64, np.float32):
        got = kx.matmul(to_dev(a.astype(dtype), torch_cuda), to_dev(b.astype(dtype), torch_cuda)).cpu().numpy()
        assert np.array_equal(got.astype(np.float64), exact)


def test_layout_modes_and_kernel_families(kx, torch_cuda):
    """Every operand loader (unit stride on k, unit stride on m/n, gathers) and
    both tile families (plain and split-K) against the compensated oracle."""
    h = kx.handle(0)
    rng = np.random.default_rng(7)
    seen = set()
    for (m, k, n) in [(64, 96, 80), (300, 520, 260), (2304, 256, 2304)]:
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        layouts = {
            "row/row": (a, (k, 1), b, (n, 1)),
            "col/col": (np.ascontiguousarray(a.T), (1, m), np.ascontiguousarray(b.T), (1, k)),
            "gather": (np.pad(a, ((0, 0), (0, 3))), (k + 3, 1), np.pad(b, ((0, 0), (0, 1))), (n + 1, 1)),
            "gather-k": (np.pad(a.T, ((0, 0), (0, 1))), (1, m + 1), np.pad(b.T, ((0, 0), (0, 1))), (1, k + 1)),
        }
        for name, (abuf, ast, bbuf, bst) in layouts.items():
            va = oracle.View(abuf, (m, k), ast)
            vb = oracle.View(bbuf, (k, n), bst)
            exp, ab = oracle.gemm_dot2(va, vb)
            got = kx.matmul(view(kx, torch_cuda, abuf, (m, k), ast), view(kx, torch_cuda, bbuf, (k, n), bst))
            seen.add(h.last_kernel)
            g = got.cpu().numpy().astype(np.float64)
            assert (np.abs(g - exp) <= 2e-6 * ab + 1e-30).all(), (name, m, k, n)
    assert {"simt_128x128", "simt_64x64_splitk"} <= seen or {"simt_128x128", "simt_64x64"} <= seen, seen


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_strided_hook_pipelined_large(kx, dtype):
    """try_strided_matmul on a product large enough for the pipelined host
    path (row pieces uploaded, multiplied and downloaded on three streams):
    A a row-strided slice of a wider buffer (disjoint rows), as in the 8192^3
    workload, checked row by row against the compensated oracle and against
    the one-shot device result."""
    import torch
    m, k, n, pitch = 4096, 1536, 1536, 1600
    rng = np.random.default_rng(3)
    abuf = rng.uniform(-1, 1, (m, pitch)).astype(dtype)
    bbuf = rng.uniform(-1, 1, (k, n)).astype(dtype)
    out = np.full(m * n, np.nan, dtype=dtype)
    ma = kx.MatrixInput(abuf.reshape(-1), [m, k], [pitch, 1], 0)
    mb = kx.MatrixInput(bbuf.reshape(-1), [k, n], [n, 1], 0)
    assert kx.try_strided_matmul(ma, mb, out)
    got = out.reshape(m, n)
    assert np.isfinite(got).all()
    bound = 2e-6 if dtype == np.float32 else 1e-13
    for r in (0, 1, 511, 512, 1023, 2048, 4095):
        exp, ab = oracle.gemm_dot2(oracle.View(abuf, (1, k), (pitch, 1), r * pitch), oracle.View.of(bbuf))
        assert (np.abs(got[r].astype(np.float64) - exp[0]) <= bound * ab[0]).all(), r
    dev = kx.matmul(kx.TensorView(torch.from_numpy(abuf.reshape(-1)).cuda(), (m, k), (pitch, 1), 0),
                    torch.from_numpy(bbuf).cuda()).cpu().numpy()
    # the pieces may take another kernel family than the one-shot call
    # (fewer tiles per launch), so the two agree within twice the bound
    ref = np.abs(bbuf).sum(axis=0)[None, :] * np.abs(abuf[:, :k]).max(axis=1)[:, None]
    assert (np.abs(got.astype(np.float64) - dev) <= 2 * bound * ref).all()
