"""Pin the CPU oracle to the reference's own known answers (CPU only).

The reference (Rust) cannot be built in this image, so the oracle is trusted
only after it reproduces every literal known answer and exact-dyadic property
of Kernix's matmul/conv/softmax tests (values in tests/golden/kats.json).
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from golden import golden as G
from kernix_b200 import rng

KATS = json.loads((Path(__file__).parent / "golden" / "kats.json").read_text())


def _view(spec, dtype):
    if "storage" in spec:
        return oracle.View(np.asarray(spec["storage"], dtype=dtype), spec["dims"], spec["strides"], spec["origin"])
    return oracle.View.of(np.asarray(spec["values"], dtype=dtype).reshape(spec["dims"]))


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("case", KATS["matmul_int"], ids=lambda c: c["cite"].split()[-1])
def test_matmul_known_answers(case, dtype):
    out = oracle.matmul_reference(_view(case["a"], dtype), _view(case["b"], dtype))
    assert list(out.shape) == case["out_dims"]
    assert out.reshape(-1).tolist() == case["out"]


@pytest.mark.parametrize("case", KATS["matmul_errors"], ids=lambda c: c["error"])
def test_matmul_error_known_answers(case):
    if case["error"] == "CapacityOverflow":
        out, _, _ = oracle.matmul_shape(case["a_dims"], case["b_dims"])
        n = math.prod(out)
        assert n * 8 > (1 << 63) - 1 and n == case["fields"]["len"]
        return
    with pytest.raises(oracle.OracleError) as e:
        oracle.matmul_shape(case["a_dims"], case["b_dims"])
    assert e.value.kind == case["error"]
    assert e.value.fields == case["fields"]


def test_matmul_empty_output_shapes():
    for case in KATS["matmul_empty_ok"]:
        out, _, _ = oracle.matmul_shape(case["a_dims"], case["b_dims"])
        assert out == case["out_dims"]


@pytest.mark.parametrize("pair", KATS["batched_shapes"]["pairs"], ids=str)
def test_batched_geometry_shapes_and_values(pair):
    a_dims, b_dims, out_dims = pair
    a = G.batched_values(a_dims, "left")
    b = G.batched_values(b_dims, "right")
    out = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
    assert list(out.shape) == out_dims
    np.testing.assert_allclose(out, np.matmul(a, b) if a.size and b.size else np.zeros(out_dims), rtol=0,
                               atol=2e-13 * (1 + np.abs(out).max(initial=0)))


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_dyadic_boundary_grid_is_exact(dtype):
    """small_matmul_tests.rs:59-106: dyadic data makes every sum exact."""
    for m in G.DYADIC_M:
        for k in G.DYADIC_K:
            for n in G.DYADIC_N:
                av, bv = G.dyadic_pair(m, k, n, dtype)
                a, b = av[1:], bv[1:]
                got = oracle.dense_matmul(a, b, m, k, n)
                exact = (a.astype(np.float64).reshape(m, k) @ b.astype(np.float64).reshape(k, n)).reshape(-1)
                assert np.array_equal(got.astype(np.float64), exact), (m, k, n)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("shape", G.GAPPED_SHAPES)
def test_gapped_positive_strides_are_exact(shape, dtype):
    """native_kernel_tests.rs:243-294."""
    m, k, n = shape
    a, (ars, acs), ao, b, (brs, bcs), bo = G.gapped_strides(m, k, n, dtype)
    va = oracle.View(a, (m, k), (ars, acs), ao)
    vb = oracle.View(b, (k, n), (brs, bcs), bo)
    got = oracle.matmul_reference(va, vb)
    exact = va.to_array().astype(np.float64) @ vb.to_array().astype(np.float64)
    assert np.array_equal(got.astype(np.float64), exact)


@pytest.mark.parametrize("shape", G.F32_BOUNDARY_SHAPES)
def test_f32_ordered_within_reference_bound_of_f64(shape):
    """native_kernel_tests.rs:139-181: |f32 - f64| < 1e-5 (1 + |y|)."""
    m, k, n = shape
    a, b = G.f32_boundary_pair(m, k, n)
    got = oracle.dense_matmul(a.reshape(-1), b.reshape(-1), m, k, n).reshape(m, n).astype(np.float64)
    exp = a.astype(np.float64) @ b.astype(np.float64)
    assert (np.abs(got - exp) < 1e-5 * (1 + np.abs(exp))).all()


def test_dot2_oracle_matches_exact_rational_sum():
    """The compensated oracle reproduces a hard cancellation exactly."""
    a = np.array([[1e16, 1.0, -1e16]], dtype=np.float64)
    b = np.array([[1.0], [1.0], [1.0]], dtype=np.float64)
    out, ab = oracle.gemm_dot2(oracle.View.of(a), oracle.View.of(b), threads=1)
    assert out[0, 0] == 1.0 and ab[0, 0] == 2e16 + 1.0


def test_conv_hand_oracle():
    """neural_vision_tests.rs:29-46 (and its reversed view)."""
    c = KATS["conv_hand"]
    x = np.asarray(c["x"]["values"], dtype=np.float64).reshape(c["x"]["dims"])
    w = np.asarray(c["w"]["values"], dtype=np.float64).reshape(c["w"]["dims"])
    assert oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w)).reshape(-1).tolist() == c["out"]
    # reverse_axis(3): stride -1 on the last axis, origin at the last column.
    xr = oracle.View(x.reshape(-1), (1, 1, 3, 3), (9, 3, 3, -1), 2)
    assert oracle.conv2d_reference(xr, oracle.View.of(w)).reshape(-1).tolist() == c["out_x_reversed_axis3"]


def test_conv_geometry_errors():
    c = KATS["conv_errors"]
    for case in c["cases"]:
        opts = dict(stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1)
        for k, v in case["options"].items():
            opts[k] = tuple(v) if isinstance(v, list) else v
        if "error" in case:
            with pytest.raises(oracle.OracleError) as e:
                oracle.conv_shape(c["x_dims"], c["w_dims"], **opts)
            assert e.value.kind == case["error"]
        else:
            assert oracle.conv_shape(c["x_dims"], c["w_dims"], **opts) == case["out_dims"]


@pytest.mark.parametrize("options", G.CONV_OPTIONS, ids=["default", "grouped_dilated_padded"])
def test_conv_reference_matches_compensated(options):
    """native_kernel_tests.rs:201-241 tolerance 1e-13 (1 + |y|)."""
    x, w = G.conv_inputs(4, options["groups"])
    ref = oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w), **options)
    d2, _ = oracle.conv2d_dot2(oracle.View.of(x), oracle.View.of(w), **options)
    assert (np.abs(ref - d2) < 1e-13 * (1 + np.abs(d2))).all()


def test_softmax_known_answers():
    s = KATS["softmax"]
    x = np.array([[1000.0, 1001.0]])
    y = oracle.softmax_temperature(x, -1, 2.0)
    assert abs(y[0, 1] - 1.0 / (1.0 + math.exp(-0.5))) < 1e-15
    huge = np.array([2.0e38, 2.0e38], dtype=np.float32)
    assert oracle.softmax_temperature(huge, -1, 0.001).tolist() == s[1]["out"]
    mx = np.finfo(np.float64).max
    y = oracle.softmax_temperature(np.array([mx, -mx]), 0, mx)
    e = 1.0 / (1.0 + math.exp(-2.0))
    assert abs(y[0] - e) < 1e-14 and abs(y[1] - (1 - e)) < 1e-14
    for t in (0.0, -1.0, float("nan"), float("inf")):
        with pytest.raises(oracle.OracleError):
            oracle.softmax_temperature(x, 1, t)


def test_plain_softmax_known_answers():
    """ops_expansion_tests.rs:373-386 and :405-418 (values quoted there)."""
    x = np.array([[1000.0, 1001.0, 1002.0], [-1000.0, -1000.0, -1000.0]])
    y = oracle.softmax(x, -1).reshape(-1)
    for got, want, tol in zip(y, [0.09003057317, 0.24472847105, 0.66524095577, 1 / 3],
                              [1e-9, 1e-9, 1e-9, 1e-12]):
        assert abs(got - want) < tol
    with pytest.raises(oracle.OracleError) as e:
        oracle.softmax(np.array([1.0, np.nan]), 0)
    assert e.value.kind == "NonFiniteInput"
    assert e.value.fields == {"operation": "softmax", "indices": [1]}
    assert oracle.softmax(np.zeros((0, 4)), 1).shape == (0, 4)
    with pytest.raises(oracle.OracleError) as e:
        oracle.softmax(np.zeros(()), 0)
    assert e.value.kind == "AxisOutOfBounds"


def test_softmax_first_nonfinite_in_scan_order():
    x = np.zeros((3, 4, 5))
    x[2, 1, 3] = np.inf
    x[1, 3, 0] = np.nan
    with pytest.raises(oracle.OracleError) as e:
        oracle.softmax_temperature(x, 1, 1.0)
    # rows are the (axis-0, axis-2) pairs in C order; (1, *, 0) precedes (2, *, 3)
    assert e.value.fields["indices"] == [1, 3, 0]


def test_splitmix64_published_vector_and_numpy_generator():
    hexes = KATS["splitmix64_seed0"]["first_outputs_hex"]
    state = 0
    for h in hexes:
        v, state = oracle.splitmix_next(state)
        assert v == int(h, 16)
    assert np.array_equal(rng.splitmix_block(0, 0, 3), np.array([int(h, 16) for h in hexes], dtype=np.uint64))
    for seed in (0, 5, 2**63 + 11):
        assert np.array_equal(rng.uniform(seed, 4099, -1.0, 1.0), oracle.uniform(seed, 4099, -1.0, 1.0))
        assert np.array_equal(rng.uniform(seed, 777, -3.0, 2.0, np.float64),
                              oracle.uniform(seed, 777, -3.0, 2.0, np.float64))


def test_normal_generator_moments():
    z = rng.normal(1, 200001)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    assert np.isfinite(z).all()


def test_parallel_ordered_equals_serial():
    a = rng.uniform(3, 129 * 67, -1, 1).reshape(129, 67)
    b = rng.uniform(4, 67 * 33, -1, 1).reshape(67, 33)
    ser = oracle.dense_matmul(a.reshape(-1), b.reshape(-1), 129, 67, 33).reshape(129, 33)
    par = oracle.gemm_ordered_par(oracle.View.of(a), oracle.View.of(b), threads=4)
    assert np.array_equal(ser, par)


def test_conv2d_backward_oracle_central_differences():
    """grouped_dilated_padded_convolution_gradients (neural_vision_tests.rs:46-79)
    on the oracle's restatement of conv2d_backward (neural.rs:379-430)."""
    def generated(dims):
        n = int(np.prod(dims))
        return ((np.arange(n) * 7 % 19 - 9.0) / 10.0).reshape(dims)
    x, w = generated((1, 2, 4, 5)), generated((2, 1, 2, 2))
    o = dict(groups=2, padding=(1, 1), stride=(2, 1), dilation=(2, 1))
    y = oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w), **o)
    dx, dw = oracle.conv2d_backward(oracle.View.of(x), oracle.View.of(w), y, **o)

    def objective(xx, ww):
        yy = oracle.conv2d_reference(oracle.View.of(xx), oracle.View.of(ww), **o)
        return float((yy * yy / 2.0).sum())
    h = 1e-5
    for arr, grad, first in ((x, dx, True), (w, dw, False)):
        flat = grad.reshape(-1)
        for i in range(arr.size):
            p, q = arr.copy().reshape(-1), arr.copy().reshape(-1)
            p[i] += h
            q[i] -= h
            fp = objective(p.reshape(arr.shape), w) if first else objective(x, p.reshape(arr.shape))
            fq = objective(q.reshape(arr.shape), w) if first else objective(x, q.reshape(arr.shape))
            fd = (fp - fq) / (2 * h)
            assert abs(flat[i] - fd) <= 2e-7 * (1 + abs(flat[i]) + abs(fd))


def test_matmul_backward_oracle_known_answers():
    """large_matmul_gradients_use_positive_transpose_kernels_without_changing_the_api
    (autograd_tensor_tests.rs:637-668) on the oracle's VJP restatement."""
    for m, k, n in ((65, 67, 69), (128, 32, 128)):
        a = ((np.arange(m * k) % 23) / 16.0 - 0.5).reshape(m, k)
        b = ((np.arange(k * n) % 13) / 8.0 - 0.5).reshape(k, n)
        da, db = oracle.matmul_backward(a, b, np.ones((m, n)))
        assert np.array_equal(da, np.broadcast_to(b.sum(axis=1), (m, k)))
        assert np.array_equal(db, np.broadcast_to(a.sum(axis=0)[:, None], (k, n)))


def _tape_values(dims, offset):
    """values (kernix/tests/autograd_tensor_tests.rs:7-16)."""
    count = int(np.prod(dims, dtype=np.int64))
    return (((np.arange(count) * 7 + offset) % 19) / 13.0 - 0.6).reshape(dims)


@pytest.mark.parametrize("ad,bd,out", [
    ((3,), (3,), ()), ((3,), (3, 2), (2,)), ((2, 3), (3,), (2,)), ((3,), (2, 3, 2), (2, 2)),
    ((2, 2, 3), (3,), (2, 2)), ((2, 1, 2, 3), (1, 3, 3, 2), (2, 3, 2, 2)),
    ((2, 1, 2, 3), (3, 3, 2), (2, 3, 2, 2)), ((2, 3), (4, 3, 2), (4, 2, 2)),
    ((4, 2, 3), (3, 2), (4, 2, 2)), ((1, 1, 1, 2, 3), (2, 3, 2), (1, 1, 2, 2, 2)),
], ids=lambda v: "x".join(map(str, v)) or "scalar")
def test_matmul_backward_oracle_central_differences(ad, bd, out):
    """matmul_fd over matmul_vector_matrix_and_broadcast_batch_finite_differences
    (autograd_tensor_tests.rs:35-88) on the oracle: its VJP of sum(y * seed)
    against central differences of its ordered forward product (h = 1e-6,
    |a - n| <= 3e-7 (1 + |a| + |n|))."""
    a, b, seed = _tape_values(ad, 1), _tape_values(bd, 5), _tape_values(out, 3)

    def objective(l, r):
        y = oracle.matmul_reference(oracle.View.of(l), oracle.View.of(r))
        assert y.shape == out
        return float((np.asarray(y).reshape(-1) * seed.reshape(-1)).sum())
    da, db = oracle.matmul_backward(a, b, seed)
    h = 1e-6
    for side, (inp, grad) in enumerate(((a, da), (b, db))):
        assert grad.shape == inp.shape
        for i in range(inp.size):
            hi, lo = inp.copy().reshape(-1), inp.copy().reshape(-1)
            hi[i] += h
            lo[i] -= h
            hi, lo = hi.reshape(inp.shape), lo.reshape(inp.shape)
            num = objective(a, hi) - objective(a, lo) if side else objective(hi, b) - objective(lo, b)
            g, n = float(grad.reshape(-1)[i]), num / (2 * h)
            assert abs(g - n) <= 3e-7 * (1 + abs(g) + abs(n)), (side, i, g, n)


def test_tensordot_oracle_known_answers_and_errors():
    """tensordot_contracts_arbitrary_axes_and_empty_k and
    tensordot_scalar_outer_and_zero_result_shapes (ops_completeness_03.rs:
    224-237, 312-323), the reversed-axis case (contraction_paths.rs:90-101),
    agreement with numpy's tensordot on exactly representable values, and the
    errors in the reference order (linalg_extra.rs:164-200)."""
    x = np.array([[1, 2, 3], [4, 5, 6]], np.float64)
    y = np.array([[1, 0, 0], [0, 1, 0], [0, 0, 1], [1, 1, 1]], np.float64)
    assert oracle.tensordot(x, y, [1], [1]).reshape(-1).tolist() == [1, 2, 3, 6, 4, 5, 6, 15]
    z = oracle.tensordot(np.zeros((2, 0)), np.zeros((0, 3)), [1], [0])
    assert z.shape == (2, 3) and not z.any()
    assert oracle.tensordot(np.array(3.0), np.array([5.0, 7.0]), [], []).tolist() == [15.0, 21.0]
    assert oracle.tensordot(np.zeros((0, 2)), np.ones((2, 3)), [1], [0]).shape == (0, 3)
    a = np.arange(6, dtype=np.float64).reshape(2, 3)[:, ::-1]
    assert oracle.tensordot(a, np.ones((3, 2)), [1], [0]).reshape(-1).tolist() == [3.0, 3.0, 12.0, 12.0]
    a = (np.arange(120) % 7 - 3.0).reshape(4, 5, 6)
    b = (np.arange(180) % 5 - 2.0).reshape(6, 5, 6)
    assert np.array_equal(oracle.tensordot(a, b, [2, 1], [0, 1]), np.tensordot(a, b, ([2, 1], [0, 1])))
    cases = {"ContractAxesMismatch": ([1, 2], [0]), "AxisOutOfBounds": ([3], [0]),
             "DuplicateAxis": ([2, -1], [0, 1]), "ContractDimensionMismatch": ([1], [0])}
    for kind, (aa, ba) in cases.items():
        with pytest.raises(oracle.OracleError) as e:
            oracle.tensordot(np.zeros((2, 3, 4)), np.zeros((4, 3)), aa, ba)
        assert e.value.kind == kind
    with pytest.raises(oracle.OracleError) as e:
        oracle.tensordot(np.zeros((2, 3, 4)), np.zeros((4, 3)), [2], [-3])
    assert e.value.fields == {"axis": -3, "rank": 2}
