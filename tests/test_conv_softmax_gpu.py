"""Device conv2d (implicit GEMM, fused im2col) and softmax_temperature parity."""
import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from golden import golden as G

pytestmark = pytest.mark.gpu
KATS = json.loads((Path(__file__).parent / "golden" / "kats.json").read_text())


def to_dev(arr, torch):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def test_conv_hand_oracle(kx, torch_cuda):
    """neural_vision_tests.rs:29-46, including the reversed (negative-stride) input."""
    c = KATS["conv_hand"]
    x = np.asarray(c["x"]["values"], dtype=np.float64).reshape(c["x"]["dims"])
    w = np.asarray(c["w"]["values"], dtype=np.float64).reshape(c["w"]["dims"])
    for dtype in (np.float64, np.float32):
        dx, dw = to_dev(x.astype(dtype), torch_cuda), to_dev(w.astype(dtype), torch_cuda)
        assert kx.conv2d(dx, dw).cpu().numpy().reshape(-1).tolist() == c["out"]
        xr = kx.TensorView(dx.reshape(-1), (1, 1, 3, 3), (9, 3, 3, -1), 2)
        assert kx.conv2d(xr, dw).cpu().numpy().reshape(-1).tolist() == c["out_x_reversed_axis3"]


@pytest.mark.parametrize("options", G.CONV_OPTIONS, ids=["default", "grouped_dilated_padded"])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_conv_matches_reference_across_geometry(kx, torch_cuda, options, dtype):
    """native_kernel_tests.rs:201-241: tiled conv vs conv2d_reference (f64 1e-13;
    f32 against the compensated oracle with the f32 scaled bound)."""
    x, w = G.conv_inputs(4, options["groups"], dtype)
    opts = kx.Conv2dOptions(**options)
    got = kx.conv2d(to_dev(x, torch_cuda), to_dev(w, torch_cuda), opts).cpu().numpy().astype(np.float64)
    ref = oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w), **options).astype(np.float64)
    d2, ab = oracle.conv2d_dot2(oracle.View.of(x), oracle.View.of(w), **options)
    assert got.shape == ref.shape
    if dtype == np.float64:
        assert (np.abs(got - ref) < 1e-13 * (1 + np.abs(ref))).all()
    else:
        assert (np.abs(got - d2) <= 2e-6 * ab + 1e-30).all()
    # reversed last axis of the input (reverse_axis(3))
    n, c, h, wd = x.shape
    xr = kx.TensorView(to_dev(x, torch_cuda).reshape(-1), x.shape, (c * h * wd, h * wd, wd, -1), wd - 1)
    got_r = kx.conv2d(xr, to_dev(w, torch_cuda), opts).cpu().numpy().astype(np.float64)
    ref_r = oracle.conv2d_reference(oracle.View(x, x.shape, (c * h * wd, h * wd, wd, -1), wd - 1),
                                    oracle.View.of(w), **options).astype(np.float64)
    tol = 1e-13 if dtype == np.float64 else 1e-5
    assert (np.abs(got_r - ref_r) < tol * (1 + np.abs(ref_r))).all()


@pytest.mark.parametrize("options", G.CONV_OPTIONS, ids=["default", "grouped_dilated_padded"])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_conv_reference_mode_is_bitwise(kx, torch_cuda, options, dtype):
    """conv2d_reference on the device reproduces the ordered scalar path exactly
    (native_kernel_tests.rs:237-239 asserts this equality for reversed inputs)."""
    x, w = G.conv_inputs(4, options["groups"], dtype)
    opts = kx.Conv2dOptions(**options)
    ref = oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w), **options)
    got = kx.conv2d_reference(to_dev(x, torch_cuda), to_dev(w, torch_cuda), opts).cpu().numpy()
    assert np.array_equal(got, ref)


def test_conv_errors_and_empty(kx, torch_cuda):
    x = torch_cuda.zeros(1, 2, 2, 3, device="cuda")
    w = torch_cuda.zeros(2, 2, 3, 3, device="cuda")
    with pytest.raises(kx.InvalidParameter):
        kx.conv2d(x, w, kx.Conv2dOptions(stride=(0, 1)))
    with pytest.raises(kx.InvalidParameter):
        kx.conv2d(x, w, kx.Conv2dOptions(groups=3))
    assert kx.conv2d(x, w).numel() == 0


def test_conv_nonfinite_weight_in_padding_matches_scalar_path(kx, torch_cuda):
    """A NaN weight tap that only ever lands on padding must not poison the
    output (the reference sends nonfinite data to its ordered scalar path)."""
    x = np.arange(1 * 1 * 4 * 4, dtype=np.float32).reshape(1, 1, 4, 4) / 7.0
    w = np.ones((1, 1, 3, 3), dtype=np.float32)
    w[0, 0, 0, 0] = np.nan
    opts = dict(stride=(3, 3), padding=(1, 1), dilation=(1, 1), groups=1)
    ref = oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w), **opts)
    got = kx.conv2d(to_dev(x, torch_cuda), to_dev(w, torch_cuda), kx.Conv2dOptions(**opts)).cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(got[~np.isnan(got)], ref[~np.isnan(ref)])


def test_conv_medium_igemm_vs_compensated(kx, torch_cuda):
    """A padded 3x3 conv large enough for the 128x128 tile family."""
    from kernix_b200 import rng
    x = rng.uniform(11, 4 * 64 * 28 * 28, -1, 1).reshape(4, 64, 28, 28)
    w = rng.normal(12, 128 * 64 * 9, math.sqrt(2 / 576)).reshape(128, 64, 3, 3)
    opts = dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1)
    got = kx.conv2d(to_dev(x, torch_cuda), to_dev(w, torch_cuda), kx.Conv2dOptions(**opts)).cpu().numpy()
    d2, ab = oracle.conv2d_dot2(oracle.View.of(x), oracle.View.of(w), **opts)
    assert (np.abs(got.astype(np.float64) - d2) <= 2e-6 * ab + 1e-30).all()


# ---------------------------------------------------------------------------
# softmax_temperature
# ---------------------------------------------------------------------------
def test_softmax_known_answers(kx, torch_cuda):
    """softmax_temperature_preserves_extreme_logits (kernix-ops/tests/numeric_dispatch_04.rs:172-190)
    and large_temperature_preserves_finite_logit_differences
    (kernix-ops/tests/qa_extreme_numerics.rs:10-24)."""
    x = to_dev(np.array([[1000.0, 1001.0]]), torch_cuda)
    y = kx.softmax_temperature(x, -1, 2.0).cpu().numpy()
    assert abs(y[0, 1] - 1.0 / (1.0 + math.exp(-0.5))) < 1e-15
    huge = to_dev(np.array([2.0e38, 2.0e38], dtype=np.float32), torch_cuda)
    assert kx.softmax_temperature(huge, -1, 0.001).cpu().numpy().tolist() == [0.5, 0.5]
    mx = np.finfo(np.float64).max
    y = kx.softmax_temperature(to_dev(np.array([mx, -mx]), torch_cuda), 0, mx).cpu().numpy()
    e = 1.0 / (1.0 + math.exp(-2.0))
    assert abs(y[0] - e) < 1e-14 and abs(y[1] - (1 - e)) < 1e-14
    for t in (0.0, -1.0, float("nan"), float("inf")):
        with pytest.raises(kx.InvalidParameter):
            kx.softmax_temperature(x, 1, t)
    with pytest.raises(kx.AxisOutOfBounds) as err:
        kx.softmax_temperature(x, 2, 1.0)
    assert (err.value.axis, err.value.rank) == (2, 2)


def softmax_truth(x, axis, t):
    """Extended-precision softmax of the same inputs (the accuracy yardstick)."""
    xl = x.astype(np.longdouble)
    m = xl.max(axis=axis, keepdims=True)
    e = np.exp((xl - m) / np.longdouble(t))
    return e / e.sum(axis=axis, keepdims=True)


def softmax_tol(dtype, length):
    """Relative bound: exp and division ulps plus a tree-sum term log2(len)."""
    eps = np.finfo(dtype).eps
    return (8 + 2 * math.log2(max(length, 2))) * eps


def softmax_tol_cond(x, axis, t):
    """softmax_tol plus the conditioning of exp: rounding the argument
    d = (x - max) / T to the working precision perturbs exp(d) by |d| ulps,
    for the reference as much as for any implementation."""
    xl = x.astype(np.longdouble)
    d = np.abs((xl - xl.max(axis=axis, keepdims=True)) / np.longdouble(t))
    return softmax_tol(x.dtype, x.shape[axis]) + 2 * d.astype(np.float64) * np.finfo(x.dtype).eps


@pytest.mark.parametrize("shape,axis", [((7, 11), -1), ((3, 5, 300), 2), ((4, 2048), -1), ((2, 3, 4, 5), 1),
                                        ((3, 5000), 1), ((6, 33), 0), ((1, 1), 0)])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_softmax_matches_oracle(kx, torch_cuda, shape, axis, dtype):
    from kernix_b200 import rng
    x = rng.normal(21, int(np.prod(shape)), 3.0, dtype).reshape(shape)
    exp = oracle.softmax_temperature(x, axis, 1.7)
    got = kx.softmax_temperature(to_dev(x, torch_cuda), axis, 1.7).cpu().numpy()
    truth = softmax_truth(x, axis, 1.7)
    tol = softmax_tol(dtype, shape[axis])
    assert (np.abs(got - truth) <= tol * np.abs(truth) + np.finfo(dtype).tiny).all()
    # the oracle (sequential sum) obeys the sequential bound len * eps
    seq = (8 + shape[axis]) * np.finfo(dtype).eps
    assert (np.abs(exp - truth) <= seq * np.abs(truth) + np.finfo(dtype).tiny).all()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_softmax_block_rows_paths(kx, torch_cuda, dtype):
    """Long contiguous rows (one block per row): reciprocal path, the
    divide-first fallback for overflowing differences, a huge temperature
    (subnormal reciprocal), outer dims that do not nest, and +inf rows."""
    from kernix_b200 import rng
    torch = torch_cuda
    x = rng.normal(31, 6 * 4 * 2048, 2.0, dtype).reshape(6, 4, 2048)
    for t in (0.37, 11.3, 1e38 if dtype == np.float32 else 1e307):
        got = kx.softmax_temperature(to_dev(x, torch), -1, t).cpu().numpy()
        assert kx.handle(0).last_kernel == "softmax_rows_block_vec"
        truth = softmax_truth(x, -1, t)
        assert (np.abs(got - truth) <= softmax_tol_cond(x, -1, t) * np.abs(truth) + np.finfo(dtype).tiny).all()
    # (x - max) overflows: the reference divides first, x/T - max/T
    big = np.finfo(dtype).max * 0.75
    y = np.zeros((3, 2048), dtype=dtype)
    y[:, ::2] = big
    y[:, 1::2] = -big
    y[1, 7] = big * 0.5
    got = kx.softmax_temperature(to_dev(y, torch), -1, big).cpu().numpy()
    truth = softmax_truth(y, -1, big)   # no overflow in extended precision: same value as divide-first
    assert (np.abs(got - truth) <= softmax_tol(dtype, 2048) * np.abs(truth) + np.finfo(dtype).tiny).all()
    exp = oracle.softmax_temperature(y, -1, big)   # sequential sum: the looser len * eps bound
    assert (np.abs(exp - truth) <= (8 + 2048) * np.finfo(dtype).eps * np.abs(truth)).all()
    # outer dims that do not collapse into one row stride: (4, 6, 2048) view of a (6, 4, 2048) buffer
    src = to_dev(x, torch).permute(1, 0, 2)
    got = kx.softmax_temperature(src, 2, 0.8).cpu().numpy()
    xt = np.transpose(x, (1, 0, 2))
    truth = softmax_truth(xt, 2, 0.8)
    assert (np.abs(got - truth) <= softmax_tol_cond(xt, 2, 0.8) * np.abs(truth) + np.finfo(dtype).tiny).all()
    # +inf alone in a long row, then NaN before it in a later row: first index wins
    z = np.zeros((5, 1536), dtype=dtype)
    z[3, 1000] = np.inf
    z[4, 2] = np.nan
    with pytest.raises(kx.NonFiniteInput) as ge:
        kx.softmax_temperature(to_dev(z, torch), -1, 1.0)
    assert ge.value.indices == [3, 1000]


def test_softmax_strided_input(kx, torch_cuda):
    """A transposed (non-contiguous) source with the reduction on its middle axis."""
    from kernix_b200 import rng
    base = rng.normal(5, 4 * 6 * 9).reshape(4, 6, 9)
    src = to_dev(base, torch_cuda).permute(2, 0, 1)     # dims (9,4,6), strides (1,54,9)
    truth = softmax_truth(np.transpose(base, (2, 0, 1)), 1, 0.5)
    got = kx.softmax_temperature(src, 1, 0.5).cpu().numpy()
    assert (np.abs(got - truth) <= softmax_tol(np.float32, 4) * np.abs(truth) + 1e-37).all()


def test_softmax_first_nonfinite_indices(kx, torch_cuda):
    x = np.zeros((3, 4, 5), dtype=np.float32)
    x[2, 1, 3] = np.inf
    x[1, 3, 0] = np.nan
    with pytest.raises(oracle.OracleError) as oe:
        oracle.softmax_temperature(x, 1, 1.0)
    with pytest.raises(kx.NonFiniteInput) as ge:
        kx.softmax_temperature(to_dev(x, torch_cuda), 1, 1.0)
    assert ge.value.indices == oe.value.fields["indices"] == [1, 3, 0]
    y = np.zeros((2, 2048), dtype=np.float32)
    y[1, 5] = -np.inf
    y[1, 1000] = np.nan
    with pytest.raises(kx.NonFiniteInput) as ge:
        kx.softmax_temperature(to_dev(y, torch_cuda), -1, 1.0)
    assert ge.value.indices == [1, 5]


def test_status_words_do_not_alias(kx, torch_cuda):
    """softmax's nonfinite record, conv's weight flag and the device status word
    live in separate words: neither operation reads as an expired wait."""
    h = kx.handle(0)
    x = to_dev(np.zeros((4, 8), dtype=np.float32), torch_cuda)
    kx.softmax_temperature(x, -1, 1.0)
    h.synchronize()
    bad = x.clone()
    bad[1, 2] = float("inf")
    with pytest.raises(kx.NonFiniteInput):
        kx.softmax_temperature(bad, -1, 1.0)
    h.synchronize()
    w = torch_cuda.ones(2, 1, 3, 3, device="cuda")
    w[0, 0, 0, 0] = float("nan")
    kx.conv2d(torch_cuda.ones(1, 1, 5, 5, device="cuda"), w, kx.Conv2dOptions(padding=(1, 1)))
    h.synchronize()


# ---------------------------------------------------------------------------
# plain softmax (ops/math.rs:398-465, 531-536)
# ---------------------------------------------------------------------------
def test_plain_softmax_known_answers(kx, torch_cuda):
    """ops_expansion_tests.rs:373-418: large logits along both axes, F-order
    views, the nonfinite error with operation "softmax", empty and scalar."""
    x = to_dev(np.array([[1000.0, 1001.0, 1002.0], [-1000.0, -1000.0, -1000.0]]), torch_cuda)
    y = kx.softmax(x, -1).cpu().numpy().reshape(-1)
    for got, want, tol in zip(y, [0.09003057317, 0.24472847105, 0.66524095577, 1 / 3, 1 / 3, 1 / 3],
                              [1e-9, 1e-9, 1e-9, 1e-12, 1e-12, 1e-12]):
        assert abs(got - want) < tol
    f = to_dev(np.array([[0.0, 1.0, 2.0], [3.0, 4.0, 5.0]], dtype=np.float32), torch_cuda)
    fview = kx.TensorView(f.reshape(-1), (2, 3), (1, 2))       # Order::F storage [0,3,1,4,2,5]
    y = kx.softmax(fview, 0).cpu().numpy()
    assert (np.abs(y.sum(axis=0) - 1) < 1e-6).all() and (y[0] < y[1]).all()
    with pytest.raises(kx.NonFiniteInput) as ge:
        kx.softmax(to_dev(np.array([1.0, np.nan]), torch_cuda), 0)
    assert ge.value.indices == [1] and ge.value.operation == "softmax"
    assert tuple(kx.softmax(torch_cuda.zeros(0, 4, device="cuda", dtype=torch_cuda.float64), 1).shape) == (0, 4)
    with pytest.raises(kx.AxisOutOfBounds):
        kx.softmax(torch_cuda.zeros((), device="cuda", dtype=torch_cuda.float64), 0)


@pytest.mark.parametrize("shape,axis", [((7, 11), -1), ((4, 2048), -1), ((3, 5000), 1), ((6, 33), 0)])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_plain_softmax_matches_oracle(kx, torch_cuda, shape, axis, dtype):
    from kernix_b200 import rng
    x = rng.normal(23, int(np.prod(shape)), 3.0, dtype).reshape(shape)
    exp = oracle.softmax(x, axis)
    got = kx.softmax(to_dev(x, torch_cuda), axis).cpu().numpy()
    truth = softmax_truth(x, axis, 1.0)
    assert (np.abs(got - truth) <= softmax_tol_cond(x, axis, 1.0) * np.abs(truth) + np.finfo(dtype).tiny).all()
    seq = (8 + shape[axis]) * np.finfo(dtype).eps
    assert (np.abs(exp - truth) <= seq * np.abs(truth) + np.finfo(dtype).tiny).all()
    # the same values as softmax_temperature at temperature 1 (execution_tests.rs:33-49 pins
    # the fast and indexed paths to each other; here the plain and tempered entries)
    same = kx.softmax_temperature(to_dev(x, torch_cuda), axis, 1.0).cpu().numpy()
    assert np.array_equal(got, same)


def test_plain_softmax_first_nonfinite_matches_oracle(kx, torch_cuda):
    x = np.zeros((7, 11), dtype=np.float64)
    x[3, 7] = np.nan
    x[5, 1] = np.inf
    with pytest.raises(oracle.OracleError) as oe:
        oracle.softmax(x, -1)
    with pytest.raises(kx.NonFiniteInput) as ge:
        kx.softmax(to_dev(x, torch_cuda), -1)
    assert ge.value.indices == oe.value.fields["indices"] == [3, 7]
    assert ge.value.operation == oe.value.fields["operation"] == "softmax"
