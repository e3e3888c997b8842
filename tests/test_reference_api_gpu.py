"""More of the reference's own tests on the device path.

* batched_forward_matmul (kernix/tests/api_ergonomics.rs:25-31);
* explicit_layout_policy_and_reusable_output (api_ergonomics.rs:105-117):
  ordered matmul_into into a reused output, through a context made from
  ``[cpu] ordered_matmul = true``;
* matmul_and_dense_shared_parameter_gradients and
  convolution_and_pooling_gradients (kernix/tests/autograd_tests.rs:142-167):
  the backward products against central differences of sum(y * seed), seed_i =
  0.3 + 0.11 i, h = 1e-6, |analytic - numeric| < 2e-6 (1 + |a| + |n|)
  (autograd_tests.rs:7-12, 55-100);
* the reconstruction check of cholesky_layouts_scales_branch_boundaries
  (kernix-ops/tests/factorization_regressions.rs:39-61): matmul_reference(L,
  L^T view) at scales 1e-200, 1, 1e200 -- bit for bit the oracle's ordered
  product, and within 1e-12 * scale of the original matrix;
* the dense arm of Matrix::matmul with signed-stride vectors and views
  (kernix-ops/tests/sparse_tests.rs:134-200), against matmul_reference;
* the matmul cases of kernix/tests/autograd_tensor_tests.rs:35-217: vector,
  matrix and broadcast-batch VJPs against central differences, exactly zero
  gradients of zero extents, a shared operand on both sides, reversed and
  transposed views with a constant side;
* the direct-memory and reversed-axis products of
  kernix-ops/tests/numeric_dispatch_04.rs:116-152;
* the reconstruction products of kernix-ops/tests/linalg_tests.rs:13-57,
  100-137 (LU, inverse, QR, least squares) with host-computed factors.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def dev(torch, arr):
    return torch.from_numpy(np.array(arr, order="C")).cuda()


def test_batched_forward_matmul(kx, torch_cuda):
    torch = torch_cuda
    c = kx.matmul(torch.ones(2, 2, 3, device="cuda"), torch.ones(3, 2, device="cuda"))
    assert tuple(c.shape) == (2, 2, 2) and c.cpu().numpy().reshape(-1).tolist() == [3.0] * 8


def test_ordered_matmul_into_reuses_the_output(kx, torch_cuda):
    torch = torch_cuda
    column_major = np.array([1.0, 3.0, 2.0, 4.0]).reshape(2, 2).T      # Order::F [[1, 2], [3, 4]]
    a = dev(torch, np.ascontiguousarray(column_major))
    out = torch.zeros(2, 2, dtype=torch.float64, device="cuda")
    pointer = out.data_ptr()
    ctx = kx.Context.new(kx.Config.from_toml("[cpu]\nordered_matmul = true"))
    ctx.cuda().matmul_into(a, a, out)
    assert out.cpu().numpy().reshape(-1).tolist() == [7.0, 10.0, 15.0, 22.0]
    assert out.data_ptr() == pointer


def _seed(n):
    return 0.3 + 0.11 * np.arange(n)


def _near(a, b):
    assert abs(a - b) < 2e-6 * (1.0 + abs(a) + abs(b)), (a, b)


def _check_binary(forward, backward, left, right):
    """binary (autograd_tests.rs:55-100): the analytic gradients of
    sum(forward(l, r) * seed) against central differences."""
    out = forward(left, right)
    seed = _seed(out.size).reshape(out.shape)
    gl, gr = backward(left, right, seed)

    def evaluate(l, r):
        return float((forward(l, r).reshape(-1) * _seed(out.size)).sum())
    h = 1e-6
    for which, (inp, grad) in enumerate(((left, gl), (right, gr))):
        for i in range(inp.size):
            hi, lo = inp.copy().reshape(-1), inp.copy().reshape(-1)
            hi[i] += h
            lo[i] -= h
            hi, lo = hi.reshape(inp.shape), lo.reshape(inp.shape)
            num = (evaluate(hi, right) - evaluate(lo, right)) if which == 0 else \
                (evaluate(left, hi) - evaluate(left, lo))
            _near(float(grad.reshape(-1)[i]), num / (2 * h))


def test_matmul_gradients_against_central_differences(kx, torch_cuda):
    torch = torch_cuda
    left = np.array([0.2, 0.4, 0.6, 0.8, 1.0, 1.2]).reshape(2, 3)
    right = np.array([0.1, 0.3, 0.5, 0.7, 0.9, 1.1]).reshape(3, 2)

    def forward(a, b):
        return kx.matmul(dev(torch, a), dev(torch, b)).cpu().numpy()

    def backward(a, b, g):
        ga, gb = kx.matmul_backward(dev(torch, a), dev(torch, b), dev(torch, g))
        return ga.cpu().numpy(), gb.cpu().numpy()
    _check_binary(forward, backward, left, right)


def test_conv2d_gradients_against_central_differences(kx, torch_cuda):
    torch = torch_cuda
    x = np.array([0.1, 0.3, 0.7, 0.4, 0.2, 0.8, 0.9, 0.6, 0.5]).reshape(1, 1, 3, 3)
    w = np.array([0.2, 0.4, 0.7, 0.9]).reshape(1, 1, 2, 2)

    def forward(a, b):
        return kx.conv2d(dev(torch, a), dev(torch, b)).cpu().numpy()

    def backward(a, b, g):
        gx, gw = kx.conv2d_backward(dev(torch, a), dev(torch, b), dev(torch, g))
        return gx.cpu().numpy(), gw.cpu().numpy()
    _check_binary(forward, backward, x, w)


def _spd(n, scale, seed):
    rs = np.random.default_rng(seed)
    m = rs.uniform(-1, 1, (n, n))
    return (m @ m.T + n * np.eye(n)) * scale


@pytest.mark.parametrize("n", [1, 7, 31, 64, 96, 97, 128])
@pytest.mark.parametrize("scale", [1e-200, 1.0, 1e200])
def test_cholesky_reconstruction_in_ordered_mode(kx, torch_cuda, n, scale):
    torch = torch_cuda
    a = _spd(n, scale, n)
    low = np.linalg.cholesky(a)
    want = oracle.matmul_reference(oracle.View.of(low), oracle.View(low, (n, n), (1, n)))
    dl = dev(torch, low)
    got = kx.matmul_reference(dl, dl.transpose(0, 1)).cpu().numpy()
    assert np.array_equal(got, want)
    assert (np.abs((got - a) / scale) < 1e-12 * n).all()


def _sparse_matrix(m, n, shift):
    """matrix (kernix-ops/tests/sparse_tests.rs:5-19)."""
    p = np.arange(m * n)
    return np.where((p * 7 + shift) % 11 < 2, (p % 13) / 8.0 - 0.5, 0.0).reshape(m, n)


def _close(x, y):
    """assert_close (sparse_tests.rs:20-25)."""
    assert x.shape == y.shape
    assert (np.abs(x - y) < 2e-12 * (1.0 + np.abs(y))).all()


@pytest.mark.parametrize("m,k,n", [(0, 3, 4), (3, 0, 4), (3, 4, 0), (1, 1, 1), (3, 5, 4), (7, 9, 13),
                                   (17, 31, 9), (65, 33, 7)])
def test_dense_matrix_products_and_reversed_vectors(kx, torch_cuda, m, k, n):
    """The dense arm of Matrix::matmul and the signed-stride vector products of
    all_four_storage_products_and_signed_stride_vectors_match_independent_oracles
    (sparse_tests.rs:134-179), against matmul_reference."""
    torch = torch_cuda
    a, b = _sparse_matrix(m, k, 1), _sparse_matrix(k, n, 2)
    want = oracle.matmul_reference(oracle.View.of(a), oracle.View.of(b))
    _close(kx.matmul(dev(torch, a), dev(torch, b)).cpu().numpy(), want)
    v = np.arange(k) / 16.0 - 0.5
    buf = dev(torch, v)
    rev = kx.TensorView(buf, (k,), (-1,), max(k - 1, 0))                 # reverse_axis(0)
    want_v = oracle.matmul_reference(oracle.View.of(a), oracle.View(v, (k,), (-1,), max(k - 1, 0)))
    _close(kx.matmul(dev(torch, a), rev).cpu().numpy(), want_v)


def test_transposed_and_reversed_dense_operands(kx, torch_cuda):
    """transpose_csc_and_reversed_dense_rhs_remain_zero_copy_and_correct
    (sparse_tests.rs:181-200), dense operands: a^T times b with axis 0
    reversed, and a times b with axis 1 reversed, as views."""
    torch = torch_cuda
    a = _sparse_matrix(7, 9, 3)
    b = _sparse_matrix(7, 5, 4)
    at = kx.TensorView(dev(torch, a).reshape(-1), (9, 7), (1, 9), 0)
    brev = kx.TensorView(dev(torch, b).reshape(-1), (7, 5), (-5, 1), 6 * 5)
    want = oracle.matmul_reference(oracle.View(a, (9, 7), (1, 9)), oracle.View(b, (7, 5), (-5, 1), 30))
    _close(kx.matmul(at, brev).cpu().numpy(), want)
    b2 = _sparse_matrix(9, 5, 2)
    b2rev = kx.TensorView(dev(torch, b2).reshape(-1), (9, 5), (5, -1), 4)
    want2 = oracle.matmul_reference(oracle.View.of(a), oracle.View(b2, (9, 5), (5, -1), 4))
    _close(kx.matmul(dev(torch, a), b2rev).cpu().numpy(), want2)


def _values(dims, offset):
    """values (kernix/tests/autograd_tensor_tests.rs:7-16)."""
    count = int(np.prod(dims, dtype=np.int64))
    return (((np.arange(count) * 7 + offset) % 19) / 13.0 - 0.6).reshape(dims)


def _near_tape(a, b):
    """near (autograd_tensor_tests.rs:20-25)."""
    assert abs(a - b) <= 3e-7 * (1.0 + abs(a) + abs(b)), (a, b)


@pytest.mark.parametrize("ad,bd,out", [
    ((3,), (3,), ()), ((3,), (3, 2), (2,)), ((2, 3), (3,), (2,)), ((3,), (2, 3, 2), (2, 2)),
    ((2, 2, 3), (3,), (2, 2)), ((2, 1, 2, 3), (1, 3, 3, 2), (2, 3, 2, 2)),
    ((2, 1, 2, 3), (3, 3, 2), (2, 3, 2, 2)), ((2, 3), (4, 3, 2), (4, 2, 2)),
    ((4, 2, 3), (3, 2), (4, 2, 2)), ((1, 1, 1, 2, 3), (2, 3, 2), (1, 1, 2, 2, 2)),
], ids=lambda v: "x".join(map(str, v)) or "scalar")
def test_matmul_vjp_vector_and_broadcast_batch_finite_differences(kx, torch_cuda, ad, bd, out):
    """matmul_fd over matmul_vector_matrix_and_broadcast_batch_finite_differences
    (autograd_tensor_tests.rs:35-88): the VJP of sum(y * seed) against central
    differences (h = 1e-6) of the device forward product, f64."""
    torch = torch_cuda
    a, b, seed = _values(ad, 1), _values(bd, 5), _values(out, 3)

    def objective(l, r):
        y = kx.matmul(dev(torch, l), dev(torch, r)).cpu().numpy()
        assert y.shape == out
        return float((y.reshape(-1) * seed.reshape(-1)).sum())
    da, db = kx.matmul_backward(dev(torch, a), dev(torch, b), dev(torch, seed))
    h = 1e-6
    for side, (inp, grad) in enumerate(((a, da.cpu().numpy()), (b, db.cpu().numpy()))):
        assert grad.shape == inp.shape
        for i in range(inp.size):
            hi, lo = inp.copy().reshape(-1), inp.copy().reshape(-1)
            hi[i] += h
            lo[i] -= h
            hi, lo = hi.reshape(inp.shape), lo.reshape(inp.shape)
            num = objective(a, hi) - objective(a, lo) if side else objective(hi, b) - objective(lo, b)
            _near_tape(float(grad.reshape(-1)[i]), num / (2 * h))


@pytest.mark.parametrize("ad,bd,out", [
    ((1, 2, 3), (0, 3, 4), (0, 2, 4)), ((0, 2, 3), (1, 3, 4), (0, 2, 4)), ((3,), (0, 3, 4), (0, 4)),
    ((0, 2, 3), (3,), (0, 2)), ((2, 0), (0, 3), (2, 3)), ((0, 3), (3, 2), (0, 2)),
    ((2, 3), (3, 0), (2, 0)), ((0,), (0,), ()), ((0,), (2, 0, 3), (2, 3)), ((2, 3, 0), (0,), (2, 3)),
], ids=lambda v: "x".join(map(str, v)) or "scalar")
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_matmul_zero_extents_have_exact_shaped_zero_gradients(kx, torch_cuda, ad, bd, out, dtype):
    """matmul_zero_extents_have_exact_shaped_zero_gradients
    (autograd_tensor_tests.rs:89-116): the gradients of sum(y) keep their
    operands' shapes and are exactly zero."""
    torch = torch_cuda
    a, b = _values(ad, 1).astype(dtype), _values(bd, 2).astype(dtype)
    y = kx.matmul(dev(torch, a), dev(torch, b))
    assert tuple(y.shape) == out
    da, db = kx.matmul_backward(dev(torch, a), dev(torch, b), dev(torch, np.ones(out, dtype)))
    for g, dims in ((da, ad), (db, bd)):
        g = g.cpu().numpy()
        assert g.shape == dims and (g == 0).all()


def test_matmul_shared_operand_and_seeded_dot(kx, torch_cuda):
    """matmul_shared_dag_repeated_backward_and_seeded_dot
    (autograd_tensor_tests.rs:117-155): d sum(x.x + x.x) / dx is the sum of both
    VJP sides with seed 2, equal to 2 (row j of x summed + column i of x
    summed) per batch, and the same on a repeated pass; d (v.v) / dv with seed
    2 is 4 v."""
    torch = torch_cuda
    x = _values((2, 2, 2), 1)
    dx = dev(torch, x)
    g = dev(torch, np.full((2, 2, 2), 2.0))
    first = sum(t.cpu().numpy() for t in kx.matmul_backward(dx, dx, g))
    second = sum(t.cpu().numpy() for t in kx.matmul_backward(dx, dx, g))
    for batch in range(2):
        a = x[batch].reshape(-1)
        for i in range(2):
            for j in range(2):
                _near_tape(first[batch, i, j], 2.0 * (a[j * 2] + a[j * 2 + 1] + a[i] + a[2 + i]))
    assert np.array_equal(first, second)
    v = dev(torch, np.array([1.0, 2.0, 3.0]))
    gv = sum(t.cpu().numpy() for t in kx.matmul_backward(v, v, dev(torch, np.array(2.0))))
    assert gv.tolist() == [4.0, 8.0, 12.0]


def test_matmul_transposed_reversed_inputs_and_constant_side(kx, torch_cuda):
    """matmul_transposed_reversed_inputs_and_constants
    (autograd_tensor_tests.rs:178-217): a [2,2,3] with axis 2 reversed times
    b [2,4,3] with axes 1 and 2 swapped, both zero-copy views; the product
    against matmul_reference, and d sum(permute(y)) / da = ones[2,2,4] . b
    with the constant side's gradient not computed."""
    torch = torch_cuda
    a, b = _values((2, 2, 3), 1), _values((2, 4, 3), 2)
    av = kx.TensorView(dev(torch, a).reshape(-1), (2, 2, 3), (6, 3, -1), 2)
    bv = kx.TensorView(dev(torch, b).reshape(-1), (2, 3, 4), (12, 1, 3), 0)
    oa, ob = oracle.View(a, (2, 2, 3), (6, 3, -1), 2), oracle.View(b, (2, 3, 4), (12, 1, 3), 0)
    y = kx.matmul(av, bv).cpu().numpy()
    want = oracle.matmul_reference(oa, ob)
    for p, q in zip(y.reshape(-1), want.reshape(-1)):
        _near_tape(float(p), float(q))
    da, db = kx.matmul_backward(av, bv, dev(torch, np.ones((2, 2, 4))), need_b=False)
    assert db is None
    want_da = oracle.matmul_reference(oracle.View.of(np.ones((2, 2, 4))), oracle.View.of(b))
    for p, q in zip(da.cpu().numpy().reshape(-1), want_da.reshape(-1)):
        _near_tape(float(p), float(q))


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_direct_memory_and_reversed_matrix_products(kx, torch_cuda, dtype):
    """contiguous_matrix_mult_uses_direct_memory, contiguous_dot_uses_direct_memory
    and noncontiguous_matrix_falls_back_to_checked_indexing
    (kernix-ops/tests/numeric_dispatch_04.rs:116-152): exact small-integer
    answers for the contiguous, the dot and the axis-1-reversed operand."""
    torch = torch_cuda
    a = np.arange(1, 7, dtype=dtype).reshape(2, 3)
    b = np.arange(7, 13, dtype=dtype).reshape(3, 2)
    assert kx.matmul(dev(torch, a), dev(torch, b)).cpu().numpy().reshape(-1).tolist() == [58, 64, 139, 154]
    d = kx.matmul(dev(torch, np.array([1, 2, 3], dtype)), dev(torch, np.array([4, 5, 6], dtype)))
    assert tuple(d.shape) == () and float(d.cpu()) == 32.0
    rev = kx.TensorView(dev(torch, a).reshape(-1), (2, 3), (3, -1), 2)
    assert kx.matmul(rev, dev(torch, b)).cpu().numpy().reshape(-1).tolist() == [50, 56, 131, 146]


def _near12(a, b):
    """near (kernix-ops/tests/linalg_tests.rs:7-12)."""
    assert abs(a - b) <= 2e-12 * (1.0 + abs(a) + abs(b)), (a, b)


def test_decomposition_reconstruction_products(kx, torch_cuda):
    """The matmul checks of linalg_tests.rs:13-57 and 100-137 on the device,
    with the factors computed on the host: P A = L U, A inverse(A) = I, Q R = A
    for a tall and a wide matrix, Q^T Q = I through Q's transposed view, and
    the least-squares normal equations A^T (A x - b) = 0 with A^T a view."""
    import scipy.linalg as sl
    torch = torch_cuda

    def mm(x, y):
        return kx.matmul(x if isinstance(x, kx.TensorView) else dev(torch, x),
                         y if isinstance(y, kx.TensorView) else dev(torch, y)).cpu().numpy()
    a = np.array([0.0, 2.0, 1.0, 1.0, 1.0, 0.0, 2.0, 0.0, 1.0]).reshape(3, 3)
    p, low, up = sl.lu(a)                              # a = p @ low @ up
    prod = mm(low, up)
    pa = p.T @ a
    for i in range(3):
        for j in range(3):
            _near12(prod[i, j], pa[i, j])
    ident = mm(a, np.linalg.inv(a))
    for i in range(3):
        for j in range(3):
            _near12(ident[i, j], 1.0 if i == j else 0.0)
    tall = np.array([1.0, 0.0, 1.0, 1.0, 1.0, 2.0]).reshape(3, 2)
    for mat in (tall, np.arange(1.0, 7.0).reshape(2, 3)):
        q, r = np.linalg.qr(mat)
        for x, y in zip(mm(q, r).reshape(-1), mat.reshape(-1)):
            _near12(x, y)
    q, r = np.linalg.qr(tall)
    qbuf = dev(torch, q).reshape(-1)
    qt = kx.TensorView(qbuf, (2, 3), (1, 2), 0)         # q.transpose(), zero-copy
    for x, y in zip(mm(qt, kx.TensorView(qbuf, (3, 2), (2, 1), 0)).reshape(-1), [1.0, 0.0, 0.0, 1.0]):
        _near12(x, y)
    x_ls = np.array([7.0 / 6.0, 0.5])
    b = np.array([1.0, 2.0, 2.0])
    residual = mm(tall, x_ls) - b
    _near12(float(np.linalg.norm(residual)), (1.0 / 6.0) ** 0.5)
    at = kx.TensorView(dev(torch, tall).reshape(-1), (2, 3), (1, 2), 0)
    _near12(float(np.linalg.norm(mm(at, residual))), 0.0)
