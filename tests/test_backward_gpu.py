"""Backward products on the device against the reference's own tests and the oracle.

* matmul VJP: large_matmul_gradients_use_positive_transpose_kernels_without_
  changing_the_api (kernix/tests/autograd_tensor_tests.rs:637-668, exact
  dyadic sums), every matmul geometry of Tape::matmul (autograd.rs:622-690:
  vectors, batches, broadcast batches summed back, the shared-right-matrix
  flattening) exactly on dyadic data against oracle.matmul_backward, and f32
  products within the f32 bound;
* conv2d_backward: grouped_dilated_padded_convolution_gradients
  (kernix-ops/tests/neural_vision_tests.rs:46-79, central differences of
  sum(y^2)/2) and bit-for-bit equality with the oracle's restatement of the
  reference loop (neural.rs:379-430) on strided, grouped and dilated cases.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def dev(torch, arr):
    return torch.from_numpy(np.array(arr, order="C")).cuda()      # keeps 0-d gradients 0-d


@pytest.mark.parametrize("m,k,n", [(65, 67, 69), (128, 32, 128)])
def test_large_matmul_gradients_known_answers(kx, torch_cuda, m, k, n):
    av = (np.arange(m * k) % 23) / 16.0 - 0.5
    bv = (np.arange(k * n) % 13) / 8.0 - 0.5
    a, b = av.reshape(m, k), bv.reshape(k, n)
    g = np.ones((m, n))                     # d sum(y) / dy
    da, db = kx.matmul_backward(dev(torch_cuda, a), dev(torch_cuda, b), dev(torch_cuda, g))
    da, db = da.cpu().numpy(), db.cpu().numpy()
    assert np.array_equal(da, np.broadcast_to(b.sum(axis=1), (m, k)))
    assert np.array_equal(db, np.broadcast_to(a.sum(axis=0)[:, None], (k, n)))


GEOMETRIES = [
    ((5,), (5,)), ((5,), (5, 3)), ((4, 5), (5,)), ((4, 5), (5, 3)),
    ((2, 4, 5), (5, 3)), ((2, 3, 4, 5), (5,)), ((2, 4, 5), (2, 5, 3)),
    ((2, 1, 4, 5), (1, 3, 5, 3)), ((3, 4, 5), (1, 5, 3)), ((4, 5), (2, 5, 3)), ((5,), (2, 5, 3)),
    ((2, 0, 4, 5), (5, 3)), ((4, 0), (0, 3)), ((0, 5), (5, 3)),
]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("ad,bd", GEOMETRIES, ids=lambda v: "x".join(map(str, v)))
def test_matmul_vjp_exact_on_dyadic_data(kx, torch_cuda, ad, bd, dtype):
    rs = np.random.default_rng(hash((ad, bd)) % 2**32)
    a = (rs.integers(-8, 9, ad) / 8).astype(dtype)
    b = (rs.integers(-8, 9, bd) / 4).astype(dtype)
    out_dims = kx.matmul_shape(ad, bd)
    g = (rs.integers(-4, 5, out_dims) / 2).astype(dtype)
    want_a, want_b = oracle.matmul_backward(a, b, g)
    da, db = kx.matmul_backward(dev(torch_cuda, a), dev(torch_cuda, b), dev(torch_cuda, g))
    assert da.cpu().numpy().tolist() == want_a.astype(dtype).tolist()
    assert db.cpu().numpy().tolist() == want_b.astype(dtype).tolist()


def test_matmul_vjp_f32_transposed_views_within_bound(kx, torch_cuda):
    """Views as inputs (a transposed, b a column slice) and a long flattened
    contraction for the shared right matrix: within 2e-6 sum|terms|."""
    from kernix_b200 import rng
    torch = torch_cuda
    a_t = rng.uniform(81, 300 * 6 * 96, -1, 1).reshape(6, 96, 300)        # a = a_t^T per batch
    bbuf = rng.uniform(82, 96 * 260, -1, 1).reshape(96, 260)
    a = np.swapaxes(a_t, 1, 2)                                             # [6, 300, 96]
    b = bbuf[:, :200]
    g = rng.uniform(83, 6 * 300 * 200, -1, 1).reshape(6, 300, 200)
    da, db = kx.matmul_backward(dev(torch, a_t).transpose(1, 2), dev(torch, bbuf)[:, :200], dev(torch, g))
    want_a, want_b = oracle.matmul_backward(a, b, g)
    abs_a, abs_b = oracle.matmul_backward(np.abs(a), np.abs(b), np.abs(g))
    assert (np.abs(da.cpu().numpy() - want_a) <= 2e-6 * abs_a + 1e-30).all()
    assert (np.abs(db.cpu().numpy() - want_b) <= 2e-6 * abs_b + 1e-30).all()


def test_matmul_vjp_errors_and_partial_requests(kx, torch_cuda):
    torch = torch_cuda
    a, b = torch.ones(3, 4, device="cuda"), torch.ones(4, 2, device="cuda")
    with pytest.raises(kx.InvalidParameter):
        kx.matmul_backward(a, b, torch.ones(3, 3, device="cuda"))
    with pytest.raises(kx.ContractDimensionMismatch):
        kx.matmul_backward(a, torch.ones(5, 2, device="cuda"), torch.ones(3, 2, device="cuda"))
    da, db = kx.matmul_backward(a, b, torch.ones(3, 2, device="cuda"), need_b=False)
    assert db is None and bool((da == 2).all())


def generated(dims):
    """neural_vision_tests.rs:7-13."""
    n = int(np.prod(dims))
    return ((np.arange(n) * 7 % 19 - 9.0) / 10.0).reshape(dims)


def test_grouped_dilated_padded_gradients_match_central_differences(kx, torch_cuda):
    x, w = generated((1, 2, 4, 5)), generated((2, 1, 2, 2))
    o = dict(groups=2, padding=(1, 1), stride=(2, 1), dilation=(2, 1))
    opts = kx.Conv2dOptions(**o)
    y = oracle.conv2d_reference(oracle.View.of(x), oracle.View.of(w), **o)
    dx, dw = kx.conv2d_backward(dev(torch_cuda, x), dev(torch_cuda, w), dev(torch_cuda, y), opts)
    dx, dw = dx.cpu().numpy().reshape(-1), dw.cpu().numpy().reshape(-1)

    def objective(xx, ww):
        yy = oracle.conv2d_reference(oracle.View.of(xx), oracle.View.of(ww), **o)
        return float((yy * yy / 2.0).sum())
    h = 1e-5
    for arr, grad, which in ((x, dx, 0), (w, dw, 1)):
        for i in range(arr.size):
            p, q = arr.copy().reshape(-1), arr.copy().reshape(-1)
            p[i] += h
            q[i] -= h
            args_p = (p.reshape(arr.shape), w) if which == 0 else (x, p.reshape(arr.shape))
            args_q = (q.reshape(arr.shape), w) if which == 0 else (x, q.reshape(arr.shape))
            fd = (objective(*args_p) - objective(*args_q)) / (2 * h)
            assert abs(grad[i] - fd) <= 2e-7 * (1 + abs(grad[i]) + abs(fd)), (which, i)


CONV_CASES = [
    ((2, 3, 7, 6), (4, 3, 3, 3), dict(stride=(1, 1), padding=(1, 1), dilation=(1, 1), groups=1)),
    ((1, 4, 9, 8), (6, 2, 2, 3), dict(stride=(2, 3), padding=(0, 2), dilation=(2, 1), groups=2)),
    ((3, 2, 5, 5), (2, 2, 5, 5), dict(stride=(1, 1), padding=(2, 2), dilation=(1, 1), groups=1)),
    ((2, 6, 6, 7), (6, 1, 3, 3), dict(stride=(2, 2), padding=(1, 0), dilation=(1, 2), groups=6)),
]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("xd,wd,o", CONV_CASES)
def test_conv2d_backward_bitwise_reference_loop(kx, torch_cuda, xd, wd, o, dtype):
    from kernix_b200 import rng
    torch = torch_cuda
    x = rng.uniform(91, int(np.prod(xd)), -1, 1, dtype).reshape(xd)
    w = rng.uniform(92, int(np.prod(wd)), -1, 1, dtype).reshape(wd)
    yd = oracle.conv_shape(xd, wd, **o)
    gy = rng.uniform(93, int(np.prod(yd)), -1, 1, dtype).reshape(yd)
    want_dx, want_dw = oracle.conv2d_backward(oracle.View.of(x), oracle.View.of(w), gy, **o)
    # input as a permuted view of a channels-last buffer: strides taken in place
    xt = dev(torch, np.ascontiguousarray(x.transpose(0, 2, 3, 1))).permute(0, 3, 1, 2)
    dx, dw = kx.conv2d_backward(xt, dev(torch, w), dev(torch, gy), kx.Conv2dOptions(**o))
    assert np.array_equal(dx.cpu().numpy(), want_dx)
    assert np.array_equal(dw.cpu().numpy(), want_dw)


def test_conv2d_backward_errors_and_empty(kx, torch_cuda):
    torch = torch_cuda
    x, w = torch.ones(1, 2, 5, 5, device="cuda"), torch.ones(3, 2, 3, 3, device="cuda")
    with pytest.raises(kx.InvalidParameter):
        kx.conv2d_backward(x, w, torch.ones(1, 3, 4, 4, device="cuda"))
    dx, dw = kx.conv2d_backward(torch.ones(0, 2, 5, 5, device="cuda"), w, torch.ones(0, 3, 3, 3, device="cuda"))
    assert tuple(dx.shape) == (0, 2, 5, 5) and not bool(dw.any())
