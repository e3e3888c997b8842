"""tensordot on the device, and the blocked factorisations' trailing updates
through the strided hook.

tensordot: the reference's tests (ops_completeness_03.rs:224-237, 312-323;
contraction_paths.rs:61-102) with their exact values, the ordered mode bit
for bit against the oracle's restatement (linalg_extra.rs:164-276: sums in
C order over the contraction index space), errors in the reference order, and
layouts that force the gather into GEMM order.

Trailing updates: the calls blocked_cholesky.rs:75-100 and blocked_qr.rs:
55-64, 137-139 make to MatmulElement::try_strided_matmul (a panel times its own
transposed view, a Gram matrix of transposed views) through
kx_try_strided_matmul against the compensated oracle.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def dev(torch, arr):
    return torch.from_numpy(np.array(arr, order="C")).cuda()


def test_known_answers(kx, torch_cuda):
    torch = torch_cuda
    x = np.array([[1, 2, 3], [4, 5, 6]], np.float64)
    y = np.array([[1, 0, 0], [0, 1, 0], [0, 0, 1], [1, 1, 1]], np.float64)
    z = kx.tensordot(dev(torch, x), dev(torch, y), [1], [1])
    assert z.shape == (2, 4) and z.cpu().numpy().reshape(-1).tolist() == [1, 2, 3, 6, 4, 5, 6, 15]
    zeros = kx.tensordot(torch.zeros(2, 0, dtype=torch.float64, device="cuda"),
                         torch.zeros(0, 3, dtype=torch.float64, device="cuda"), [1], [0])
    assert zeros.shape == (2, 3) and not bool(zeros.any())
    with pytest.raises(kx.ContractDimensionMismatch):
        kx.tensordot(dev(torch, x), dev(torch, y), [0], [1])
    p = kx.tensordot(dev(torch, np.array(3.0)), dev(torch, np.array([5.0, 7.0])), [], [])
    assert p.shape == (2,) and p.cpu().numpy().tolist() == [15.0, 21.0]
    e = kx.tensordot(torch.zeros(0, 2, dtype=torch.float64, device="cuda"), dev(torch, np.ones((2, 3))), [1], [0])
    assert e.shape == (0, 3)
    # reverse_axis view (contraction_paths.rs:90-101): a Order::F [2,3], axis 1 reversed
    a = np.arange(6, dtype=np.float64).reshape(2, 3)
    buf = dev(torch, a.T.copy().reshape(-1))                          # F order storage
    rev = kx.TensorView(buf, (2, 3), (1, -2), 4)                      # column 2 - j
    r = kx.tensordot(rev, dev(torch, np.ones((3, 2))), [1], [0])
    assert r.cpu().numpy().reshape(-1).tolist() == [3.0, 3.0, 12.0, 12.0]


CASES = [
    ((2, 3, 4), (3, 4, 5), [1, 2], [0, 1]),
    ((2, 3, 4), (4, 3, 5), [2, 1], [0, 1]),        # contracted axes out of order: gathered
    ((2, 0, 4), (0, 4, 5), [1, 2], [0, 1]),
    ((2, 3), (4,), [], []),
    ((), (), [], []),
    ((5, 6, 7), (7, 2, 6), [-1, 1], [0, -1]),
    ((3, 4, 5, 6), (6, 4, 2), [3, 1], [0, 1]),
]


@pytest.mark.parametrize("ad,bd,aa,ba", CASES)
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_ordered_mode_bitwise_reference_order(kx, torch_cuda, ad, bd, aa, ba, dtype):
    """contraction_paths.rs:61-88 values, every output summed in the reference
    order: bit for bit in ordered mode."""
    n_a, n_b = int(np.prod(ad)), int(np.prod(bd))
    a = ((np.arange(n_a) - 3.0) / 47.0).astype(dtype).reshape(ad)
    b = ((np.arange(n_b) - 2.0) / 13.0).astype(dtype).reshape(bd)
    want = oracle.tensordot(a, b, aa, ba)
    h = kx.handle(0)
    h.set_ordered_matmul(True)
    try:
        got = kx.tensordot(dev(torch_cuda, a), dev(torch_cuda, b), aa, ba).cpu().numpy()
    finally:
        h.set_ordered_matmul(False)
    assert got.shape == want.shape and np.array_equal(got, want)
    fast = kx.tensordot(dev(torch_cuda, a), dev(torch_cuda, b), aa, ba).cpu().numpy()
    absum = oracle.tensordot(np.abs(a).astype(np.float64), np.abs(b).astype(np.float64), aa, ba)
    bound = 2e-6 if dtype == np.float32 else 1e-13
    assert (np.abs(fast.astype(np.float64) - want) <= bound * absum + 1e-300).all()


def test_large_contraction_on_the_tensor_cores(kx, torch_cuda):
    """[8, 64, 96] x [96, 64, 80] over a's axes (2, 1) and b's (0, 1): a's
    contracted axes do not nest in that order, so a is gathered into [8, 6144]
    and b is read in place as [6144, 80]; one 8 x 6144 x 80 GEMM."""
    from kernix_b200 import rng
    a = rng.uniform(101, 8 * 64 * 96, -1, 1).reshape(8, 64, 96)
    b = rng.uniform(102, 96 * 64 * 80, -1, 1).reshape(96, 64, 80)
    got = kx.tensordot(dev(torch_cuda, a), dev(torch_cuda, b), [2, 1], [0, 1]).cpu().numpy()
    want = np.tensordot(a.astype(np.float64), b.astype(np.float64), ([2, 1], [0, 1]))
    absum = np.tensordot(np.abs(a).astype(np.float64), np.abs(b).astype(np.float64), ([2, 1], [0, 1]))
    assert (np.abs(got - want) <= 2e-6 * absum).all()


def test_errors_in_reference_order(kx, torch_cuda):
    torch = torch_cuda
    a, b = torch.zeros(2, 3, 4, device="cuda"), torch.zeros(4, 3, device="cuda")
    with pytest.raises(kx.ContractAxesMismatch) as e:
        kx.tensordot(a, b, [1, 2], [0])
    assert (e.value.left, e.value.right) == (2, 1)
    with pytest.raises(kx.AxisOutOfBounds) as e:
        kx.tensordot(a, b, [3], [0])
    assert (e.value.axis, e.value.rank) == (3, 3)
    with pytest.raises(kx.AxisOutOfBounds) as e:
        kx.tensordot(a, b, [2], [-3])
    assert (e.value.axis, e.value.rank) == (-3, 2)
    with pytest.raises(kx.DuplicateAxis) as e:
        kx.tensordot(a, b, [2, -1], [0, 1])
    assert e.value.axis == 2
    with pytest.raises(kx.ContractDimensionMismatch):
        kx.tensordot(a, b, [1], [0])


@pytest.mark.parametrize("n,row,col,rows,cols,depth", [(384, 128, 0, 256, 128, 128), (200, 64, 64, 136, 70, 64)])
def test_cholesky_trailing_update_through_the_hook(kx, n, row, col, rows, cols, depth):
    """blocked_cholesky.rs:85-87: left = a[row.., 0..depth] ([rows, depth],
    strides [n, 1]), right = the transposed view of rows col.. ([depth, cols],
    strides [1, n])."""
    from kernix_b200 import rng
    a = rng.uniform(111, n * n, -1, 1, np.float64)
    left = kx.MatrixInput(a, [rows, depth], [n, 1], row * n)
    right = kx.MatrixInput(a, [depth, cols], [1, n], col * n)
    out = np.empty(rows * cols)
    assert kx.try_strided_matmul(left, right, out)
    want, absum = oracle.gemm_dot2(oracle.View(a, (rows, depth), (n, 1), row * n),
                                   oracle.View(a, (depth, cols), (1, n), col * n))
    assert (np.abs(out.reshape(rows, cols) - want) <= 1e-13 * absum).all()


def test_qr_gram_update_through_the_hook(kx):
    """blocked_qr.rs:55-64: the Gram matrix V^T V of a block of Householder
    vectors, both operands views of one buffer (stride m, origin start)."""
    from kernix_b200 import rng
    m, width, start = 1000, 32, 96
    v = rng.normal(112, width * m, 1.0, np.float64)
    vt = kx.MatrixInput(v, [width, m - start], [m, 1], start)
    vv = kx.MatrixInput(v, [m - start, width], [1, m], start)
    w = np.empty(width * width)
    assert kx.try_strided_matmul(vt, vv, w)
    want, absum = oracle.gemm_dot2(oracle.View(v, (width, m - start), (m, 1), start),
                                   oracle.View(v, (m - start, width), (1, m), start))
    assert (np.abs(w.reshape(width, width) - want) <= 1e-13 * absum).all()


def test_qr_apply_update_through_the_hook(kx):
    """blocked_qr.rs:137-139: V [rows, width] read through its transposed
    storage (strides [1, m], origin start) times a row-major W [width, columns]."""
    from kernix_b200 import rng
    m, width, start, columns = 700, 32, 64, 90
    v = rng.normal(113, width * m, 1.0, np.float64)
    w = rng.uniform(114, width * columns, -1, 1, np.float64)
    vin = kx.MatrixInput(v, [m - start, width], [1, m], start)
    win = kx.MatrixInput(w, [width, columns], [columns, 1], 0)
    product = np.empty((m - start) * columns)
    assert kx.try_strided_matmul(vin, win, product)
    want, absum = oracle.gemm_dot2(oracle.View(v, (m - start, width), (1, m), start),
                                   oracle.View(w, (width, columns), (columns, 1), 0))
    assert (np.abs(product.reshape(m - start, columns) - want) <= 1e-13 * absum).all()
