"""Parity at the benchmark's full sizes, on the same seeded inputs.

Small-shape tests cover the edge cases; these run the four large
configurations end to end and check sampled outputs against the compensated
oracle with the reference's own bounds:

* f32: |x - y| <= 2e-6 * sum|a b| per output (small_matmul_tests.rs:153-186)
  and the normwise max|x - y| / max|y| <= 1e-5;
* f64: |x - y| <= 1e-13 * sum|a b| and |x - y| <= 1e-12 (1 + |y|)
  (native_kernel_tests.rs:29-108);
* attention: the f32 bound on P v plus the f32 score bound carried through
  the softmax (see test_attention_gpu.py).

Rows are spread over every row tile of the output (the tile boundaries the
kernels partition by), at varying offsets inside each tile.
"""
import math

import numpy as np
import pytest

import oracle
from kernix_b200 import rng

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def spread_rows(m, count=64, tile=128):
    tiles = max(1, m // tile)
    return sorted({min(m - 1, (i * tiles // count) * tile + (i * 53 + 7) % tile) for i in range(count)})


def f32_check(got, want, absum):
    d = np.abs(np.asarray(got, np.float64) - want)
    assert (d <= 2e-6 * absum + 1e-30).all(), float((d / absum).max())
    assert d.max() <= 1e-5 * np.abs(want).max()


def test_c5_gemm_8192_strided_a(kx, torch_cuda):
    """f32 8192^3, A the first 8192 columns of an 8192 x 8704 buffer (seed 5), B
    row-major (seed 6): 64 rows over all 64 row tiles."""
    torch = torch_cuda
    M = N = K = 8192
    RS = 8704
    a = rng.uniform(5, M * RS, -1.0, 1.0)
    b = rng.uniform(6, K * N, -1.0, 1.0).reshape(K, N)
    da = kx.TensorView(torch.from_numpy(a).cuda(), (M, K), (RS, 1))
    c = kx.matmul(da, torch.from_numpy(b).cuda())
    assert "tf32" in kx.handle(0).last_kernel
    rows = spread_rows(M)
    sub = np.ascontiguousarray(a.reshape(M, RS)[rows, :K])
    want, absum = oracle.gemm_dot2(oracle.View.of(sub), oracle.View.of(b))
    f32_check(c[rows].cpu().numpy(), want, absum)


def test_c2_f64_4096_transposed_b(kx, torch_cuda):
    """f64 4096^3, B a transposed (column-major) view, N(0,1) entries (seed 1)."""
    torch = torch_cuda
    n = 4096
    v = rng.normal(1, 2 * n * n, 1.0, np.float64)
    a, bt = v[:n * n].reshape(n, n), v[n * n:].reshape(n, n)
    c = kx.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(bt).cuda().t())
    assert "dmma" in kx.handle(0).last_kernel
    rows = spread_rows(n)
    want, absum = oracle.gemm_dot2(oracle.View.of(np.ascontiguousarray(a[rows])), oracle.View(bt, (n, n), (1, n)))
    d = np.abs(c[rows].cpu().numpy() - want)
    assert (d <= 1e-13 * absum).all(), float((d / absum).max())
    assert (d <= 1e-12 * (1 + np.abs(want))).all()


def test_c3_attention_one_batch_of_32_heads(kx, torch_cuda):
    """One batch of the attention workload (32 heads, seq 2048, d 128, N(0,1),
    seed 2): the fused call on four heads x 16 rows against exact attention,
    and the composed path's scores against the compensated product."""
    torch = torch_cuda
    shape = (1, 32, 2048, 128)
    n = int(np.prod(shape))
    q, k, v = (rng.normal(2, n, 1.0, start=j * n * 16).reshape(shape) for j in range(3))
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    t = math.sqrt(128.0)
    o = kx.attention(dq, dk.transpose(2, 3), dv, t)
    assert kx.handle(0).last_kernel.startswith("attn_3xtf32")
    rows = spread_rows(2048, 16)
    for hd in (0, 11, 22, 31):
        truth, absv, sabs = oracle.attention_truth(q[0, hd][None], k[0, hd][None], v[0, hd][None], t, rows)
        err = np.abs(o[0, hd, rows].cpu().numpy().astype(np.float64) - truth[0])
        tol = (2e-6 + 4e-6 * sabs[0][:, None] / t) * absv[0]
        assert (err <= tol).all(), (hd, float((err / tol).max()))
    s = kx.matmul(dq[0, :4], dk[0, :4].transpose(1, 2))
    for hd in range(4):
        want, absum = oracle.gemm_dot2(oracle.View.of(np.ascontiguousarray(q[0, hd][rows])),
                                       oracle.View(k[0, hd], (128, 2048), (1, 128)))
        d = np.abs(s[hd, rows].cpu().numpy().astype(np.float64) - want)
        assert (d <= 2e-6 * absum).all()


def test_c4_conv_64x128x56_3x3_256(kx, torch_cuda):
    """conv2d 64 x 128 x 56 x 56, 256 3x3 filters, pad 1 (x uniform[-1,1] seed
    3, w Kaiming-normal seed 4): the first and last image, every channel."""
    torch = torch_cuda
    x = rng.uniform(3, 64 * 128 * 56 * 56, -1.0, 1.0).reshape(64, 128, 56, 56)
    w = rng.normal(4, 256 * 128 * 9, math.sqrt(2.0 / 1152.0)).reshape(256, 128, 3, 3)
    y = kx.conv2d(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), kx.Conv2dOptions(padding=(1, 1)))
    assert "conv_tc" in kx.handle(0).last_kernel
    imgs = [0, 63]
    want, absum = oracle.conv2d_dot2(oracle.View.of(np.ascontiguousarray(x[imgs])), oracle.View.of(w),
                                     padding=(1, 1))
    f32_check(y[imgs].cpu().numpy(), want, absum)
