"""The attention products in one call (kx_attention_f32) against the oracle.

out = matmul(softmax_temperature(matmul(q, kt), -1, T), v) is how a Kernix user
composes attention (ops/linalg.rs:68-214, ops/math_extra.rs:425-500,544-557).
The fused tensor-core kernel must match the exact attention of the same f32
inputs within the f32 bound the rest of the suite uses (small_matmul_tests.rs:
153-186: |x - y| <= 2e-6 sum|a b|) applied to both products -- P v directly,
the scores through the softmax (see _check) -- and everything
the composition treats specially (inf/NaN scores, inf/NaN in v, layouts the
kernel does not take, ordered mode) must give exactly the composed result.
"""
import math

import numpy as np
import pytest

import oracle
from kernix_b200 import rng

pytestmark = pytest.mark.gpu
FUSED = "attn_3xtf32_128x64"
PAIR = "attn_3xtf32_pair_256x64"       # CTA pairs: chosen from 74 units of 256 query rows


def _inputs(seed, nb, sq, sk, d=128, dv=128, std=1.0):
    q = rng.normal(seed, nb * sq * d, std).reshape(nb, sq, d)
    k = rng.normal(seed + 1, nb * sk * d, std).reshape(nb, sk, d)
    v = rng.normal(seed + 2, nb * sk * dv, 1.0).reshape(nb, sk, dv)
    return q, k, v


def _dev(torch, *arrs):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def _check(got, q, k, v, t, rows=None):
    """|out - exact| <= (2e-6 + 2 * 2e-6 * max_j sum|q k_j| / T) * sum_j p_j |v_j|
    per output: the f32 bound on the product P v, plus the f32 bound on the
    scores (|dS| <= 2e-6 sum|q k|) carried through the softmax, whose
    derivative dp_j/dS_i = p_j (delta_ij - p_i) / T moves P v by at most
    2 max|dS| / T * sum_j p_j |v_j|.  The composed path obeys the same bound."""
    truth, absv, sabs = oracle.attention_truth(q, k, v, t, rows)
    g = got if rows is None else got[:, rows]
    err = np.abs(g.astype(np.float64) - truth)
    tol = (2e-6 + 4e-6 * sabs[..., None] / t) * absv
    assert (err <= tol).all(), float((err / tol).max())
    return float((err / absv).max())


@pytest.mark.parametrize("nb,sq,sk", [(1, 128, 64), (2, 300, 200), (3, 1, 65), (1, 257, 1), (2, 129, 2048),
                                      (1, 2048, 2048)])
def test_fused_matches_exact_attention(kx, torch_cuda, nb, sq, sk):
    torch = torch_cuda
    q, k, v = _inputs(100 + sq + sk, nb, sq, sk)
    t = math.sqrt(128.0)
    dq, dk, dv = _dev(torch, q, k, v)
    h = kx.handle(0)
    out = kx.attention(dq, dk.transpose(1, 2), dv, t)
    assert h.last_kernel == FUSED
    got = out.cpu().numpy()
    rows = None if sq <= 300 else sorted({0, 1, 127, 128, 1000, sq - 1})
    _check(got, q, k, v, t, rows)


@pytest.mark.parametrize("nb,sq,sk", [(74, 256, 64), (40, 520, 1000), (38, 300, 33), (80, 129, 2048)])
def test_pair_kernel_matches_exact_attention(kx, torch_cuda, nb, sq, sk):
    """The CTA-pair kernel: query rows ending inside either CTA's half of a
    256-row unit (520, 300, 129), key blocks ending inside either CTA's 32
    keys (1000 = 15 blocks + 40, 33), and one key block in all (64, 33)."""
    torch = torch_cuda
    q, k, v = _inputs(200 + sq + sk, nb, sq, sk)
    t = math.sqrt(128.0)
    dq, dk, dv = _dev(torch, q, k, v)
    out = kx.attention(dq, dk.transpose(1, 2), dv, t)
    assert kx.handle(0).last_kernel == PAIR
    got = out.cpu().numpy()
    rows = sorted({r for r in (0, 1, 127, 128, 129, 255, 256, 300, 383, 384, 511, 512, sq - 1) if r < sq})
    heads = [0, 1, nb // 2, nb - 1]
    _check(got[heads], q[heads], k[heads], v[heads], t, rows)


def test_pair_kernel_four_dim_heads_and_nonfinite_fallback(kx, torch_cuda):
    """[2, 37, 256, 128] heads on CTA pairs, then an inf score in one head:
    the composed path's NonFiniteInput, and the pair kernel again after it."""
    torch = torch_cuda
    q, k, v = _inputs(51, 74, 256, 192, std=0.5)
    dq, dk, dv = _dev(torch, q.reshape(2, 37, 256, 128), k.reshape(2, 37, 192, 128), v.reshape(2, 37, 192, 128))
    out = kx.attention(dq, dk.transpose(2, 3), dv, 0.9)
    assert kx.handle(0).last_kernel == PAIR
    heads = [0, 36, 37, 73]
    _check(out.cpu().numpy().reshape(74, 256, 128)[heads], q[heads], k[heads], v[heads], 0.9)
    q[40, 200, 3] = np.inf
    dq, = _dev(torch, q.reshape(2, 37, 256, 128))
    with pytest.raises(kx.NonFiniteInput) as e:
        kx.attention(dq, dk.transpose(2, 3), dv, 0.9)
    assert e.value.indices[:3] == [1, 3, 200]
    q[40, 200, 3] = 0.25
    dq, = _dev(torch, q.reshape(2, 37, 256, 128))
    out = kx.attention(dq, dk.transpose(2, 3), dv, 0.9)
    assert kx.handle(0).last_kernel == PAIR
    _check(out.cpu().numpy().reshape(74, 256, 128)[[40]], q[[40]], k[[40]], v[[40]], 0.9)


def test_fused_four_dim_batches_and_small_temperature(kx, torch_cuda):
    """[2, 3, sq, 128] heads (the c3 layout), a temperature well below 1 (large
    exponent arguments), and output rows past the last full block."""
    torch = torch_cuda
    q, k, v = _inputs(7, 6, 200, 320, std=0.3)
    dq, dk, dv = _dev(torch, q.reshape(2, 3, 200, 128), k.reshape(2, 3, 320, 128), v.reshape(2, 3, 320, 128))
    for t in (0.37, 11.3137):
        out = kx.attention(dq, dk.transpose(2, 3), dv, t)
        assert kx.handle(0).last_kernel == FUSED
        _check(out.cpu().numpy().reshape(6, 200, 128), q, k, v, t)


def test_fused_strided_views(kx, torch_cuda):
    """q, k and v as column slices of wider buffers (row strides 160, 192,
    136), the batch axis outermost."""
    torch = torch_cuda
    q, k, v = _inputs(11, 2, 150, 100)
    bq = np.zeros((2, 150, 160), np.float32)
    bk = np.zeros((2, 100, 192), np.float32)
    bv = np.zeros((2, 100, 136), np.float32)
    bq[..., 16:144], bk[..., 64:], bv[..., :128] = q, k, v
    dq, dk, dv = _dev(torch, bq, bk, bv)
    out = kx.attention(dq[..., 16:144], dk[..., 64:].transpose(1, 2), dv[..., :128], 2.5)
    assert kx.handle(0).last_kernel == FUSED
    _check(out.cpu().numpy(), q, k, v, 2.5)


def test_matches_composed_where_the_kernel_declines(kx, torch_cuda):
    """Head dim 64, broadcast batches and ordered mode run the three calls:
    bit for bit the composed result."""
    torch = torch_cuda
    h = kx.handle(0)

    def composed(q, kt, v, t):
        return kx.matmul(kx.softmax_temperature(kx.matmul(q, kt), -1, t), v)

    q, k, v = _inputs(21, 2, 70, 90, d=64, dv=64)
    dq, dk, dv = _dev(torch, q, k, v)
    a = kx.attention(dq, dk.transpose(1, 2), dv, 1.5)
    assert torch.equal(a, composed(dq, dk.transpose(1, 2), dv, 1.5))
    q, k, v = _inputs(22, 2, 70, 90)
    dq, dk, dv = _dev(torch, q, k[:1], v[:1])          # k and v broadcast over the batch
    a = kx.attention(dq, dk.transpose(1, 2), dv, 1.5)
    assert h.last_kernel != FUSED
    assert torch.equal(a, composed(dq, dk.transpose(1, 2), dv, 1.5))
    dq, dk, dv = _dev(torch, q, k, v)
    h.set_ordered_matmul(True)
    try:
        a = kx.attention(dq, dk.transpose(1, 2), dv, 1.5)
        b = composed(dq, dk.transpose(1, 2), dv, 1.5)
    finally:
        h.set_ordered_matmul(False)
    assert torch.equal(a, b)


def test_nonfinite_scores_raise_the_composed_error(kx, torch_cuda):
    """An inf in q makes its score row inf/NaN: NonFiniteInput from the
    softmax step with the first index of the scores, as the oracle's
    composition reports it."""
    torch = torch_cuda
    q, k, v = _inputs(31, 2, 130, 70)
    q[1, 77, 5] = np.inf
    q[1, 90, 0] = np.nan
    s = np.stack([oracle.matmul_reference(oracle.View.of(q[b]), oracle.View(k[b], (128, 70), (1, 128)))
                  for b in range(2)])
    with pytest.raises(oracle.OracleError) as oe:
        oracle.softmax_temperature(s, -1, 3.0)
    dq, dk, dv = _dev(torch, q, k, v)
    with pytest.raises(kx.NonFiniteInput) as ge:
        kx.attention(dq, dk.transpose(1, 2), dv, 3.0)
    assert ge.value.indices == oe.value.fields["indices"]
    assert ge.value.operation == "softmax_temperature"
    # the fused kernel still serves the next call
    q[1, 77, 5] = q[1, 90, 0] = 0.5
    dq, = _dev(torch, q)
    out = kx.attention(dq, dk.transpose(1, 2), dv, 3.0)
    assert kx.handle(0).last_kernel == FUSED
    _check(out.cpu().numpy(), q, k, v, 3.0)


def test_nonfinite_values_propagate_like_the_composition(kx, torch_cuda):
    """inf and NaN in v reach the output through the composed path's IEEE
    propagation (bit for bit the composed result, NaN in the same places)."""
    torch = torch_cuda
    q, k, v = _inputs(41, 1, 140, 130)
    v[0, 3, 7] = np.inf
    v[0, 100, 20] = np.nan
    dq, dk, dv = _dev(torch, q, k, v)
    a = kx.attention(dq, dk.transpose(1, 2), dv, 2.0).cpu().numpy()
    b = kx.matmul(kx.softmax_temperature(kx.matmul(dq, dk.transpose(1, 2)), -1, 2.0), dv).cpu().numpy()
    assert np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(a[~np.isnan(a)], b[~np.isnan(b)])
    assert np.isinf(a[:, :, 7]).all() and np.isnan(a[:, :, 20]).all()


def test_errors_in_the_composition_order(kx, torch_cuda):
    torch = torch_cuda
    z = lambda *s: torch.zeros(*s, device="cuda")  # noqa: E731
    with pytest.raises(kx.ContractDimensionMismatch):
        kx.attention(z(2, 4, 128), z(2, 127, 6), z(2, 6, 128), 1.0)
    with pytest.raises(kx.InvalidParameter) as e:
        kx.attention(z(2, 4, 128), z(2, 128, 6), z(2, 5, 128), 0.0)   # temperature before matmul(P, v)
    assert e.value.operation == "softmax_temperature"
    with pytest.raises(kx.ContractDimensionMismatch):
        kx.attention(z(2, 4, 128), z(2, 128, 6), z(2, 5, 128), 1.0)
    with pytest.raises(kx.AxisOutOfBounds):
        kx.attention(z(128), z(128), z(3), 1.0)                          # scalar scores
    out = kx.attention(z(2, 4, 128), z(2, 128, 0), z(2, 0, 128), 1.0)    # no keys: zeros
    assert tuple(out.shape) == (2, 4, 128) and not bool(out.any())
