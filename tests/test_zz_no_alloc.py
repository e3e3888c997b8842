"""The allocation-free split-K entry point against the oracle and the regular one.

kx_matmul_splitk_f32_static serves callers that may not call cudaMalloc while
they run (a process whose GPU memory is owned up front by its own pool, or a
latency-critical loop that cannot afford the device synchronisation cudaMalloc
and cudaFree can cause): its split-K partial sums live in a fixed static device
array instead of a workspace allocated on demand.  This file is collected last
on purpose, and its tests pass both alone in a fresh process and after the
rest of the suite.  The array keeps the previous call's contents, so every
case runs right after a call on different data that fills the array with other
partial sums: a result that read stale partials would differ from the oracle.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from kernix_b200 import rng

pytestmark = pytest.mark.gpu


def _static_matmul(kx, a, b, out, torch):
    err = kx.KxError()
    da, db, do = kx._descriptor(a), kx._descriptor(b), kx._descriptor(out)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = kx.lib.kx_matmul_splitk_f32_static(C.byref(da), C.byref(db), C.byref(do), stream, C.byref(err))
    return rc, err


def _operands(torch, seed, m, k, n, pad):
    """A [m, k] as a slice of an [m, k + pad] buffer (row stride k + pad) and a
    row-major B [k, n], uniform[-1, 1] from the seeded stream."""
    abuf = rng.uniform(seed, m * (k + pad), -1.0, 1.0).reshape(m, k + pad)
    bbuf = rng.uniform(seed + 1, k * n, -1.0, 1.0).reshape(k, n)
    da = torch.from_numpy(abuf).cuda()[:, :k]
    db = torch.from_numpy(bbuf).cuda()
    want, absum = oracle.gemm_dot2(oracle.View(abuf, (m, k), (k + pad, 1)), oracle.View.of(bbuf))
    return da, db, want, absum


def _fill_scratch(kx, torch):
    """A call whose partial sums cover the array's first M*N*splits entries
    with values unrelated to the next case."""
    a = torch.full((256, 2048), 3.0, device="cuda")
    b = torch.full((2048, 256), -5.0, device="cuda")
    out = torch.empty(256, 256, device="cuda")
    rc, err = _static_matmul(kx, a, b, out, torch)
    assert rc == 0, (rc, err.parameter)
    torch.cuda.synchronize()
    assert bool((out == -30720.0).all())


# (m, k, n, pad): short K takes the single-split path that stores C directly,
# longer K goes through the array; odd extents and strided A throughout.
CASES = [
    (37, 1, 45, 3), (64, 7, 33, 1), (33, 16, 64, 4), (70, 17, 19, 5),
    (300, 127, 129, 2), (96, 128, 80, 0), (512, 512, 512, 0), (300, 1000, 257, 24),
]


@pytest.mark.parametrize("m,k,n,pad", CASES, ids=lambda v: str(v))
def test_static_scratch_matches_oracle_after_a_foreign_call(kx, torch_cuda, m, k, n, pad):
    torch = torch_cuda
    torch.cuda.set_device(0)
    a, b, want, absum = _operands(torch, 4000 + k, m, k, n, pad)
    for call in range(2):                   # two calls in a row on the same inputs
        _fill_scratch(kx, torch)
        got = torch.full((m, n), float("nan"), device="cuda")
        rc, err = _static_matmul(kx, a, b, got, torch)
        assert rc == 0, (rc, err.parameter)
        torch.cuda.synchronize()
        g = got.cpu().numpy().astype(np.float64)
        assert np.isfinite(g).all(), call
        # f32 tolerance used throughout: |x - y| <= 2e-6 * sum |a b| (small_matmul_tests.rs:153-186)
        bad = np.abs(g - want) > 2e-6 * absum + 1e-30
        assert not bad.any(), (call, np.argwhere(bad)[:4].tolist())
        # and the regular entry point on the same operands, within the same bound
        reg = torch.empty(m, n, device="cuda")
        kx.matmul_into(a, b, reg)
        torch.cuda.synchronize()
        assert (np.abs(g - reg.cpu().numpy().astype(np.float64)) <= 4e-6 * absum + 1e-30).all()


def test_static_scratch_rejects_oversized_outputs(kx, torch_cuda):
    torch = torch_cuda
    a = torch.zeros(2048, 8, device="cuda")
    b = torch.zeros(8, 2048, device="cuda")            # 4,194,304 outputs > 2,097,152
    out = torch.full((2048, 2048), 7.0, device="cuda")
    rc, err = _static_matmul(kx, a, b, out, torch)
    assert rc == kx._abi.KX_E_UNSUPPORTED
    assert b"static split-K scratch" in err.parameter
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
