"""The allocation-free split-K entry point against the regular one.

kx_matmul_splitk_f32_static serves callers that may not call cudaMalloc while
they run (a process whose GPU memory is owned up front by its own pool, or a
latency-critical loop that cannot afford the device synchronisation cudaMalloc
and cudaFree can cause): its split-K partial sums live in a fixed static device
array instead of a workspace allocated on demand.  This file is collected last
on purpose, and its test passes both alone in a fresh process and after the
rest of the suite (the array keeps the previous call's contents, so two calls
in a row with different inputs also show that nothing stale leaks through).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _desc(kx, t):
    return kx._descriptor(t)


def _static_matmul(kx, a, b, out, torch):
    err = kx.KxError()
    da, db, do = _desc(kx, a), _desc(kx, b), _desc(kx, out)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = kx.lib.kx_matmul_splitk_f32_static(C.byref(da), C.byref(db), C.byref(do), stream, C.byref(err))
    return rc, err


def test_static_scratch_split_k_matches_regular_entry_point(kx, torch_cuda):
    torch = torch_cuda
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda").manual_seed(1234)
    cases = [
        (512, 512, 512, False),    # c1's shape, row-major
        (300, 1000, 257, True),    # odd extents, A a strided slice (row stride k + 24)
    ]
    for m, k, n, strided in cases:       # two calls in a row with different inputs
        if strided:
            abuf = torch.rand(m, k + 24, device="cuda", generator=gen) * 2 - 1
            a = abuf[:, :k]
        else:
            a = torch.rand(m, k, device="cuda", generator=gen) * 2 - 1
        b = torch.rand(k, n, device="cuda", generator=gen) * 2 - 1
        want = torch.empty(m, n, device="cuda")
        kx.matmul_into(a, b, want)                      # the existing entry point
        got = torch.full((m, n), float("nan"), device="cuda")
        rc, err = _static_matmul(kx, a, b, got, torch)
        assert rc == 0, (rc, err.parameter)
        torch.cuda.synchronize()
        # tolerance used throughout the f32 tests: |x - y| <= 2e-6 * sum |a b|
        absum = (a.double().abs() @ b.double().abs())
        diff = (got.double() - want.double()).abs()
        assert torch.isfinite(got).all()
        assert bool((diff <= 2e-6 * absum + 1e-30).all()), float((diff / absum).max())


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
