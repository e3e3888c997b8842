"""Input formulas of the reference's own matmul/conv tests, restated.

Each generator reproduces the data a Kernix test builds (cited by file:line in
the kernix repository) so that the same known answers and exact-dyadic
properties can be checked against the oracle and the device path.  Literal
known answers live in kats.json beside this file.
"""
from __future__ import annotations

import numpy as np


def tensor_native(m: int, n: int, dtype=np.float64) -> np.ndarray:
    """native_kernel_tests.rs:7-16: ((i*7 % 37) - 18) / 17, shape [m, n]."""
    i = np.arange(m * n)
    return (((i * 7 % 37) - 18) / 17.0).astype(dtype).reshape(m, n)


def f32_boundary_pair(m: int, k: int, n: int):
    """native_kernel_tests.rs:152-157: A ((i*7%37)-18)/17, B ((i*11%29)-14)/13 in f32."""
    ia, ib = np.arange(m * k), np.arange(k * n)
    a = ((ia * 7 % 37).astype(np.float32) - 18.0) / np.float32(17.0)
    b = ((ib * 11 % 29).astype(np.float32) - 14.0) / np.float32(13.0)
    return a.reshape(m, k), b.reshape(k, n)


def dyadic_pair(m: int, k: int, n: int, dtype):
    """small_matmul_tests.rs:63-72: offset-by-one dyadic slices (exact products and sums)."""
    p, q = np.arange(m * k + 1), np.arange(k * n + 1)
    av = (((p * 7 % 29) - 14) / 8.0).astype(dtype)
    bv = (((q * 11 % 37) - 18) / 16.0).astype(dtype)
    return av, bv   # use av[1:], bv[1:]


DYADIC_M = [0, 1, 3, 4, 5, 6, 7, 8, 15, 16, 17, 31, 32, 33]
DYADIC_K = [0, 1, 3, 4, 5, 31, 32, 63, 64, 65]
DYADIC_N = [0, 1, 7, 8, 9, 15, 16, 17, 24, 31, 32, 33]


def gapped_strides(m: int, k: int, n: int, dtype):
    """native_kernel_tests.rs:258-268: A rows at stride 2k+5 (origin 7, column
    stride 2), B columns at stride 3k+7 (origin 3, row stride 3); NaN gaps."""
    ar, bc = 2 * k + 5, 3 * k + 7
    a = np.full(7 + (m - 1) * ar + 2 * (k - 1) + 1, np.nan, dtype=dtype)
    b = np.full(3 + 3 * (k - 1) + (n - 1) * bc + 1, np.nan, dtype=dtype)
    for i in range(m):
        for p in range(k):
            a[7 + i * ar + 2 * p] = ((i * 7 + p * 3) % 23) / 16.0 - 0.5
    for p in range(k):
        for j in range(n):
            b[3 + 3 * p + j * bc] = ((p * 5 + j * 11) % 13) / 8.0 - 0.5
    return a, (ar, 2), 7, b, (3, bc), 3


GAPPED_SHAPES = [(63, 65, 67), (64, 64, 64), (65, 67, 69), (128, 128, 128), (32, 128, 128), (128, 32, 128),
                 (128, 128, 32)]

F64_BOUNDARY_SHAPES = [(63, 64, 64), (64, 63, 64), (64, 64, 63), (64, 64, 64), (65, 67, 69), (96, 65, 80),
                       (128, 128, 128), (129, 127, 131)]
F32_BOUNDARY_SHAPES = [(63, 64, 65), (64, 63, 65), (65, 64, 63), (64, 64, 64), (65, 67, 69), (128, 128, 128),
                       (129, 127, 131)]


def batched_values(dims, kind: str) -> np.ndarray:
    """batched_matmul_tests.rs:25-38: i/17 - 0.3 (left) and i/13 - 0.2 (right)."""
    n = int(np.prod(dims)) if len(dims) else 1
    i = np.arange(n, dtype=np.float64)
    v = i / 17.0 - 0.3 if kind == "left" else i / 13.0 - 0.2
    return v.reshape(dims)


def conv_inputs(channels: int, groups: int, dtype=np.float64):
    """native_kernel_tests.rs:214-228: input [2, channels, 17, 19], weight [6, channels/groups, 3, 2]."""
    i = np.arange(2 * channels * 17 * 19)
    x = (((i * 7 % 31) - 15) / 31.0).astype(dtype).reshape(2, channels, 17, 19)
    j = np.arange(6 * (channels // groups) * 3 * 2)
    w = (((j * 11 % 29) - 14) / 29.0).astype(dtype).reshape(6, channels // groups, 3, 2)
    return x, w


CONV_OPTIONS = [
    dict(stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1),
    dict(stride=(2, 1), padding=(2, 1), dilation=(2, 1), groups=2),
]


def scaled_pair(scale: float, dtype):
    """small_matmul_tests.rs:158-166: (m,k,n) = (31,63,32) non-dyadic data times scale."""
    m, k, n = 31, 63, 32
    p, q = np.arange(m * k), np.arange(k * n)
    a = ((p * 7 % 37).astype(dtype) - dtype(18.0)) / dtype(17.0) * dtype(scale)
    b = ((q * 11 % 29).astype(dtype) - dtype(14.0)) / dtype(13.0) * dtype(scale)
    return a.reshape(m, k), b.reshape(k, n)


def execution_pair(m: int, k: int, n: int):
    """execution_tests.rs:86-87: (i%23)/16 - 0.5 and (i%13)/8 - 0.5 (exact in f32 and f64)."""
    a = (np.arange(m * k) % 23) / 16.0 - 0.5
    b = (np.arange(k * n) % 13) / 8.0 - 0.5
    return a.reshape(m, k), b.reshape(k, n)


EXECUTION_SHAPES = [(64, 64, 64), (96, 128, 65), (127, 64, 67), (128, 128, 128), (129, 65, 67), (193, 64, 65),
                    (256, 128, 64), (0, 3, 4), (4, 0, 5)]
