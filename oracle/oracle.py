"""CPU oracle for Kernix's dense matmul path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only as the checker.  The product never calls it.

The numeric kernels live in kx_oracle.c (compiled with -ffp-contract=off); this
module restates the shape and dispatch logic of ``matmul_impl``
(crates/kernix-ops/src/ops/linalg.rs:68-232), ``broadcast_shape``
(ops/broadcast.rs:6-34), ``ConvGeometry`` (neural.rs:57-133),
``normalized_exp_advanced`` (ops/math_extra.rs:425-500) and SplitMix64
``SeededRng`` (crates/kernix/src/training.rs:132-171).

Parity pin: the reference (Rust) cannot be built here, so this oracle is pinned
against the known-answer values and exact-dyadic properties of the reference's
own tests (tests/golden/kats.json and tests/test_oracle_golden.py).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libkx_oracle.so"


def build() -> Path:
    srcs = [HERE / "kx_oracle.c", HERE / "kx_engine.c", HERE / "Makefile"]
    if not LIB.exists() or any(LIB.stat().st_mtime < s.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-C", str(HERE), "-s"], check=True)
    return LIB


def _load() -> C.CDLL:
    build()
    lib = C.CDLL(str(LIB))
    i64, u64, vp, dbl = C.c_int64, C.c_uint64, C.c_void_p, C.c_double
    lib.kxo_splitmix_next.argtypes = [C.POINTER(u64)]
    lib.kxo_splitmix_next.restype = u64
    for t in ("f32", "f64"):
        getattr(lib, f"kxo_uniform_{t}").argtypes = [u64, u64, dbl, dbl, vp]
        getattr(lib, f"kxo_uniform_{t}").restype = u64
        getattr(lib, f"kxo_dense_matmul_{t}").argtypes = [vp, vp, vp, u64, u64, u64]
        getattr(lib, f"kxo_gemm_ordered_{t}").argtypes = [vp, i64, i64, vp, i64, i64, vp, i64, i64, i64, i64, i64]
        getattr(lib, f"kxo_gemm_ordered_par_{t}").argtypes = [vp, i64, i64, vp, i64, i64, vp, i64, i64, i64, i64,
                                                             i64, C.c_int]
        getattr(lib, f"kxo_gemm_dot2_{t}").argtypes = [vp, i64, i64, vp, i64, i64, vp, vp, i64, i64, i64, C.c_int]
        getattr(lib, f"kxo_conv2d_reference_{t}").argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp]
        getattr(lib, f"kxo_conv2d_dot2_{t}").argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, C.c_int]
        getattr(lib, f"kxo_conv2d_backward_{t}").argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
        getattr(lib, f"kxo_softmax_rows_{t}").argtypes = [vp, vp, i64, i64, C.c_float if t == "f32" else dbl]
        getattr(lib, f"kxo_softmax_rows_{t}").restype = i64
        getattr(lib, f"kxo_engine_gemm_{t}").argtypes = [vp, i64, i64, vp, i64, i64, vp, i64, i64, i64, C.c_int]
        getattr(lib, f"kxo_engine_gemm_{t}").restype = C.c_int
    lib.kxo_openmp_threads.restype = C.c_int
    return lib


lib = _load()
THREADS = int(os.environ.get("KX_ORACLE_THREADS", "0")) or lib.kxo_openmp_threads()


def _t(dtype) -> str:
    dtype = np.dtype(dtype)
    if dtype == np.float32:
        return "f32"
    if dtype == np.float64:
        return "f64"
    raise TypeError(f"oracle handles f32/f64, got {dtype}")


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


# ---------------------------------------------------------------------------
# Seeded inputs (SplitMix64)
# ---------------------------------------------------------------------------
def splitmix_next(state: int) -> tuple[int, int]:
    s = C.c_uint64(state)
    v = lib.kxo_splitmix_next(C.byref(s))
    return int(v), int(s.value)


def uniform(seed: int, n: int, low: float, high: float, dtype=np.float32) -> np.ndarray:
    out = np.empty(n, dtype=dtype)
    getattr(lib, f"kxo_uniform_{_t(dtype)}")(seed, n, low, high, _p(out))
    return out


# ---------------------------------------------------------------------------
# Strided views over numpy buffers (element strides, signed)
# ---------------------------------------------------------------------------
class View:
    """Element (i0..) of ``buf[origin + sum(i_j * strides[j])]``."""

    def __init__(self, buf: np.ndarray, dims, strides, origin: int = 0):
        self.buf = np.ascontiguousarray(buf).reshape(-1)
        self.dims = tuple(int(d) for d in dims)
        self.strides = tuple(int(s) for s in strides)
        self.origin = int(origin)

    @staticmethod
    def of(arr: np.ndarray) -> "View":
        arr = np.ascontiguousarray(arr)
        st = tuple(s // arr.itemsize for s in arr.strides)
        return View(arr.reshape(-1), arr.shape, st, 0)

    @property
    def dtype(self):
        return self.buf.dtype

    def ptr(self, offset: int = 0) -> int:
        return self.buf.ctypes.data + (self.origin + offset) * self.buf.itemsize

    def to_array(self) -> np.ndarray:
        out = np.empty(self.dims, dtype=self.buf.dtype)
        for idx in np.ndindex(*self.dims):
            out[idx] = self.buf[self.origin + sum(i * s for i, s in zip(idx, self.strides))]
        return out


class OracleError(Exception):
    def __init__(self, kind: str, **fields):
        super().__init__(kind, fields)
        self.kind = kind
        self.fields = fields


def broadcast_shape(left, right):
    """ops/broadcast.rs:6-34."""
    rank = max(len(left), len(right))
    out = []
    for axis in range(rank):
        a = left[axis + len(left) - rank] if axis + len(left) >= rank else 1
        b = right[axis + len(right) - rank] if axis + len(right) >= rank else 1
        if a == b or b == 1:
            out.append(a)
        elif a == 1:
            out.append(b)
        else:
            raise OracleError("BroadcastIncompatible", axis=axis, left=a, right=b)
    return out


def validate_dims(dims):
    """Kahen::new (kernix-core shape/utils.rs:3-21)."""
    if 0 in dims:
        return
    acc = 1
    for axis, d in enumerate(dims):
        if acc * d > (1 << 64) - 1:
            raise OracleError("ElementCountOverflow", axis=axis, accumulated=acc, dim=d)
        acc *= d


def matmul_shape(a, b):
    """matmul_impl validation prefix (linalg.rs:77-116)."""
    if len(a) == 0:
        raise OracleError("InvalidRank", minimum=1, actual=0)
    if len(b) == 0:
        raise OracleError("InvalidRank", minimum=1, actual=0)
    av, bv = len(a) == 1, len(b) == 1
    abr = 0 if av else len(a) - 2
    bbr = 0 if bv else len(b) - 2
    m = 1 if av else a[-2]
    k = a[-1]
    kb = b[0] if bv else b[-2]
    n = 1 if bv else b[-1]
    if k != kb:
        raise OracleError("ContractDimensionMismatch", left=k, right=kb)
    batch = broadcast_shape(list(a[:abr]), list(b[:bbr]))
    out = list(batch) + ([] if av else [m]) + ([] if bv else [n])
    validate_dims(out)
    return out, batch, (av, bv, abr, bbr, m, k, n)


def matmul_reference(a: View, b: View) -> np.ndarray:
    """matmul_reference: increasing-k `value += a*b` per output for any layout
    (linalg.rs:57-64 with the general fallback :176-213)."""
    if a.dtype != b.dtype:
        raise TypeError("dtype mismatch")
    out_dims, batch, (av, bv, abr, bbr, m, k, n) = matmul_shape(a.dims, b.dims)
    out = np.zeros(out_dims, dtype=a.dtype)
    if out.size == 0:
        return out
    flat = out.reshape(-1)
    gemm = getattr(lib, f"kxo_gemm_ordered_{_t(a.dtype)}")
    a_rs = 0 if av else a.strides[-2]
    a_cs = a.strides[-1]
    b_rs = b.strides[0] if bv else b.strides[-2]
    b_cs = 0 if bv else b.strides[-1]
    nb = len(batch)
    mn = m * n
    for bi, coords in enumerate(np.ndindex(*batch) if nb else [()]):
        oa = sum(0 if a.dims[i] == 1 else coords[nb - abr + i] * a.strides[i] for i in range(abr))
        ob = sum(0 if b.dims[i] == 1 else coords[nb - bbr + i] * b.strides[i] for i in range(bbr))
        sub = flat[bi * mn:(bi + 1) * mn]
        gemm(a.ptr(oa), a_rs, a_cs, b.ptr(ob), b_rs, b_cs, sub.ctypes.data, n, 1, m, n, k)
    return out


def dense_matmul(a: np.ndarray, b: np.ndarray, m: int, k: int, n: int) -> np.ndarray:
    """linalg.rs:236-316 on C-order slices."""
    out = np.empty(m * n, dtype=a.dtype)
    getattr(lib, f"kxo_dense_matmul_{_t(a.dtype)}")(_p(np.ascontiguousarray(a)), _p(np.ascontiguousarray(b)),
                                                    _p(out), m, k, n)
    return out


def gemm_dot2(a: View, b: View, threads: int | None = None):
    """Compensated f64 product of two rank-2 views and the sum |a_ip * b_pj|."""
    m, k = a.dims
    k2, n = b.dims
    assert k == k2
    out = np.empty((m, n), dtype=np.float64)
    absm = np.empty((m, n), dtype=np.float64)
    getattr(lib, f"kxo_gemm_dot2_{_t(a.dtype)}")(a.ptr(), a.strides[0], a.strides[1], b.ptr(), b.strides[0],
                                                 b.strides[1], _p(out), _p(absm), m, n, k, threads or THREADS)
    return out, absm


def engine_gemm(a: View, b: View, threads: int = 1) -> np.ndarray:
    """The blocked fp32/f64 engine restatement (kx_engine.c): the BLIS loop
    nest gemm-f32/f64 0.19.0 and matrixmultiply 0.3.11 implement, serial for
    threads=1, else row chunks over threads as CpuExecutor::matmul_into
    (execution.rs:188-233).  Rounding: fp32 (f64) FMA accumulation per k
    block, blocks added into C -- a CPU result of the kind Kernix returns."""
    m, k = a.dims
    k2, n = b.dims
    assert k == k2
    out = np.empty((m, n), dtype=a.dtype)
    rc = getattr(lib, f"kxo_engine_gemm_{_t(a.dtype)}")(a.ptr(), a.strides[0], a.strides[1], b.ptr(), b.strides[0],
                                                        b.strides[1], _p(out), m, n, k, int(threads))
    if rc:
        raise MemoryError("engine packing buffers")
    return out


def gemm_ordered_par(a: View, b: View, threads: int | None = None) -> np.ndarray:
    """Row-parallel ordered GEMM (bits equal to the serial ordered result)."""
    m, k = a.dims
    _, n = b.dims
    out = np.empty((m, n), dtype=a.dtype)
    getattr(lib, f"kxo_gemm_ordered_par_{_t(a.dtype)}")(a.ptr(), a.strides[0], a.strides[1], b.ptr(), b.strides[0],
                                                        b.strides[1], _p(out), n, 1, m, n, k, threads or THREADS)
    return out


# ---------------------------------------------------------------------------
# conv2d
# ---------------------------------------------------------------------------
def conv_extent(size, kernel, stride, padding, dilation):
    """neural.rs:57-83."""
    if kernel == 0 or stride == 0 or dilation == 0:
        raise OracleError("InvalidParameter", parameter="kernel, stride and dilation must be positive")
    effective = (kernel - 1) * dilation + 1
    padded = size + 2 * padding
    if effective > (1 << 64) - 1 or padded > (1 << 64) - 1:
        raise OracleError("DimensionOverflow", axis=2)
    return 0 if padded < effective else (padded - effective) // stride + 1


def conv_shape(x_dims, w_dims, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1):
    """ConvGeometry::new (neural.rs:91-125)."""
    validate_dims(x_dims)
    if len(x_dims) != 4:
        raise OracleError("ExactRank", expected=4, actual=len(x_dims))
    validate_dims(w_dims)
    if len(w_dims) != 4:
        raise OracleError("ExactRank", expected=4, actual=len(w_dims))
    n, ci, h, w = x_dims
    co, cg, kh, kw = w_dims
    g = groups
    if g == 0 or ci == 0 or co == 0 or ci % g or co % g or cg != ci // g:
        raise OracleError("InvalidParameter", parameter="groups and input/output channels must agree")
    oh = conv_extent(h, kh, stride[0], padding[0], dilation[0])
    ow = conv_extent(w, kw, stride[1], padding[1], dilation[1])
    out = [n, co, oh, ow]
    validate_dims(out)
    return out


def _conv_args(x: View, w: View, stride, padding, dilation, groups):
    yd = conv_shape(x.dims, w.dims, stride, padding, dilation, groups)
    a = lambda v: np.asarray(v, dtype=np.int64)  # noqa: E731
    opt = a([stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1], groups])
    return yd, a(x.dims), a(x.strides), a(w.dims), a(w.strides), a(yd), opt


def conv2d_reference(x: View, w: View, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1) -> np.ndarray:
    """conv2d_reference: ordered scalar path (neural.rs:341-357)."""
    yd, xd, xs, wd, ws, yda, opt = _conv_args(x, w, stride, padding, dilation, groups)
    y = np.zeros(yd, dtype=x.dtype)
    if y.size:
        getattr(lib, f"kxo_conv2d_reference_{_t(x.dtype)}")(x.ptr(), _p(xd), _p(xs), w.ptr(), _p(wd), _p(ws), _p(y),
                                                            _p(yda), _p(opt))
    return y


def conv2d_dot2(x: View, w: View, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1, threads=None):
    yd, xd, xs, wd, ws, yda, opt = _conv_args(x, w, stride, padding, dilation, groups)
    y = np.zeros(yd, dtype=np.float64)
    ab = np.zeros(yd, dtype=np.float64)
    if y.size:
        getattr(lib, f"kxo_conv2d_dot2_{_t(x.dtype)}")(x.ptr(), _p(xd), _p(xs), w.ptr(), _p(wd), _p(ws), _p(y),
                                                       _p(ab), _p(yda), _p(opt), threads or THREADS)
    return y, ab


# ---------------------------------------------------------------------------
# softmax_temperature
# ---------------------------------------------------------------------------
def softmax(x: np.ndarray, axis: int) -> np.ndarray:
    """normalized_exp, not logarithmic (math.rs:398-465): axis check, finite
    scan, max, sequential sum of exp(x - max), exp(x - max) / sum.  The values
    are those of temperature 1 ((x - max) / 1 is exact, and the divide-first
    branch gives x - max again), so the same row routine computes them."""
    return _softmax_rows(x, axis, 1.0, "softmax")


def softmax_temperature(x: np.ndarray, axis: int, temperature: float) -> np.ndarray:
    """normalized_exp_advanced without mask (math_extra.rs:425-500)."""
    if not np.isfinite(temperature) or not temperature > 0:
        raise OracleError("InvalidParameter", parameter="temperature (must be finite and > 0)")
    return _softmax_rows(x, axis, temperature, "softmax_temperature")


def _softmax_rows(x: np.ndarray, axis: int, temperature: float, operation: str) -> np.ndarray:
    rank = x.ndim
    ax = axis + rank if axis < 0 else axis
    if not 0 <= ax < rank:
        raise OracleError("AxisOutOfBounds", axis=axis, rank=rank)
    if x.size == 0:
        return np.zeros_like(x)
    moved = np.ascontiguousarray(np.moveaxis(x, ax, -1))
    rows, length = moved.size // moved.shape[-1], moved.shape[-1]
    out = np.empty_like(moved)
    t = x.dtype.type(temperature)
    bad = getattr(lib, f"kxo_softmax_rows_{_t(x.dtype)}")(_p(moved), _p(out), rows, length, t)
    if bad >= 0:
        # First nonfinite in the reference scan order (outer C order, then axis).
        r, pos = divmod(int(bad), length)
        outer = list(np.unravel_index(r, moved.shape[:-1])) if moved.ndim > 1 else []
        idx = outer[:ax] + [pos] + outer[ax:]
        raise OracleError("NonFiniteInput", operation=operation, indices=[int(i) for i in idx])
    return np.moveaxis(out, -1, ax)


# ---------------------------------------------------------------------------
# attention products (matmul -> softmax_temperature -> matmul)
# ---------------------------------------------------------------------------
def attention_truth(q: np.ndarray, k: np.ndarray, v: np.ndarray, temperature: float, rows=None):
    """Attention of f32 inputs q [nb, sq, d], k [nb, sk, d], v [nb, sk, dv]
    in extended precision: S by the compensated product, P = exp((S - max)/T)
    / sum in long double, O = P v in f64.  Returns (O, P|v| row sums per
    output, max over keys of sum|q k|) for the selected query rows."""
    nb, sq, d = q.shape
    rows = list(range(sq)) if rows is None else list(rows)
    outs, absv, sabs = [], [], []
    for b in range(nb):
        qb = np.ascontiguousarray(q[b][rows])
        s, ab = gemm_dot2(View.of(qb), View(np.ascontiguousarray(k[b]), (d, k.shape[1]), (1, d)))
        sl = s.astype(np.longdouble)
        e = np.exp((sl - sl.max(axis=1, keepdims=True)) / np.longdouble(temperature))
        p = (e / e.sum(axis=1, keepdims=True)).astype(np.float64)
        vb = v[b].astype(np.float64)
        outs.append(p @ vb)
        absv.append(p @ np.abs(vb))
        sabs.append(ab.max(axis=1))
    return np.stack(outs), np.stack(absv), np.stack(sabs)


# ---------------------------------------------------------------------------
# backward products
# ---------------------------------------------------------------------------
def conv2d_backward(x: View, w: View, dy: np.ndarray, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1):
    """conv2d_backward (neural.rs:379-430): (dx, dw) by the reference's loop,
    every contribution `dy * w` / `dy * x` added separately rounded."""
    yd, xd, xs, wd, ws, yda, opt = _conv_args(x, w, stride, padding, dilation, groups)
    if list(dy.shape) != list(yd):
        raise OracleError("InvalidParameter", parameter="gradient shape differs from forward output")
    dx = np.zeros(x.dims, dtype=x.dtype)
    dw = np.zeros(w.dims, dtype=x.dtype)
    if dy.size:
        g = np.ascontiguousarray(dy, dtype=x.dtype)
        getattr(lib, f"kxo_conv2d_backward_{_t(x.dtype)}")(x.ptr(), _p(xd), _p(xs), w.ptr(), _p(wd), _p(ws), _p(g),
                                                           _p(yda), _p(dx), _p(dw), _p(opt))
    return dx, dw


def _unbroadcast(full: np.ndarray, dims) -> np.ndarray:
    """Sum a gradient over the batch axes its operand was broadcast along
    (missing leading axes and axes of extent 1), to the operand's dims."""
    lead = full.ndim - len(dims)
    out = full.sum(axis=tuple(range(lead))) if lead else full
    axes = tuple(i for i, d in enumerate(dims) if d == 1 and out.shape[i] != 1)
    if axes:
        out = out.sum(axis=axes, keepdims=True)
    return out.reshape(dims)


def matmul_backward(a: np.ndarray, b: np.ndarray, g: np.ndarray):
    """Tape::matmul's VJP (crates/kernix/src/autograd.rs:622-690) in float64:
    dA = G B^T and dB = A^T G on the vector-extended operands, each summed
    back over the batch axes its operand was broadcast along.  Exact for
    dyadic data whose sums stay within 53 bits."""
    out_dims, _, (av, bv, _, _, m, k, n) = matmul_shape(a.shape, b.shape)
    if list(g.shape) != list(out_dims):
        raise OracleError("InvalidParameter", parameter="gradient shape differs from forward output")
    a2 = a.astype(np.float64).reshape((1, k) if av else a.shape)
    b2 = b.astype(np.float64).reshape((k, 1) if bv else b.shape)
    seed = g.astype(np.float64).reshape(tuple(out_dims[:len(out_dims) - (not av) - (not bv)]) + (m, n))
    da = np.matmul(seed, np.swapaxes(b2, -1, -2))
    db = np.matmul(np.swapaxes(a2, -1, -2), seed)
    da = _unbroadcast(da, (1, k) if av else a.shape).reshape(a.shape)
    db = _unbroadcast(db, (k, 1) if bv else b.shape).reshape(b.shape)
    return da, db


def tensordot(a: np.ndarray, b: np.ndarray, a_axes, b_axes) -> np.ndarray:
    """tensordot (ops/linalg_extra.rs:164-276): validation in the reference
    order, then every output element summed over the contraction index space
    in C order (`sum += a * b`, separately rounded) -- the ordered matrix
    product of a permuted to [free, contracted] and b to [contracted, free]."""
    if len(a_axes) != len(b_axes):
        raise OracleError("ContractAxesMismatch", left=len(a_axes), right=len(b_axes))
    cl, cr, al, ar = set(), set(), [], []
    for l, r in zip(a_axes, b_axes):
        li = l + a.ndim if l < 0 else l
        if not 0 <= li < a.ndim:
            raise OracleError("AxisOutOfBounds", axis=l, rank=a.ndim)
        ri = r + b.ndim if r < 0 else r
        if not 0 <= ri < b.ndim:
            raise OracleError("AxisOutOfBounds", axis=r, rank=b.ndim)
        if li in cl or ri in cr:
            raise OracleError("DuplicateAxis", axis=li if li in cl else ri)
        if a.shape[li] != b.shape[ri]:
            raise OracleError("ContractDimensionMismatch", left=a.shape[li], right=b.shape[ri])
        cl.add(li)
        cr.add(ri)
        al.append(li)
        ar.append(ri)
    fl = [i for i in range(a.ndim) if i not in cl]
    fr = [i for i in range(b.ndim) if i not in cr]
    out_dims = [a.shape[i] for i in fl] + [b.shape[i] for i in fr]
    m = int(np.prod([a.shape[i] for i in fl]))
    k = int(np.prod([a.shape[i] for i in al]))
    n = int(np.prod([b.shape[i] for i in fr]))
    if int(np.prod(out_dims)) == 0:
        return np.zeros(out_dims, dtype=a.dtype)
    a2 = np.ascontiguousarray(np.transpose(a, fl + al)).reshape(m, k)
    b2 = np.ascontiguousarray(np.transpose(b, ar + fr)).reshape(k, n)
    return matmul_reference(View.of(a2), View.of(b2)).reshape(out_dims)
