"""kernix_b200 -- Kernix's dense matmul path on B200 (sm_100a), Python mirror.

The public names follow the reference crate (kernix-ops):

* ``matmul(a, b)``                 ops/linalg.rs:31-44  (NumPy matmul semantics)
* ``conv2d(x, w, Conv2dOptions())`` neural.rs:177-183
* ``softmax_temperature(s, axis, t)`` ops/math_extra.rs:544-557
* ``softmax(s, axis)``             ops/math.rs:531-536
* ``attention(q, kt, v, t)``       matmul + softmax_temperature + matmul in one call
* ``MatrixInput`` / ``try_dense_matmul`` / ``try_strided_matmul``
                                   ops/matmul_element.rs:14-44, 262-300
* ``CudaExecutor``                 the ``MatmulDevice`` / ``Device`` plug point
                                   (execution.rs:25-36, kernix-core device.rs:22-35)

Device tensors are torch CUDA tensors (plumbing only) or :class:`TensorView`
descriptors over a device buffer, which can also express the negative strides
torch cannot.  Every computation runs in ``libkernix_b200.so``; errors surface
as :class:`OpsError` subclasses carrying the reference variant's fields.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import threading
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from . import _abi
from ._abi import (  # noqa: F401  (re-exported error types)
    AxisOutOfBounds, BroadcastIncompatible, CapacityOverflow, ContractAxesMismatch, ContractDimensionMismatch,
    CudaError, DeviceTimeout, DimensionOverflow, DuplicateAxis, ElementCountOverflow, ExactRank, InvalidParameter, InvalidRank, KxConv2dOptions,
    KxError, KxMatrix, KxTensor, LayoutError, NoDevice, NonFiniteInput, OpsError, OverlappingOutput,
    Unsupported, raise_for, u64_array)

lib = _abi.lib
MAX_RANK = _abi.MAX_RANK

__all__ = [
    "matmul", "matmul_reference", "matmul_shape", "matmul_into", "conv2d", "conv2d_reference", "conv2d_shape",
    "Conv2dOptions", "attention", "attention_into", "matmul_backward", "conv2d_backward", "tensordot", "softmax", "softmax_into", "softmax_temperature", "matmul_into_replicated", "conv2d_into", "softmax_temperature_into",
    "MatrixInput", "try_dense_matmul", "try_strided_matmul", "TensorView", "CudaExecutor", "Handle",
    "handle", "OpsError", "InvalidRank", "ContractDimensionMismatch", "BroadcastIncompatible",
    "ElementCountOverflow", "DimensionOverflow", "LayoutError", "InvalidParameter", "ExactRank",
    "NonFiniteInput", "AxisOutOfBounds", "OverlappingOutput", "CudaError", "NoDevice", "Unsupported",
    "CapacityOverflow", "ContractAxesMismatch", "DuplicateAxis", "using", "Config", "Context", "ConfigError",
]


# ---------------------------------------------------------------------------
# handles
# ---------------------------------------------------------------------------
class Handle:
    """One library handle bound to a CUDA device (kx_create/kx_destroy)."""

    def __init__(self, device: int = 0):
        self.device = device
        ptr = C.c_void_p()
        err = KxError()
        raise_for(lib.kx_create(device, C.byref(ptr), C.byref(err)), err)
        self._h = ptr
        self._stream = 0            # the raw stream the library handle orders work on

    @classmethod
    def adopt(cls, ptr: C.c_void_p, device: int) -> "Handle":
        """Own a handle the library created elsewhere (kx_context_create)."""
        h = cls.__new__(cls)
        h.device = device
        h._h = ptr
        h._stream = 0
        return h

    @property
    def ptr(self) -> C.c_void_p:
        return self._h

    def close(self) -> None:
        if self._h:
            lib.kx_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter teardown order varies
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream) -> None:
        """Order later work on ``stream`` (a torch.cuda.Stream or raw cudaStream_t)."""
        raw = int(getattr(stream, "cuda_stream", stream) or 0)
        if raw != self._stream:     # every call binds the current stream: skip the unchanged case
            lib.kx_set_stream(self._h, C.c_void_p(raw))
            self._stream = raw

    def set_f32_variant(self, variant: int) -> None:
        raise_for(lib.kx_set_f32_variant(self._h, int(variant)), None)

    def set_f64_variant(self, variant: int) -> None:
        """0 = automatic, 1 = SIMT DFMA, 2 = FP64 tensor pipe (DMMA)."""
        raise_for(lib.kx_set_f64_variant(self._h, int(variant)), None)

    def set_ordered_matmul(self, ordered: bool) -> None:
        """Increasing-k, separately rounded accumulation (bitwise equal to
        matmul_reference); see CpuExecutor::with_ordered_matmul."""
        raise_for(lib.kx_set_ordered_matmul(self._h, int(bool(ordered))), None)

    @property
    def ordered_matmul(self) -> bool:
        return bool(lib.kx_ordered_matmul(self._h))

    def synchronize(self) -> None:
        err = KxError()
        raise_for(lib.kx_synchronize(self._h, C.byref(err)), err)

    def diag_expire_next_gemm(self, wait_ns: int) -> None:
        """Diagnostic: the next one-SM split-TF32 GEMM on this handle issues no
        copies and bounds its waits by ``wait_ns`` (1 ms .. 2 s), so they expire
        and the next ``synchronize`` raises DeviceTimeout."""
        raise_for(lib.kx_diag_expire_next_gemm(self._h, int(wait_ns)), None)

    @property
    def launches(self) -> int:
        return int(lib.kx_launch_count(self._h))

    @property
    def last_kernel(self) -> str:
        return lib.kx_last_kernel(self._h).decode()


_handles: dict[int, Handle] = {}
_active = threading.local()


@contextlib.contextmanager
def using(h: Handle):
    """Route this thread's calls on ``h.device`` through ``h`` (a context's
    handle with its own variants and ordered mode) instead of the default."""
    stack = getattr(_active, "handles", None)
    if stack is None:
        stack = _active.handles = {}
    prev = stack.get(h.device)
    stack[h.device] = h
    try:
        yield h
    finally:
        if prev is None:
            del stack[h.device]
        else:
            stack[h.device] = prev


def handle(device: int | None = None) -> Handle:
    """The per-process default handle of ``device`` (torch's current device by default)."""
    import torch
    if device is None:
        device = torch.cuda.current_device()
    h = _handles.get(device)
    if h is None:
        h = Handle(device)
        _handles[device] = h
    return h


# ---------------------------------------------------------------------------
# device tensor descriptors
# ---------------------------------------------------------------------------
@dataclass
class TensorView:
    """A strided view over a device buffer: element (i0..) at
    ``buffer[origin + sum(i_j * strides[j])]`` (kernix_core::Layout semantics,
    signed and zero strides allowed)."""

    buffer: "object"            # 1-d contiguous torch CUDA tensor
    dims: Sequence[int]
    strides: Sequence[int]
    origin: int = 0

    @property
    def dtype(self):
        return self.buffer.dtype

    @property
    def device(self):
        return self.buffer.device

    @property
    def shape(self):
        return tuple(self.dims)


def _descriptor(t) -> KxTensor:
    d = KxTensor()
    if isinstance(t, TensorView):
        buf = t.buffer
        d.data = buf.data_ptr()
        d.storage_len = buf.numel()
        d.origin = int(t.origin)
        dims, strides = [int(n) for n in t.dims], [int(s) for s in t.strides]
    else:
        st = t.untyped_storage()
        d.data = st.data_ptr()
        d.storage_len = st.nbytes() // t.element_size()
        d.origin = t.storage_offset()
        dims, strides = t.shape, t.stride()
    rank = len(dims)
    if rank != len(strides):
        raise LayoutError("stride rank mismatch", kind="StrideRankMismatch")
    if rank > MAX_RANK:
        raise Unsupported(f"rank {rank} above {MAX_RANK}")
    d.rank = rank
    d.dims[:rank] = dims            # one slice store per array: the call path's largest host cost
    d.strides[:rank] = strides
    return d


def _device_index(t) -> int:
    dev = t.device
    if dev.type != "cuda":
        raise NoDevice(f"expected a CUDA tensor, got {dev}")
    return dev.index if dev.index is not None else 0


def _current_stream(dev: int) -> int:
    """torch's current stream on ``dev`` as a raw cudaStream_t (the raw query
    when this torch build has it: no Stream object per call)."""
    import torch
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return int(raw(dev)) if raw is not None else int(torch.cuda.current_stream(dev).cuda_stream)


def _bind(t) -> Handle:
    dev = _device_index(t)
    h = getattr(_active, "handles", {}).get(dev) or handle(dev)
    h.set_stream(_current_stream(dev))
    return h


def _empty(dims, dtype, device):
    """Allocate a C-contiguous output; byte sizes above isize::MAX fail like
    kernix's Tensor allocation (StorageError::CapacityOverflow)."""
    import torch
    n = 1
    for d in dims:
        n *= int(d)
    esize = torch.empty((), dtype=dtype).element_size()
    if n * esize > (1 << 63) - 1:
        raise CapacityOverflow("output allocation exceeds isize::MAX bytes", len=n, element_size=esize)
    return torch.empty(tuple(dims), dtype=dtype, device=device)


def _fn(name: str, dtype):
    import torch
    if dtype == torch.float32:
        return getattr(lib, name + "_f32")
    if dtype == torch.float64:
        return getattr(lib, name + "_f64")
    raise Unsupported(f"dtype {dtype}: the device path computes f32 and f64")


# ---------------------------------------------------------------------------
# matmul
# ---------------------------------------------------------------------------
def matmul_shape(a_dims: Sequence[int], b_dims: Sequence[int]) -> tuple[int, ...]:
    """Output dims of ``matmul`` with the reference's error order (host only)."""
    out = (C.c_uint64 * MAX_RANK)()
    rank = C.c_uint32()
    err = KxError()
    rc = lib.kx_matmul_shape(u64_array(a_dims), len(a_dims), u64_array(b_dims), len(b_dims), C.byref(rank), out,
                             C.byref(err))
    raise_for(rc, err)
    return tuple(out[:rank.value])


def matmul(a, b):
    """NumPy-style matmul of two device tensors (vectors, matrices, broadcast
    batches; any signed/zero strides).  Returns a new C-contiguous tensor."""
    import torch
    if a.dtype != b.dtype:
        raise InvalidParameter("matmul: operand dtypes differ", operation="matmul", parameter="dtype")
    out_dims = matmul_shape(a.shape, b.shape)
    out = _empty(out_dims, a.dtype, a.device)
    matmul_into(a, b, out)
    return out


def matmul_into(a, b, out) -> None:
    """Write ``matmul(a, b)`` into an existing C-contiguous device tensor."""
    fn = _fn("kx_matmul", a.dtype)
    h = _bind(a)
    err = KxError()
    da, db, do = _descriptor(a), _descriptor(b), _descriptor(out)
    raise_for(fn(h.ptr, C.byref(da), C.byref(db), C.byref(do), C.byref(err)), err)


def matmul_into_replicated(a, b, out, out_mc: int) -> None:
    """``matmul_into`` whose stores go through ``out_mc``, the NVLink multicast
    address of ``out``'s first element: the product lands in the copy of
    ``out`` on every GPU bound to the multicast object."""
    fn = _fn("kx_matmul_replicated", a.dtype)
    h = _bind(a)
    err = KxError()
    da, db, do = _descriptor(a), _descriptor(b), _descriptor(out)
    # out_mc addresses out's first element; the library adds the origin itself
    base = int(out_mc) - do.origin * out.element_size()
    raise_for(fn(h.ptr, C.byref(da), C.byref(db), C.byref(do), C.c_void_p(base), C.byref(err)), err)


class _Ordered:
    """Run the enclosed device calls of ``h`` in ordered mode."""

    def __init__(self, h: Handle):
        self.h = h

    def __enter__(self):
        self.prev = self.h.ordered_matmul
        self.h.set_ordered_matmul(True)
        return self.h

    def __exit__(self, *exc):
        self.h.set_ordered_matmul(self.prev)
        return False


def matmul_reference(a, b):
    """``matmul_reference`` on the device: every output accumulated in
    increasing k with separately rounded multiply and add (linalg.rs:57-64),
    so the bits equal Kernix's ordered CPU result."""
    with _Ordered(_bind(a)):
        return matmul(a, b)


# ---------------------------------------------------------------------------
# conv2d
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class Conv2dOptions:
    """Conv2dOptions (neural.rs:22-42); defaults match the reference."""

    stride: tuple[int, int] = (1, 1)
    padding: tuple[int, int] = (0, 0)
    dilation: tuple[int, int] = (1, 1)
    groups: int = 1

    def to_c(self) -> KxConv2dOptions:
        o = KxConv2dOptions()
        for i in range(2):
            o.stride[i] = int(self.stride[i])
            o.padding[i] = int(self.padding[i])
            o.dilation[i] = int(self.dilation[i])
        o.groups = int(self.groups)
        return o


def conv2d_shape(input_dims: Sequence[int], weight_dims: Sequence[int],
                 options: Conv2dOptions = Conv2dOptions()) -> tuple[int, int, int, int]:
    out = (C.c_uint64 * 4)()
    err = KxError()
    o = options.to_c()
    rc = lib.kx_conv2d_shape(u64_array(input_dims), len(input_dims), u64_array(weight_dims), len(weight_dims),
                             C.byref(o), out, C.byref(err))
    raise_for(rc, err)
    return tuple(int(x) for x in out)


def conv2d(x, w, options: Conv2dOptions = Conv2dOptions()):
    """NCHW cross-correlation with weights [out, in/groups, kh, kw]."""
    out_dims = conv2d_shape(x.shape, w.shape, options)
    out = _empty(out_dims, x.dtype, x.device)
    conv2d_into(x, w, out, options)
    return out


def conv2d_into(x, w, out, options: Conv2dOptions = Conv2dOptions()) -> None:
    """``conv2d`` written into an existing C-contiguous device tensor."""
    fn = _fn("kx_conv2d", x.dtype)
    h = _bind(x)
    err = KxError()
    o = options.to_c()
    dx, dw, do = _descriptor(x), _descriptor(w), _descriptor(out)
    raise_for(fn(h.ptr, C.byref(dx), C.byref(dw), C.byref(o), C.byref(do), C.byref(err)), err)


def conv2d_reference(x, w, options: Conv2dOptions = Conv2dOptions()):
    """``conv2d_reference`` on the device: the ordered scalar loop
    (neural.rs:188-198, 341-357), bitwise equal to Kernix's CPU result."""
    with _Ordered(_bind(x)):
        return conv2d(x, w, options)


def tensordot(a, b, a_axes: Sequence[int], b_axes: Sequence[int]):
    """tensordot (ops/linalg_extra.rs:164-276): contract the axis pairs
    (a_axes[i], b_axes[i]); the result has a's free axes then b's.  One GEMM
    on the device (bit for bit the reference's sums in ordered mode)."""
    ra, rb = len(a.shape), len(b.shape)
    fa = [i for i in range(ra) if i not in {(x + ra if x < 0 else x) for x in a_axes}]
    fb = [i for i in range(rb) if i not in {(x + rb if x < 0 else x) for x in b_axes}]
    dims = [a.shape[i] for i in fa] + [b.shape[i] for i in fb]
    ok = len(a_axes) == len(b_axes) and all(-ra <= x < ra for x in a_axes) and all(-rb <= x < rb for x in b_axes)
    out = _empty(tuple(dims) if ok else (), a.dtype, a.device)
    fn = _fn("kx_tensordot", a.dtype)
    h = _bind(a)
    la = (C.c_int64 * max(1, len(a_axes)))(*[int(x) for x in a_axes])
    lb = (C.c_int64 * max(1, len(b_axes)))(*[int(x) for x in b_axes])
    err = KxError()
    ta, tb, to = _descriptor(a), _descriptor(b), _descriptor(out)
    raise_for(fn(h.ptr, C.byref(ta), C.byref(tb), la, len(a_axes), lb, len(b_axes), C.byref(to), C.byref(err)), err)
    return out


# ---------------------------------------------------------------------------
# backward products
# ---------------------------------------------------------------------------
def matmul_backward(a, b, grad, need_a: bool = True, need_b: bool = True):
    """Tape::matmul's VJP (autograd.rs:622-690): (grad . b^T, a^T . grad), each
    summed back over the batch axes its operand was broadcast along; a
    gradient not asked for is None."""
    fn = _fn("kx_matmul_backward", a.dtype)
    h = _bind(a)
    da = _empty(tuple(a.shape), a.dtype, a.device) if need_a else None
    db = _empty(tuple(b.shape), b.dtype, b.device) if need_b else None
    err = KxError()
    ta, tb, tg = _descriptor(a), _descriptor(b), _descriptor(grad)
    oa = C.byref(_descriptor(da)) if da is not None else None
    ob = C.byref(_descriptor(db)) if db is not None else None
    raise_for(fn(h.ptr, C.byref(ta), C.byref(tb), C.byref(tg), oa, ob, C.byref(err)), err)
    return da, db


def conv2d_backward(x, w, grad, options: Conv2dOptions = Conv2dOptions()):
    """conv2d_backward (neural.rs:379-430): (grad_input, grad_weight), bit for
    bit the reference loop's sums."""
    fn = _fn("kx_conv2d_backward", x.dtype)
    h = _bind(x)
    dx = _empty(tuple(x.shape), x.dtype, x.device)
    dw = _empty(tuple(w.shape), w.dtype, w.device)
    err = KxError()
    o = options.to_c()
    tx, tw, tg, ox, ow = (_descriptor(t) for t in (x, w, grad, dx, dw))
    raise_for(fn(h.ptr, C.byref(tx), C.byref(tw), C.byref(tg), C.byref(o), C.byref(ox), C.byref(ow), C.byref(err)),
              err)
    return dx, dw


# ---------------------------------------------------------------------------
# softmax_temperature
# ---------------------------------------------------------------------------
def softmax_temperature(src, axis: int, temperature: float):
    """Softmax of ``(x - max) / temperature`` along ``axis`` (negative axes
    count from the end).  Nonfinite input raises NonFiniteInput."""
    out = _empty(tuple(src.shape), src.dtype, src.device)
    softmax_temperature_into(src, axis, temperature, out)
    return out


def softmax_temperature_into(src, axis: int, temperature: float, out) -> None:
    """``softmax_temperature`` written into an existing C-contiguous tensor."""
    fn = _fn("kx_softmax_temperature", src.dtype)
    h = _bind(src)
    err = KxError()
    ds, do = _descriptor(src), _descriptor(out)
    raise_for(fn(h.ptr, C.byref(ds), int(axis), float(temperature), C.byref(do), C.byref(err)), err)


def attention(q, kt, v, temperature: float):
    """``matmul(softmax_temperature(matmul(q, kt), -1, temperature), v)`` in one
    call, with the composition's errors.  ``kt`` is the transposed view of k
    ([.., d, sk]); with head dim 128, equal batch dims and unit strides along
    the head dimension one fused tensor-core kernel runs without writing the
    scores."""
    import math
    s_dims = matmul_shape(q.shape, kt.shape)
    t = float(temperature)
    if not s_dims or not (math.isfinite(t) and t > 0):
        # softmax_temperature's own errors come before matmul(P, v)'s: the
        # library reports them without looking at the output
        attention_into(q, kt, v, t, _empty((), q.dtype, q.device))
    out = _empty(matmul_shape(s_dims, v.shape), q.dtype, q.device)
    attention_into(q, kt, v, t, out)
    return out


def attention_into(q, kt, v, temperature: float, out) -> None:
    """``attention`` written into an existing C-contiguous f32 tensor."""
    import torch
    if q.dtype != torch.float32:
        raise Unsupported(f"dtype {q.dtype}: attention runs in f32")
    h = _bind(q)
    err = KxError()
    dq, dk, dv, do = _descriptor(q), _descriptor(kt), _descriptor(v), _descriptor(out)
    raise_for(lib.kx_attention_f32(h.ptr, C.byref(dq), C.byref(dk), C.byref(dv), float(temperature), C.byref(do),
                                   C.byref(err)), err)


def softmax(src, axis: int):
    """Softmax of ``x - max`` along ``axis`` (ops/math.rs:531-536); nonfinite
    input raises NonFiniteInput with operation ``"softmax"``."""
    out = _empty(tuple(src.shape), src.dtype, src.device)
    softmax_into(src, axis, out)
    return out


def softmax_into(src, axis: int, out) -> None:
    """``softmax`` written into an existing C-contiguous tensor."""
    fn = _fn("kx_softmax", src.dtype)
    h = _bind(src)
    err = KxError()
    ds, do = _descriptor(src), _descriptor(out)
    raise_for(fn(h.ptr, C.byref(ds), int(axis), C.byref(do), C.byref(err)), err)


# ---------------------------------------------------------------------------
# MatmulElement hooks over HOST buffers (numpy)
# ---------------------------------------------------------------------------
def _np_kind(arr: np.ndarray) -> str:
    if arr.dtype == np.float32:
        return "f32"
    if arr.dtype == np.float64:
        return "f64"
    raise Unsupported(f"dtype {arr.dtype}: hooks exist for f32 and f64")


class MatrixInput:
    """Validated borrowed rank-two host matrix (matmul_element.rs:262-300).

    ``data`` is a 1-d numpy buffer; element (i, j) is ``data[origin + i*strides[0]
    + j*strides[1]]``.  Construction validates the span exactly like
    ``MatrixInput::new``; singleton strides are normalised to zero."""

    def __init__(self, data: np.ndarray, dims: Sequence[int], strides: Sequence[int], origin: int):
        if data.ndim != 1 or not data.flags.c_contiguous:
            raise LayoutError("MatrixInput storage must be a 1-d contiguous buffer", kind="Storage")
        self.data = data
        self._dims = (int(dims[0]), int(dims[1]))
        self._strides = [int(strides[0]), int(strides[1])]
        self.origin = int(origin)
        m = self._c()
        err = KxError()
        raise_for(lib.kx_matrix_validate(C.byref(m), data.itemsize, C.byref(err)), err)
        for axis in range(2):
            if self._dims[axis] <= 1:
                self._strides[axis] = 0

    def _c(self) -> KxMatrix:
        m = KxMatrix()
        m.data = self.data.ctypes.data if self.data.size else None
        m.storage_len = self.data.size
        m.dims[0], m.dims[1] = self._dims
        m.strides[0], m.strides[1] = self._strides
        m.origin = self.origin
        return m

    def dims(self):
        return list(self._dims)

    def strides(self):
        return list(self._strides)

    def storage(self):
        return self.data


def _host_handle(device: int | None) -> Handle:
    return handle(0 if device is None else device)


def try_dense_matmul(a: np.ndarray, b: np.ndarray, out: np.ndarray, m: int, k: int, n: int,
                     device: int | None = None) -> bool:
    """MatmulElement::try_dense_matmul on host buffers: False means nothing was
    written (any extent mismatch); True means all m*n outputs were written."""
    kind = _np_kind(out)
    if a.dtype != out.dtype or b.dtype != out.dtype:
        return False
    for arr in (a, b, out):
        if not arr.flags.c_contiguous:
            return False
    if m < 0 or k < 0 or n < 0 or max(m, k, n) >= 1 << 64:
        return False
    h = _host_handle(device)
    fn = getattr(lib, f"kx_try_dense_matmul_{kind}")
    rc = fn(h.ptr, a.ctypes.data, a.size, b.ctypes.data, b.size, out.ctypes.data, out.size, m, k, n)
    return rc == _abi.KX_OK


def try_strided_matmul(a: MatrixInput, b: MatrixInput, out: np.ndarray, device: int | None = None) -> bool:
    """MatmulElement::try_strided_matmul on validated host matrices."""
    kind = _np_kind(out)
    if a.data.dtype != out.dtype or b.data.dtype != out.dtype or not out.flags.c_contiguous:
        return False
    h = _host_handle(device)
    fn = getattr(lib, f"kx_try_strided_matmul_{kind}")
    ma, mb = a._c(), b._c()
    rc = fn(h.ptr, C.byref(ma), C.byref(mb), out.ctypes.data, out.size)
    return rc == _abi.KX_OK


# ---------------------------------------------------------------------------
# Device / MatmulDevice mirror
# ---------------------------------------------------------------------------
@dataclass
class CudaExecutor:
    """A ``MatmulDevice`` for one GPU: device-owned buffers, explicit
    transfers, and matmul that never changes device or layout."""

    device: int = 0
    _handle: Handle | None = field(default=None, repr=False)

    def name(self) -> str:
        return f"cuda:{self.device}"

    @property
    def h(self) -> Handle:
        if self._handle is None:
            self._handle = handle(self.device)
        return self._handle

    def upload(self, values: np.ndarray):
        import torch
        t = torch.from_numpy(np.ascontiguousarray(values)).to(f"cuda:{self.device}")
        torch.cuda.synchronize(self.device)
        return t

    def download(self, buffer) -> np.ndarray:
        if _device_index(buffer) != self.device:
            raise InvalidParameter("buffer belongs to another device", operation="download", parameter="buffer")
        return buffer.detach().cpu().numpy()

    def synchronize(self) -> None:
        import torch
        torch.cuda.synchronize(self.device)

    def matmul(self, left, right):
        for t in (left, right):
            if _device_index(t) != self.device:
                raise InvalidParameter("tensor belongs to another device", operation="matmul", parameter="device")
        with using(self.h):
            return matmul(left, right)

    def matmul_into(self, left, right, out) -> None:
        """CpuExecutor::matmul_into's contract (execution.rs:149-240) on the
        device: the caller's C-contiguous output is reused, nothing allocated."""
        for t in (left, right, out):
            if _device_index(t) != self.device:
                raise InvalidParameter("tensor belongs to another device", operation="matmul_into",
                                       parameter="device")
        with using(self.h):
            matmul_into(left, right, out)


from .config import Config, ConfigError, Context  # noqa: E402  (needs Handle and CudaExecutor above)
