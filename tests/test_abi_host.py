"""Host side of the C ABI (CPU only, no device calls).

Covers: the library loads and exports every function include/kernix_b200.h
declares; shape planning and layout validation mirror the reference's checks
and error order; the MatmulElement hooks decline malformed extents before any
write.
"""
import ctypes as C
import itertools
import json
import re
from pathlib import Path

import numpy as np
import pytest

import kernix_b200 as kx
import oracle
from kernix_b200 import _abi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "kernix_b200.h"
KATS = json.loads((ROOT / "tests" / "golden" / "kats.json").read_text())
USIZE_MAX = (1 << 64) - 1
ISIZE_MAX = (1 << 63) - 1
ISIZE_MIN = -(1 << 63)


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    names = declared_functions()
    assert len(names) >= 25
    lib = C.CDLL(str(_abi.LIB_PATH))
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_abi.EXPORTED), set(names) ^ set(_abi.EXPORTED)
    assert _abi.lib.kx_abi_version() == 1


def test_no_device_here_is_reported_not_faked():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    count = C.c_int(-1)
    assert _abi.lib.kx_device_count(C.byref(count)) == 0 and count.value == 0
    with pytest.raises(kx.NoDevice):
        kx.Handle(0)


def _oracle_outcome(a, b):
    try:
        return ("ok", tuple(oracle.matmul_shape(a, b)[0]))
    except oracle.OracleError as e:
        return (e.kind, tuple(sorted(e.fields.items())))


def _abi_outcome(a, b):
    try:
        return ("ok", kx.matmul_shape(a, b))
    except kx.OpsError as e:
        kind = {"InvalidRank": "InvalidRank"}.get(type(e).__name__, type(e).__name__)
        fields = {k: v for k, v in e.fields.items() if k != "operation"}
        return (kind, tuple(sorted(fields.items())))


def test_matmul_shape_matches_oracle_on_a_grid():
    dims = [[], [0], [1], [3], [2, 3], [3, 2], [1, 3], [3, 1], [2, 1, 3], [4, 3, 2], [1, 4, 2, 3], [5, 1, 3, 3],
            [2, 0, 3], [0, 3], [3, 0]]
    for a, b in itertools.product(dims, repeat=2):
        assert _abi_outcome(a, b) == _oracle_outcome(a, b), (a, b)


@pytest.mark.parametrize("case", KATS["matmul_errors"], ids=lambda c: c["error"])
def test_matmul_error_known_answers_through_abi(case):
    if case["error"] == "CapacityOverflow":
        dims = kx.matmul_shape(case["a_dims"], case["b_dims"])
        import torch
        with pytest.raises(kx.CapacityOverflow) as e:
            kx._empty(dims, torch.float64, "meta")
        assert e.value.fields == case["fields"]
        return
    with pytest.raises(kx.OpsError) as e:
        kx.matmul_shape(case["a_dims"], case["b_dims"])
    assert type(e.value).__name__ == case["error"]
    for k, v in case["fields"].items():
        assert getattr(e.value, k) == v


def test_matmul_shape_overflow_and_huge_empty():
    assert kx.matmul_shape([USIZE_MAX, 0], [0, 0]) == (USIZE_MAX, 0)
    with pytest.raises(kx.ElementCountOverflow) as e:
        kx.matmul_shape([USIZE_MAX, 2, 3], [1, 3, 2])
    assert (e.value.axis, e.value.accumulated, e.value.dim) == (1, USIZE_MAX, 2)
    with pytest.raises(kx.BroadcastIncompatible) as e:
        kx.matmul_shape([2, 3, 4, 5], [3, 3, 5, 6])
    assert (e.value.axis, e.value.left, e.value.right) == (1, 3, 3) or (e.value.axis, e.value.left) == (0, 2)


def test_conv_shape_matches_reference_errors():
    c = KATS["conv_errors"]
    for case in c["cases"]:
        kw = {k: tuple(v) if isinstance(v, list) else v for k, v in case["options"].items()}
        opts = kx.Conv2dOptions(**kw)
        if "error" in case:
            with pytest.raises(kx.OpsError) as e:
                kx.conv2d_shape(c["x_dims"], c["w_dims"], opts)
            assert type(e.value).__name__ == case["error"]
        else:
            assert list(kx.conv2d_shape(c["x_dims"], c["w_dims"], opts)) == case["out_dims"]
    with pytest.raises(kx.ExactRank) as e:
        kx.conv2d_shape([1, 2, 3], [1, 2, 1, 1])
    assert (e.value.expected, e.value.actual) == (4, 3)
    assert kx.conv2d_shape([64, 128, 56, 56], [256, 128, 3, 3], kx.Conv2dOptions(padding=(1, 1))) == (64, 256, 56, 56)


def _tensor(dims, strides, origin, storage_len, data=0x1000):
    t = _abi.KxTensor()
    t.data = data
    t.storage_len = storage_len
    t.origin = origin
    t.rank = len(dims)
    for i, (d, s) in enumerate(zip(dims, strides)):
        t.dims[i] = d
        t.strides[i] = s
    return t


def _validate(dims, strides, origin, storage_len, es=8):
    err = _abi.KxError()
    t = _tensor(dims, strides, origin, storage_len)
    rc = _abi.lib.kx_validate_tensor(C.byref(t), es, C.byref(err))
    return rc, err


def test_layout_validation_mirrors_checked_span():
    assert _validate([2, 3], [3, 1], 0, 6)[0] == 0
    rc, err = _validate([2, 3], [3, 1], 0, 5)
    assert rc == _abi.KX_E_LAYOUT and err.values[0] == 4 and (err.values[1], err.values[2]) == (6, 5)
    rc, err = _validate([2, 3], [-3, 1], 0, 6)               # reaches index -3
    assert rc == _abi.KX_E_LAYOUT and err.values[0] == 3
    assert _validate([2, 3], [-3, 1], 3, 6)[0] == 0         # reversed rows, origin at last row
    assert _validate([1, 1], [ISIZE_MIN, ISIZE_MIN], 0, 1)[0] == 0   # singleton strides never move
    assert _validate([0, 5], [ISIZE_MIN, 3], 0, 0)[0] == 0  # empty: no span
    rc, err = _validate([3], [ISIZE_MAX], ISIZE_MAX, 1)      # end past usize
    assert rc == _abi.KX_E_LAYOUT and err.values[0] == 2
    rc, err = _validate([2], [1], 0, 1 << 62, es=8)          # byte extent above isize::MAX
    assert rc == _abi.KX_E_LAYOUT and err.values[0] == 5


def test_matrix_input_validation_like_reference():
    """native_kernel_tests.rs:17-28."""
    with pytest.raises(kx.LayoutError):
        kx.MatrixInput(np.array([1.0]), [2, 2], [2, 1], 0)
    m = kx.MatrixInput(np.array([1.0]), [1, 1], [ISIZE_MIN, ISIZE_MIN], 0)
    assert m.strides() == [0, 0] and m.dims() == [1, 1]
    m = kx.MatrixInput(np.arange(6.0), [2, 3], [3, 1], 0)
    assert m.strides() == [3, 1]


@pytest.mark.parametrize("t", ["f32", "f64"])
def test_dense_hook_declines_malformed_extents_without_writes(t):
    """small_matmul_tests.rs:137-151 and native_kernel_tests.rs:17-28."""
    dtype = np.float32 if t == "f32" else np.float64
    fn = getattr(_abi.lib, f"kx_try_dense_matmul_{t}")
    for (m, k, n) in [(4, 4, 16), (USIZE_MAX, 2, 16), (4, USIZE_MAX, 16)]:
        a = np.ones(16, dtype)
        b = np.full(63, 2.0, dtype)
        out = np.full(64, 7.0, dtype)
        rc = fn(None, a.ctypes.data, a.size, b.ctypes.data, b.size, out.ctypes.data, out.size, m, k, n)
        assert rc == _abi.KX_DECLINED
        assert (out == 7.0).all()
    out = np.full(4, 7.0, dtype)
    rc = fn(None, np.ones(1, dtype).ctypes.data, 1, np.full(1, 2.0, dtype).ctypes.data, 1, out.ctypes.data, 4, 2, 2, 2)
    assert rc == _abi.KX_DECLINED and (out == 7.0).all()
    # empty and k == 0 products need no device
    out = np.full(6, 7.0, dtype)
    assert fn(None, None, 0, None, 0, out.ctypes.data, 6, 2, 0, 3) == _abi.KX_OK
    assert (out == 0).all()
    assert fn(None, None, 0, np.ones(3, dtype).ctypes.data, 3, None, 0, 0, 1, 3) == _abi.KX_OK


def test_device_entry_points_validate_before_device_work():
    """Shape and layout errors come back from the host checks even with no GPU."""
    err = _abi.KxError()
    a = _tensor([2, 3], [3, 1], 0, 6)
    b = _tensor([4, 2], [2, 1], 0, 8)
    o = _tensor([2, 2], [2, 1], 0, 4)
    h = C.c_void_p(0x1)   # never dereferenced: validation fails first
    rc = _abi.lib.kx_matmul_f32(h, C.byref(a), C.byref(b), C.byref(o), C.byref(err))
    assert rc == _abi.KX_E_CONTRACT and (err.values[0], err.values[1]) == (3, 4)
    b = _tensor([3, 2], [2, 1], 0, 5)   # storage too small
    rc = _abi.lib.kx_matmul_f32(h, C.byref(a), C.byref(b), C.byref(o), C.byref(err))
    assert rc == _abi.KX_E_LAYOUT
    b = _tensor([3, 2], [2, 1], 0, 6, data=0x1000 + 4 * 100)
    o = _tensor([2, 2], [1, 2], 0, 4, data=0x9000)             # F-order output
    rc = _abi.lib.kx_matmul_f32(h, C.byref(a), C.byref(b), C.byref(o), C.byref(err))
    assert rc == _abi.KX_E_LAYOUT and err.values[0] == 6
    o = _tensor([2, 2], [2, 1], 0, 4, data=0x1000 + 4 * 2)     # overlaps a
    rc = _abi.lib.kx_matmul_f32(h, C.byref(a), C.byref(b), C.byref(o), C.byref(err))
    assert rc == _abi.KX_E_ALIAS
    # softmax: temperature is checked first, then the axis
    s = _tensor([2, 3], [3, 1], 0, 6)
    o = _tensor([2, 3], [3, 1], 0, 6, data=0x9000)
    rc = _abi.lib.kx_softmax_temperature_f32(h, C.byref(s), 5, 0.0, C.byref(o), C.byref(err))
    assert rc == _abi.KX_E_PARAM
    rc = _abi.lib.kx_softmax_temperature_f32(h, C.byref(s), 5, 1.0, C.byref(o), C.byref(err))
    assert rc == _abi.KX_E_AXIS and err.values[1] == 2
    rc = _abi.lib.kx_softmax_temperature_f32(h, C.byref(s), -3, 1.0, C.byref(o), C.byref(err))
    assert rc == _abi.KX_E_AXIS


def test_python_errors_compare_like_rust_values():
    with pytest.raises(kx.ContractDimensionMismatch) as e:
        kx.matmul_shape([2, 3], [4, 2])
    assert e.value == kx.ContractDimensionMismatch(left=3, right=4)
    with pytest.raises(kx.InvalidRank) as e:
        kx.matmul_shape([], [2])
    assert (e.value.minimum, e.value.actual) == (1, 0)


def test_descriptors_carry_layout_exactly():
    """The kx_tensor descriptors the Python mirror builds (host only): torch
    views keep their storage origin and strides, TensorView keeps signed and
    zero strides and numpy integers, rank 0 fills nothing, and a rank above
    KX_MAX_RANK or a stride list of the wrong length is refused before any
    call."""
    import torch
    base = torch.zeros(6, 8, dtype=torch.float64)
    t = base[1:, 2:].transpose(0, 1)
    d = kx._descriptor(t)
    assert (d.rank, d.origin, d.storage_len) == (2, 10, 48)
    assert list(d.dims)[:2] == [6, 5] and list(d.strides)[:2] == [1, 8]
    assert list(d.dims)[2:] == [0] * (kx.MAX_RANK - 2)
    assert d.data == base.untyped_storage().data_ptr()
    buf = torch.zeros(12)
    v = kx.TensorView(buf, (np.int64(3), 4), (-4, np.int64(0)), np.int64(8))
    d = kx._descriptor(v)
    assert (d.rank, d.origin, d.storage_len) == (2, 8, 12)
    assert list(d.dims)[:2] == [3, 4] and list(d.strides)[:2] == [-4, 0]
    d = kx._descriptor(torch.tensor(2.5))
    assert d.rank == 0 and list(d.dims) == [0] * kx.MAX_RANK
    d = kx._descriptor(kx.TensorView(buf, (USIZE_MAX, 0), (1, 1)))
    assert list(d.dims)[:2] == [USIZE_MAX, 0]
    with pytest.raises(kx.Unsupported):
        kx._descriptor(kx.TensorView(buf, (1,) * (kx.MAX_RANK + 1), (1,) * (kx.MAX_RANK + 1)))
    with pytest.raises(kx.LayoutError):
        kx._descriptor(kx.TensorView(buf, (3, 4), (4,)))


def test_gemm_sharded_checks_every_argument_before_any_work():
    """kx_gemm_sharded_f32 (host side): null and count errors, then per handle
    the window rows of A, B's shape, the outputs' shape, contiguity and
    aliasing -- all before anything is enqueued, so a handle is never touched
    (the stand-in handles here are zeroed host memory)."""
    fake = (C.c_uint8 * 65536)()
    hs = (C.c_void_p * 2)(C.addressof(fake), C.addressof(fake))
    m, k, n = 5, 3, 4

    def call(a, b, out, gather=1, ngpu=2):
        err = _abi.KxError()
        rc = _abi.lib.kx_gemm_sharded_f32(hs, ngpu, (_abi.KxTensor * 2)(*a), (_abi.KxTensor * 2)(*b),
                                          (_abi.KxTensor * 2)(*out), gather, C.byref(err))
        return rc, err

    # windows of 5 rows over 2 handles: 3 and 2 rows
    a = [_tensor([3, k], [k, 1], 0, 3 * k, 0x10000), _tensor([2, k], [k, 1], 0, 2 * k, 0x20000)]
    b = [_tensor([k, n], [n, 1], 0, k * n, 0x30000), _tensor([k, n], [n, 1], 0, k * n, 0x40000)]
    out = [_tensor([m, n], [n, 1], 0, m * n, 0x50000), _tensor([m, n], [n, 1], 0, m * n, 0x60000)]
    rc, err = call(a, b, [_tensor([m * n], [1], 0, m * n, 0x50000)] * 2)
    assert rc == _abi.KX_E_PARAM and err.parameter == b"rank-two outputs"
    rc, err = call([a[1], a[0]], b, out)
    assert rc == _abi.KX_E_PARAM and (err.values[0], err.values[1]) == (0, 3)
    rc, err = call(a, [b[0], _tensor([k, n + 1], [n + 1, 1], 0, k * (n + 1), 0x40000)], out)
    assert rc == _abi.KX_E_PARAM and err.parameter == b"b[r] must be [K, N]" and err.values[0] == 1
    rc, err = call(a, b, [out[0], _tensor([m, n + 1], [n + 1, 1], 0, m * (n + 1), 0x60000)])
    assert rc == _abi.KX_E_LAYOUT and _abi.LAYOUT_ERRORS[err.values[0]] == "OutputShapeMismatch"
    rc, err = call(a, b, [out[0], _tensor([m, n], [1, m], 0, m * n, 0x60000)])
    assert rc == _abi.KX_E_LAYOUT and _abi.LAYOUT_ERRORS[err.values[0]] == "OutputNotCContiguous"
    rc, err = call(a, b, [out[0], _tensor([m, n], [n, 1], 0, m * n, 0x20000)])      # over a[1]
    assert rc == _abi.KX_E_ALIAS
    rc, err = call(a, b, [out[0], out[0]])
    assert rc == _abi.KX_E_ALIAS and err.parameter == b"gathered outputs overlap"
    empty = [_tensor([0, k], [k, 1], 0, 0, 0x10000)] * 2
    zero_out = [_tensor([0, n], [n, 1], 0, 0, 0x50000), _tensor([0, n], [n, 1], 0, 0, 0x60000)]
    assert call(empty, b, zero_out)[0] == _abi.KX_OK               # nothing to compute or copy


def test_gemm_sharded_wrapper_needs_one_of_each_per_handle():
    """kernix_b200.sharded.gemm_sharded: one A window, B replica and output per
    handle, refused on the host before the library is called."""
    from kernix_b200.sharded import gemm_sharded
    with pytest.raises(ValueError):
        gemm_sharded([object(), object()], [None], [None, None], [None, None])
