"""ctypes binding of include/kernix_b200.h and the OpsError mirror.

Loading fails loudly when the shared library is missing: there is no CPU
fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkernix_b200.so"
MAX_RANK = 8

# kx_status
KX_OK = 0
KX_IPC_HANDLE_BYTES = 64
KX_DECLINED = 1
KX_E_INVALID_RANK = 2
KX_E_CONTRACT = 3
KX_E_BROADCAST = 4
KX_E_SHAPE_OVERFLOW = 5
KX_E_DIM_OVERFLOW = 6
KX_E_LAYOUT = 7
KX_E_PARAM = 8
KX_E_EXACT_RANK = 9
KX_E_NONFINITE = 10
KX_E_AXIS = 11
KX_E_ALIAS = 12
KX_E_CUDA = 13
KX_E_NO_DEVICE = 14
KX_E_TIMEOUT = 15
KX_E_UNSUPPORTED = 16
KX_E_AXES_MISMATCH = 17
KX_E_DUPLICATE_AXIS = 18

# kx_layout_error sub-codes
LAYOUT_ERRORS = {
    1: "StrideRankMismatch",
    2: "AddressOverflow",
    3: "NegativeStorageOffset",
    4: "StorageTooSmall",
    5: "StorageByteExtentOverflow",
    6: "OutputNotCContiguous",
    7: "OutputShapeMismatch",
    8: "MisalignedPointer",
}

KX_F32_AUTO, KX_F32_FFMA, KX_F32_3XTF32 = 0, 1, 2


class KxError(C.Structure):
    _fields_ = [
        ("status", C.c_int32),
        ("cuda_error", C.c_int32),
        ("operation", C.c_char * 40),
        ("parameter", C.c_char * 96),
        ("values", C.c_uint64 * 4),
        ("nindices", C.c_uint32),
        ("indices", C.c_uint64 * MAX_RANK),
    ]


class KxTensor(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("storage_len", C.c_uint64),
        ("origin", C.c_uint64),
        ("rank", C.c_uint32),
        ("reserved", C.c_uint32),
        ("dims", C.c_uint64 * MAX_RANK),
        ("strides", C.c_int64 * MAX_RANK),
    ]


class KxMatrix(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("storage_len", C.c_uint64),
        ("dims", C.c_uint64 * 2),
        ("strides", C.c_int64 * 2),
        ("origin", C.c_uint64),
    ]


class KxCudaConfig(C.Structure):
    """kx_cuda_config: the [cuda] table of a configuration."""
    _fields_ = [
        ("device", C.c_int32),
        ("f32_variant", C.c_int32),
        ("f64_variant", C.c_int32),
        ("ordered_matmul", C.c_int32),
        ("workspace_bytes", C.c_uint64),
    ]


class KxConv2dOptions(C.Structure):
    _fields_ = [
        ("stride", C.c_uint64 * 2),
        ("padding", C.c_uint64 * 2),
        ("dilation", C.c_uint64 * 2),
        ("groups", C.c_uint64),
    ]


_P = C.POINTER
_vp = C.c_void_p
_u64 = C.c_uint64
_SIGNATURES = {
    "kx_abi_version": (C.c_int, []),
    "kx_device_count": (C.c_int, [_P(C.c_int)]),
    "kx_create": (C.c_int, [C.c_int, _P(_vp), _P(KxError)]),
    "kx_destroy": (C.c_int, [_vp]),
    "kx_set_stream": (C.c_int, [_vp, _vp]),
    "kx_set_f32_variant": (C.c_int, [_vp, C.c_int]),
    "kx_set_ordered_matmul": (C.c_int, [_vp, C.c_int]),
    "kx_ordered_matmul": (C.c_int, [_vp]),
    "kx_synchronize": (C.c_int, [_vp, _P(KxError)]),
    "kx_diag_expire_next_gemm": (C.c_int, [_vp, C.c_uint64]),
    "kx_cuda_config_default": (None, [_P(KxCudaConfig)]),
    "kx_context_create": (C.c_int, [_P(KxCudaConfig), _P(_vp), _P(KxError)]),
    "kx_handle_config": (C.c_int, [_vp, _P(KxCudaConfig)]),
    "kx_alloc": (C.c_int, [_vp, _u64, _P(_vp), _P(KxError)]),
    "kx_free": (C.c_int, [_vp, _vp]),
    "kx_upload": (C.c_int, [_vp, _vp, _vp, _u64, _P(KxError)]),
    "kx_download": (C.c_int, [_vp, _vp, _vp, _u64, _P(KxError)]),
    "kx_matmul_shape": (C.c_int, [_P(_u64), C.c_uint32, _P(_u64), C.c_uint32, _P(C.c_uint32), _P(_u64),
                                  _P(KxError)]),
    "kx_conv2d_shape": (C.c_int, [_P(_u64), C.c_uint32, _P(_u64), C.c_uint32, _P(KxConv2dOptions), _P(_u64),
                                  _P(KxError)]),
    "kx_validate_tensor": (C.c_int, [_P(KxTensor), C.c_uint32, _P(KxError)]),
    "kx_matmul_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _P(KxError)]),
    "kx_matmul_f64": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _P(KxError)]),
    "kx_conv2d_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxConv2dOptions), _P(KxTensor), _P(KxError)]),
    "kx_conv2d_f64": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxConv2dOptions), _P(KxTensor), _P(KxError)]),
    "kx_softmax_temperature_f32": (C.c_int, [_vp, _P(KxTensor), C.c_int64, C.c_float, _P(KxTensor), _P(KxError)]),
    "kx_softmax_temperature_f64": (C.c_int, [_vp, _P(KxTensor), C.c_int64, C.c_double, _P(KxTensor), _P(KxError)]),
    "kx_attention_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), C.c_float, _P(KxTensor),
                                   _P(KxError)]),
    "kx_softmax_f32": (C.c_int, [_vp, _P(KxTensor), C.c_int64, _P(KxTensor), _P(KxError)]),
    "kx_softmax_f64": (C.c_int, [_vp, _P(KxTensor), C.c_int64, _P(KxTensor), _P(KxError)]),
    "kx_tensordot_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(C.c_int64), C.c_uint32, _P(C.c_int64),
                                   C.c_uint32, _P(KxTensor), _P(KxError)]),
    "kx_tensordot_f64": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(C.c_int64), C.c_uint32, _P(C.c_int64),
                                   C.c_uint32, _P(KxTensor), _P(KxError)]),
    "kx_matmul_backward_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _P(KxTensor),
                                         _P(KxTensor), _P(KxError)]),
    "kx_matmul_backward_f64": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _P(KxTensor),
                                         _P(KxTensor), _P(KxError)]),
    "kx_conv2d_backward_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _P(KxConv2dOptions),
                                         _P(KxTensor), _P(KxTensor), _P(KxError)]),
    "kx_conv2d_backward_f64": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _P(KxConv2dOptions),
                                         _P(KxTensor), _P(KxTensor), _P(KxError)]),
    "kx_try_dense_matmul_f32": (C.c_int, [_vp, _vp, _u64, _vp, _u64, _vp, _u64, _u64, _u64, _u64]),
    "kx_try_dense_matmul_f64": (C.c_int, [_vp, _vp, _u64, _vp, _u64, _vp, _u64, _u64, _u64, _u64]),
    "kx_try_strided_matmul_f32": (C.c_int, [_vp, _P(KxMatrix), _P(KxMatrix), _vp, _u64]),
    "kx_try_strided_matmul_f64": (C.c_int, [_vp, _P(KxMatrix), _P(KxMatrix), _vp, _u64]),
    "kx_matrix_validate": (C.c_int, [_P(KxMatrix), C.c_uint32, _P(KxError)]),
    "kx_matmul_splitk_f32_static": (C.c_int, [_P(KxTensor), _P(KxTensor), _P(KxTensor), _vp, _P(KxError)]),
    "kx_matmul_replicated_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _vp, _P(KxError)]),
    "kx_matmul_replicated_f64": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), _vp, _P(KxError)]),
    "kx_multicast_store": (C.c_int, [_vp, _vp, _vp, C.c_uint64, _P(KxError)]),
    "kx_ipc_export": (C.c_int, [_vp, _vp, C.c_char_p, _P(KxError)]),
    "kx_ipc_import": (C.c_int, [_vp, C.c_char_p, _P(_vp), _P(KxError)]),
    "kx_set_f64_variant": (C.c_int, [_vp, C.c_int]),
    "kx_ipc_close": (C.c_int, [_vp, _vp]),
    "kx_peer_broadcast": (C.c_int, [_vp, _vp, _P(_vp), C.c_int, C.c_uint64, _P(KxError)]),
    "kx_copy_async": (C.c_int, [_vp, _vp, _vp, C.c_uint64, _vp, _P(KxError)]),
    "kx_shard_window": (C.c_int, [_u64, C.c_uint32, C.c_uint32, _P(_u64), _P(_u64)]),
    "kx_row_piece": (C.c_int, [_u64, C.c_uint32, _u64, _P(_u64), _P(_u64)]),
    "kx_matmul_rows_sharded_f32": (C.c_int, [_vp, _P(KxTensor), _P(KxTensor), _P(KxTensor), C.c_uint32, C.c_uint32,
                                             _u64, _P(_vp), _vp, _P(KxError)]),
    "kx_gemm_sharded_f32": (C.c_int, [_P(_vp), C.c_uint32, _P(KxTensor), _P(KxTensor), _P(KxTensor), C.c_int,
                                      _P(KxError)]),
    "kx_launch_count": (C.c_uint64, [_vp]),
    "kx_last_kernel": (C.c_char_p, [_vp]),
    "kx_status_name": (C.c_char_p, [C.c_int]),
}


def load_library(path: Path = LIB_PATH) -> C.CDLL:
    if not path.exists():
        raise ImportError(
            f"kernix_b200: native library {path} is missing; run "
            "`python kernix_b200/_build.py` (needs nvcc). There is no CPU fallback.")
    lib = C.CDLL(str(path))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = load_library()
EXPORTED = tuple(_SIGNATURES)


# ---------------------------------------------------------------------------
# OpsError mirror (kernix-ops ops/error.rs:8-140, kernix-core layout/error.rs)
# ---------------------------------------------------------------------------
class OpsError(Exception):
    """Base of every error the C ABI reports; `status` is the kx_status code."""

    status = -1

    def __init__(self, message: str = "", **fields):
        super().__init__(message or self.__class__.__name__)
        self.fields = fields
        for k, v in fields.items():
            setattr(self, k, v)

    def __eq__(self, other):
        return type(self) is type(other) and self.fields == other.fields

    def __hash__(self):
        return hash((type(self), tuple(sorted(self.fields.items()))))

    def __repr__(self):
        inner = ", ".join(f"{k}={v!r}" for k, v in self.fields.items())
        return f"{self.__class__.__name__}({inner})"


class InvalidRank(OpsError):
    status = KX_E_INVALID_RANK


class ContractDimensionMismatch(OpsError):
    status = KX_E_CONTRACT


class BroadcastIncompatible(OpsError):
    status = KX_E_BROADCAST


class ElementCountOverflow(OpsError):
    """ShapeError::ElementCountOverflow (wrapped as OpsError::Shape)."""
    status = KX_E_SHAPE_OVERFLOW


class DimensionOverflow(OpsError):
    status = KX_E_DIM_OVERFLOW


class LayoutError(OpsError):
    status = KX_E_LAYOUT


class InvalidParameter(OpsError):
    status = KX_E_PARAM


class ExactRank(OpsError):
    status = KX_E_EXACT_RANK


class NonFiniteInput(OpsError):
    status = KX_E_NONFINITE


class AxisOutOfBounds(OpsError):
    status = KX_E_AXIS


class OverlappingOutput(OpsError):
    status = KX_E_ALIAS


class CudaError(OpsError):
    status = KX_E_CUDA


class NoDevice(OpsError):
    status = KX_E_NO_DEVICE


class DeviceTimeout(OpsError):
    status = KX_E_TIMEOUT


class Unsupported(OpsError):
    status = KX_E_UNSUPPORTED


class ContractAxesMismatch(OpsError):
    """OpsError::ContractAxesMismatch {left, right}: axis-count mismatch."""
    status = KX_E_AXES_MISMATCH


class DuplicateAxis(OpsError):
    """OpsError::DuplicateAxis {axis}."""
    status = KX_E_DUPLICATE_AXIS


class CapacityOverflow(OpsError):
    """StorageError::CapacityOverflow {len, element_size} (kernix-core
    storage/error.rs:23-30): an output allocation whose byte size exceeds
    isize::MAX.  Raised by the allocating wrappers before any device work."""
    status = -2


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def raise_for(rc: int, err: KxError | None) -> None:
    """Raise the OpsError subclass that mirrors a nonzero kx_status."""
    if rc == KX_OK:
        return
    op = err.operation.decode() if err is not None else ""
    param = err.parameter.decode() if err is not None else ""
    v = list(err.values) if err is not None else [0, 0, 0, 0]
    msg = f"{op}: {param}" if op else lib.kx_status_name(rc).decode()
    if rc == KX_E_INVALID_RANK:
        raise InvalidRank(msg, operation=op, minimum=v[0], actual=v[1])
    if rc == KX_E_CONTRACT:
        raise ContractDimensionMismatch(msg, left=v[0], right=v[1])
    if rc == KX_E_BROADCAST:
        raise BroadcastIncompatible(msg, axis=v[0], left=v[1], right=v[2])
    if rc == KX_E_SHAPE_OVERFLOW:
        raise ElementCountOverflow(msg, axis=v[0], accumulated=v[1], dim=v[2])
    if rc == KX_E_DIM_OVERFLOW:
        raise DimensionOverflow(msg, axis=v[0])
    if rc == KX_E_LAYOUT:
        kind = LAYOUT_ERRORS.get(v[0], "Unknown")
        if kind == "StorageTooSmall":
            raise LayoutError(msg, kind=kind, required=v[1], available=v[2])
        raise LayoutError(msg, kind=kind)
    if rc == KX_E_PARAM:
        raise InvalidParameter(msg, operation=op, parameter=param)
    if rc == KX_E_EXACT_RANK:
        raise ExactRank(msg, operation=op, expected=v[0], actual=v[1])
    if rc == KX_E_NONFINITE:
        idx = [int(err.indices[i]) for i in range(err.nindices)] if err is not None else []
        raise NonFiniteInput(msg, operation=op, indices=idx)
    if rc == KX_E_AXIS:
        raise AxisOutOfBounds(msg, axis=_signed(v[0]), rank=v[1])
    if rc == KX_E_ALIAS:
        raise OverlappingOutput(msg)
    if rc == KX_E_CUDA:
        raise CudaError(msg, cuda_error=err.cuda_error if err is not None else 0)
    if rc == KX_E_NO_DEVICE:
        raise NoDevice(msg)
    if rc == KX_E_TIMEOUT:
        raise DeviceTimeout(msg)
    if rc == KX_E_UNSUPPORTED:
        raise Unsupported(msg)
    if rc == KX_E_AXES_MISMATCH:
        raise ContractAxesMismatch(msg, left=v[0], right=v[1])
    if rc == KX_E_DUPLICATE_AXIS:
        raise DuplicateAxis(msg, axis=v[0])
    raise OpsError(msg, status=rc)


def u64_array(values) -> C.Array:
    vals = [int(x) for x in values]
    return (C.c_uint64 * max(len(vals), MAX_RANK))(*vals)
