"""ctypes binding of ``libdcn_b200.so``, the C ABI declared in ``include/dcn_b200.h``.

The library is built in-tree by ``jasnamacos_b200/csrc/build.py``.  There is no
fallback: if the library is missing, :func:`load` raises
:class:`NativeLibraryMissing` and every operator of the package fails loudly.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libdcn_b200.so"

# Status codes of `enum dcn_status`.
DCN_OK = 0
DCN_ERR_INVALID_SHAPE = 1
DCN_ERR_INVALID_COUNT = 2
DCN_ERR_NO_DEVICE = 3
DCN_ERR_UNSUPPORTED = 4
DCN_ERR_NONFINITE = 5
DCN_ERR_LAUNCH = 6
DCN_ERR_INVALID_ARGUMENT = 7
DCN_ERR_DEVICE_TIMEOUT = 8
DCN_ERR_SCRATCH_TOO_SMALL = 9

DCN_DTYPE_F32 = 0
DCN_DTYPE_F16 = 1

DCN_WEIGHT_OIHW = 0
DCN_WEIGHT_IC_K_OC = 1

DCN_PATH_DIRECT = 0
DCN_PATH_FUSED_TC = 1
DCN_PATH_SLAB_TC = 2

DCN_FLAG_NONFINITE = 1

SHAPE_FIELDS = (
    "batch",
    "input_channels",
    "input_height",
    "input_width",
    "output_channels",
    "output_height",
    "output_width",
    "kernel_height",
    "kernel_width",
    "pad_height",
    "pad_width",
    "stride_height",
    "stride_width",
    "dilation_height",
    "dilation_width",
    "groups",
    "offset_groups",
)


class DcnShape(ctypes.Structure):
    """`struct dcn_shape` (mirrors DeformConvShape, DeformConv.swift:3-20)."""

    _fields_ = [(name, ctypes.c_int32) for name in SHAPE_FIELDS]


class DcnCounts(ctypes.Structure):
    """`struct dcn_counts`."""

    _fields_ = [(name, ctypes.c_int64) for name in ("input", "offset", "mask", "weight", "bias", "output")]


class DcnIo(ctypes.Structure):
    """`struct dcn_io`: split input tensors and the output slot (null pointer = defaults)."""

    _fields_ = [
        ("input_second", ctypes.c_void_p),
        ("input_split", ctypes.c_int32),
        ("output_image_channels", ctypes.c_int32),
        ("output_channel_offset", ctypes.c_int32),
    ]


class DcnPlan(ctypes.Structure):
    """`struct dcn_plan`: how dcn_forward_f16 launches a shape on the current device."""

    _fields_ = [
        ("path", ctypes.c_int32),
        ("group_splits", ctypes.c_int32),
        ("tiles_per_unit", ctypes.c_int32),
        ("launches", ctypes.c_int32),
        ("grid", ctypes.c_int64),
        ("prepass_images", ctypes.c_int64),
    ]


_P = ctypes.c_void_p
_SHAPE = ctypes.POINTER(DcnShape)
_IO = ctypes.POINTER(DcnIo)

# Every entry point of include/dcn_b200.h: name -> (restype, argtypes).
PROTOTYPES = {
    "dcn_abi_version": (ctypes.c_int, []),
    "dcn_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "dcn_status_is_recoverable": (ctypes.c_int, [ctypes.c_int]),
    "dcn_shape_validate": (ctypes.c_int, [_SHAPE]),
    "dcn_shape_counts": (ctypes.c_int, [_SHAPE, ctypes.POINTER(DcnCounts)]),
    "dcn_check_counts": (
        ctypes.c_int,
        [_SHAPE] + [ctypes.c_int64] * 5 + [ctypes.POINTER(ctypes.c_int)],
    ),
    "dcn_forward_f32": (ctypes.c_int, [_SHAPE, _P, _P, _P, _P, _P, _P, _P]),
    "dcn_forward_f16_direct": (ctypes.c_int, [_SHAPE, _P, _P, _P, _P, _P, _P, _P]),
    "dcn_packed_weight_bytes": (ctypes.c_size_t, [_SHAPE]),
    "dcn_prepack_weights": (ctypes.c_int, [_SHAPE, _P, ctypes.c_int, ctypes.c_int, _P, _P]),
    "dcn_forward_f16_path": (ctypes.c_int, [_SHAPE]),
    "dcn_forward_f16_plan": (ctypes.c_int, [_SHAPE, ctypes.POINTER(DcnPlan)]),
    "dcn_forward_f16_workspace_bytes": (ctypes.c_size_t, [_SHAPE]),
    "dcn_forward_f16": (
        ctypes.c_int,
        [_SHAPE, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    ),
    "dcn_regroup_input_f16": (ctypes.c_int, [_SHAPE, _P, _P, ctypes.c_size_t, _P]),
    "dcn_forward_f16_grouped": (ctypes.c_int, [_SHAPE, _P, _P, _P, _P, _P, _P, _P, _P]),
    "dcn_regroup_input_nhwc_f16": (ctypes.c_int, [_SHAPE, _P, _P, ctypes.c_size_t, _P]),
    "dcn_forward_f16_raw_workspace_bytes": (ctypes.c_size_t, [_SHAPE]),
    "dcn_forward_f16_raw": (
        ctypes.c_int,
        [_SHAPE, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    ),
    "dcn_forward_f16_raw_grouped": (
        ctypes.c_int,
        [_SHAPE, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    ),
    "dcn_forward_f16_io": (
        ctypes.c_int,
        [_SHAPE, _IO, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    ),
    "dcn_forward_f16_raw_io": (
        ctypes.c_int,
        [_SHAPE, _IO, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    ),
    "dcn_flag_non_finite_f16": (ctypes.c_int, [_P, ctypes.c_int64, _P, _P]),
    "dcn_prepare_offsets_f16": (ctypes.c_int, [ctypes.c_int64, _P, _P, _P, _P, _P, _P]),
    "dcn_temporal_prepare_f16": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P, _P,
                                                ctypes.c_int32, _P, _P, _P, _P]),
    "dcn_temporal_slabs_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "dcn_temporal_prepare_slabs_f16": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P,
                                                      _P, ctypes.c_int32, _P, _P, _P, ctypes.c_size_t, _P]),
    "dcn_device_error": (ctypes.c_int, []),
    "dcn_check_wait_timeout": (ctypes.c_int, [ctypes.c_uint32, _P]),
    "dcn_forward_f16_host_workspace_bytes": (ctypes.c_size_t, [_SHAPE, ctypes.c_int32]),
    "dcn_forward_f16_host": (
        ctypes.c_int,
        [_SHAPE, _P, _P, _P, _P, _P, _P, _P, ctypes.c_int32, _P, ctypes.c_size_t, _P],
    ),
    "dcn_static_scratch_bytes": (ctypes.c_size_t, []),
    "dcn_forward_f16_static_scratch": (ctypes.c_int, [_SHAPE, _P, _P, _P, _P, _P, _P, _P, _P]),
}


class NativeLibraryMissing(ImportError):
    """Raised when libdcn_b200.so has not been built; there is no fallback path."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library once and declares every prototype."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise NativeLibraryMissing(
                f"{LIB_PATH} is missing; build it with `python -m jasnamacos_b200.csrc.build` "
                "(the DCNv2 operator has no CPU fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def status_string(status: int) -> str:
    return load().dcn_status_string(status).decode()
