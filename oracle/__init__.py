"""CPU oracle for DCNv2 parity -- TEST INFRASTRUCTURE ONLY.

A C restatement of the reference's ``DeformConvCPU.run``
(Sources/JasnaMetalPoC/DeformConv.swift:75-166), compiled by ``oracle/Makefile`` into
``oracle/_build/libdcn_oracle.so``.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline arm of ``bench.py`` may use it, and only as the checker or the timed CPU
reference; the product library never calls it.

Parity pin: the reference's own known-answer test (Tests/JasnaMetalPoCTests/
DeformConvCPUTests.swift:4-33) is reproduced bit-exactly in tests/test_oracle.py.  The
Swift reference cannot be compiled here (no Swift toolchain), so there is no ``_ref``
build of the reference itself.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "_build" / "libdcn_oracle.so"

_FIELDS = (
    "batch", "input_channels", "input_height", "input_width", "output_channels", "output_height",
    "output_width", "kernel_height", "kernel_width", "pad_height", "pad_width", "stride_height",
    "stride_width", "dilation_height", "dilation_width", "groups", "offset_groups",
)


class OracleShape(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int32) for f in _FIELDS]


_lock = threading.Lock()
_lib = None


def build() -> Path:
    """Compiles the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIB_PATH


def load():
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (ORACLE_DIR / "dcn_oracle.c").stat().st_mtime:
                build()
            lib = ctypes.CDLL(str(LIB_PATH))
            fp = ctypes.POINTER(ctypes.c_float)
            sp = ctypes.POINTER(OracleShape)
            lib.dcn_oracle_validate.argtypes = [sp]
            lib.dcn_oracle_validate.restype = ctypes.c_int
            lib.dcn_oracle_run_threads.argtypes = [sp, fp, fp, fp, fp, fp, fp, ctypes.c_int32, ctypes.c_int32,
                                                   ctypes.c_int, ctypes.c_int]
            lib.dcn_oracle_run_threads.restype = ctypes.c_int
            lib.dcn_oracle_run_sample.argtypes = [sp, fp, fp, fp, fp, fp, fp, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_int]
            lib.dcn_oracle_run_sample.restype = ctypes.c_int
            lib.dcn_oracle_prepare_offsets.argtypes = [ctypes.c_int64, fp, fp, fp, fp, fp]
            lib.dcn_oracle_prepare_offsets.restype = None
            lib.dcn_oracle_temporal_prepare.argtypes = [ctypes.c_int32, ctypes.c_int32, fp, fp, fp, fp, fp,
                                                        ctypes.c_int, fp, fp, fp]
            lib.dcn_oracle_temporal_prepare.restype = None
            lib.dcn_oracle_splitmix64.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
            lib.dcn_oracle_splitmix64.restype = ctypes.c_uint64
            _lib = lib
        return _lib


def _shape(shape) -> OracleShape:
    values = shape.as_tuple() if hasattr(shape, "as_tuple") else tuple(shape)
    return OracleShape(*values)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def validate(shape) -> bool:
    return load().dcn_oracle_validate(ctypes.byref(_shape(shape))) == 0


def run(shape, input, offset, mask, weight, bias, threads: int = 1, batch_range=None,
        fast: bool = True) -> np.ndarray:
    """DeformConvCPU.run on float32 arrays.  With `batch_range=(b, e)` only images b..e-1
    are computed; the returned array then holds just those images' outputs.  `fast=False`
    runs the literal reference loop; `fast=True` the bit-identical memoised form."""
    lib = load()
    s = _shape(shape)
    arrays = [np.ascontiguousarray(a, dtype=np.float32).reshape(-1) for a in (input, offset, mask, weight, bias)]
    n = s.batch
    b, e = (0, n) if batch_range is None else batch_range
    per_image = s.output_channels * s.output_height * s.output_width
    out = np.zeros(n * per_image, dtype=np.float32)
    rc = lib.dcn_oracle_run_threads(ctypes.byref(s), *[_fptr(a) for a in arrays], _fptr(out), b, e,
                                    max(1, int(threads)), 1 if fast else 0)
    if rc != 0:
        raise ValueError(f"oracle rejected the shape (rc={rc})")
    return out if batch_range is None else out[b * per_image:e * per_image].copy()


def run_sample(shape, input, offset, mask, weight, bias, rows: tuple[int, int], threads: int) -> np.ndarray:
    """The literal reference loop over output rows [rows[0], rows[1]) of every image, one
    batch slice per thread (the CPU-baseline timing sample).  Returns the full output array
    (untouched outside the rows)."""
    lib = load()
    s = _shape(shape)
    arrays = [np.ascontiguousarray(a, dtype=np.float32).reshape(-1) for a in (input, offset, mask, weight, bias)]
    out = np.zeros(s.batch * s.output_channels * s.output_height * s.output_width, dtype=np.float32)
    rc = lib.dcn_oracle_run_sample(ctypes.byref(s), *[_fptr(a) for a in arrays], _fptr(out), rows[0], rows[1],
                                   max(1, int(threads)))
    if rc != 0:
        raise ValueError(f"oracle rejected the shape (rc={rc})")
    return out


def prepare_offsets(plane: int, raw, flow1, flow2):
    lib = load()
    raw, flow1, flow2 = [np.ascontiguousarray(a, dtype=np.float32).reshape(-1) for a in (raw, flow1, flow2)]
    offset = np.zeros(288 * plane, dtype=np.float32)
    mask = np.zeros(144 * plane, dtype=np.float32)
    lib.dcn_oracle_prepare_offsets(plane, _fptr(raw), _fptr(flow1), _fptr(flow2), _fptr(offset), _fptr(mask))
    return offset, mask


def temporal_prepare(width: int, height: int, feat_prop, feat_current, feat_n2, flow1, previous_flow,
                     has_second_order: bool, deform_input: bool = True):
    """runTemporalPreparation (MetalRunner.swift:510-582) for one frame on FP16-valued float
    arrays: returns (conditions [196*plane], deform_input [128*plane] or None, flow2 [2*plane]),
    float32 arrays holding FP16 values."""
    lib = load()
    plane = width * height
    arrays = [np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
              for a in (feat_prop, feat_current, feat_n2, flow1, previous_flow)]
    cond = np.zeros(196 * plane, dtype=np.float32)
    di = np.zeros(128 * plane, dtype=np.float32) if deform_input else None
    flow2 = np.zeros(2 * plane, dtype=np.float32)
    lib.dcn_oracle_temporal_prepare(width, height, *[_fptr(a) for a in arrays], 1 if has_second_order else 0,
                                    _fptr(cond), _fptr(di) if di is not None else None, _fptr(flow2))
    return cond, di, flow2


def splitmix64_sequence(seed: int, count: int) -> list[int]:
    lib = load()
    state = ctypes.c_uint64(0x9E3779B97F4A7C15 if seed == 0 else seed)
    return [lib.dcn_oracle_splitmix64(ctypes.byref(state)) for _ in range(count)]


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
