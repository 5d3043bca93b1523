"""The C ABI without a GPU: the library loads, exports every symbol include/dcn_b200.h
declares, and its host-only entry points (validation, counts, sizes, status text) behave.
No call here launches device work."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from jasnamacos_b200 import _native
from jasnamacos_b200.deform_conv import DeformConvShape

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "dcn_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(dcn_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return _native.load()


def test_header_declarations_are_all_exported(lib):
    names = declared_functions()
    assert len(names) >= 15
    exported = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True,
                              text=True, check=True).stdout
    for name in names:
        assert re.search(rf"\bT {name}$", exported, flags=re.M), f"{name} not exported"
        getattr(lib, name)
    assert set(names) == set(_native.PROTOTYPES), "ctypes prototypes and header disagree"


def test_library_is_self_contained():
    deps = subprocess.run(["ldd", str(_native.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcudart" not in deps  # runtime linked statically


def test_abi_version_and_status_strings(lib):
    assert lib.dcn_abi_version() == 1
    for code in range(10):
        assert lib.dcn_status_string(code)
    assert lib.dcn_status_is_recoverable(_native.DCN_ERR_NONFINITE) == 1
    for code in (0, 1, 2, 3, 4, 6, 7, 8):
        assert lib.dcn_status_is_recoverable(code) == 0


def test_shape_validation_and_counts(lib):
    s = DeformConvShape.jasna_propagation().to_c()
    assert lib.dcn_shape_validate(ctypes.byref(s)) == _native.DCN_OK
    c = _native.DcnCounts()
    assert lib.dcn_shape_counts(ctypes.byref(s), ctypes.byref(c)) == 0
    assert (c.input, c.offset, c.mask, c.weight, c.bias, c.output) == (
        524288, 1179648, 589824, 73728, 64, 262144)
    bad = DeformConvShape(1, 128, 64, 64, 64, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 3).to_c()
    assert lib.dcn_shape_validate(ctypes.byref(bad)) == _native.DCN_ERR_INVALID_SHAPE
    assert lib.dcn_shape_validate(None) == _native.DCN_ERR_INVALID_ARGUMENT


def test_check_counts(lib):
    s = DeformConvShape(1, 1, 2, 2, 1, 2, 2, 1, 1, 0, 0, 1, 1, 1, 1, 1, 1).to_c()
    which = ctypes.c_int(-1)
    assert lib.dcn_check_counts(ctypes.byref(s), 4, 8, 4, 1, 1, ctypes.byref(which)) == 0
    assert lib.dcn_check_counts(ctypes.byref(s), 4, 8, 3, 1, 1, ctypes.byref(which)) == _native.DCN_ERR_INVALID_COUNT
    assert which.value == 2


def test_path_selection_and_sizes(lib):
    jasna = DeformConvShape.jasna_propagation().to_c()
    # 64x64 tiles take the shared-memory slab kernel by default.
    assert lib.dcn_forward_f16_path(ctypes.byref(jasna)) == _native.DCN_PATH_SLAB_TC
    assert lib.dcn_packed_weight_bytes(ctypes.byref(jasna)) == 16 * 5 * 2048  # 16 groups x 5 SW32 blocks
    # zero-bordered slabs: (C/8) groups x (H+2) x (W+2) positions x 16 bytes; one image
    # (32 tiles) splits its 16 groups 4 ways, with FP32 partial sums [4][64][4096] after the slabs
    assert lib.dcn_forward_f16_workspace_bytes(ctypes.byref(jasna)) == 16 * 66 * 66 * 16 + 4 * 64 * 4096 * 4
    two = DeformConvShape.jasna_propagation(2).to_c()    # 64 tiles: split 2 ways
    assert lib.dcn_forward_f16_workspace_bytes(ctypes.byref(two)) == 2 * 16 * 66 * 66 * 16 + 2 * 2 * 64 * 4096 * 4
    five = DeformConvShape.jasna_propagation(5).to_c()   # 160 tiles fill the GPU: no split
    assert lib.dcn_forward_f16_workspace_bytes(ctypes.byref(five)) == 5 * 16 * 66 * 66 * 16
    # a 270x480 frame does not fit a shared-memory slab: global-gather kernel, corner pairs
    frame = DeformConvShape.jasna_propagation(1, 270, 480).to_c()
    assert lib.dcn_forward_f16_path(ctypes.byref(frame)) == _native.DCN_PATH_FUSED_TC
    assert lib.dcn_packed_weight_bytes(ctypes.byref(frame)) == 18 * 8192
    assert lib.dcn_forward_f16_workspace_bytes(ctypes.byref(frame)) == 16 * 270 * 481 * 32
    # 32 output channels -> direct path, OIHW FP16 packed weight, no workspace.
    other = DeformConvShape(1, 128, 64, 64, 32, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 16).to_c()
    assert lib.dcn_forward_f16_path(ctypes.byref(other)) == _native.DCN_PATH_DIRECT
    assert lib.dcn_packed_weight_bytes(ctypes.byref(other)) == 32 * 128 * 9 * 2
    assert lib.dcn_forward_f16_workspace_bytes(ctypes.byref(other)) == 0
    # 5x5 output plane (25 px, not a multiple of 8) -> direct path.
    odd = DeformConvShape.jasna_propagation(1, 5, 5).to_c()
    assert lib.dcn_forward_f16_path(ctypes.byref(odd)) == _native.DCN_PATH_DIRECT


def test_kernel_choice_can_be_pinned_per_process():
    import sys

    code = ("import ctypes; from jasnamacos_b200 import _native; from jasnamacos_b200.deform_conv import "
            "DeformConvShape as S; lib=_native.load(); s=S.jasna_propagation().to_c(); "
            "print(lib.dcn_forward_f16_path(ctypes.byref(s)), lib.dcn_packed_weight_bytes(ctypes.byref(s)))")
    import os

    env = dict(os.environ, DCN_B200_FUSED_KERNEL="pairs", PYTHONPATH=str(REPO))
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, check=True).stdout
    assert out.split() == [str(_native.DCN_PATH_FUSED_TC), str(18 * 8192)]


def test_group_split_can_be_turned_off_per_process():
    import os
    import sys

    code = ("import ctypes; from jasnamacos_b200 import _native; from jasnamacos_b200.deform_conv import "
            "DeformConvShape as S; lib=_native.load(); s=S.jasna_propagation().to_c(); "
            "print(lib.dcn_forward_f16_workspace_bytes(ctypes.byref(s)))")
    env = dict(os.environ, DCN_B200_GROUP_SPLIT="0", PYTHONPATH=str(REPO))
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, check=True).stdout
    assert int(out) == 16 * 66 * 66 * 16  # slabs only: no partial sums


def test_null_pointers_are_rejected_before_any_device_work(lib):
    s = DeformConvShape.jasna_propagation().to_c()
    args = [None] * 6
    assert lib.dcn_forward_f32(ctypes.byref(s), *args, None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_forward_f16_direct(ctypes.byref(s), *args, None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_forward_f16(ctypes.byref(s), *args, None, None, 0, None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_prepack_weights(ctypes.byref(s), None, 0, 0, None, None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_flag_non_finite_f16(None, 4, None, None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_prepare_offsets_f16(0, None, None, None, None, None, None) == _native.DCN_ERR_INVALID_SHAPE


def test_io_plumbing_is_validated_before_device_work(lib):
    """dcn_io rules (split on an 8-channel boundary for the tensor-core paths, the slot inside
    the output tensor) are checked before the device is touched: here, without a GPU, a valid
    dcn_io gets as far as DCN_ERR_NO_DEVICE and an invalid one stops at DCN_ERR_INVALID_ARGUMENT."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("checks the no-device status")
    s = DeformConvShape.jasna_propagation().to_c()
    p = ctypes.c_void_p(256)

    def call(io):
        return lib.dcn_forward_f16_io(ctypes.byref(s), io, p, p, p, p, p, p, None, p, 1 << 30, None)

    def raw_call(io):
        return lib.dcn_forward_f16_raw_io(ctypes.byref(s), io, p, p, p, p, p, p, p, None, p, 1 << 30, None)

    second = ctypes.c_void_p(512)
    for good in (None, _native.DcnIo(second, 64, 0, 0), _native.DcnIo(None, 0, 192, 128),
                 _native.DcnIo(second, 8, 64, 0)):
        arg = None if good is None else ctypes.byref(good)
        assert call(arg) == _native.DCN_ERR_NO_DEVICE
        assert raw_call(arg) == _native.DCN_ERR_NO_DEVICE
    for bad in (_native.DcnIo(second, 60, 0, 0),     # not a deformable-group boundary
                _native.DcnIo(second, 0, 0, 0),      # empty first part
                _native.DcnIo(second, 128, 0, 0),    # empty second part
                _native.DcnIo(None, 64, 0, 0),       # split without a second tensor
                _native.DcnIo(None, 0, 0, 5),        # offset without a channel count
                _native.DcnIo(None, 0, 100, 40),     # slot past the end of the tensor
                _native.DcnIo(None, 0, 192, -1)):
        assert call(ctypes.byref(bad)) == _native.DCN_ERR_INVALID_ARGUMENT
        assert raw_call(ctypes.byref(bad)) == _native.DCN_ERR_INVALID_ARGUMENT


def test_host_entry_sizes_and_argument_checks(lib):
    """dcn_forward_f16_host's staging workspace: up to three chunks in flight, each holding the
    chunk's input, offset, mask, output and the operator's own workspace (the larger of a full
    chunk's and the short last chunk's), plus one flag word; 0 for direct-path shapes.  Bad
    arguments are rejected before the device is touched."""
    one = DeformConvShape.jasna_propagation(1)
    per = 2 * (one.input_count + one.offset_count + one.mask_count + one.output_count)
    for batch, chunk in ((2048, 64), (5, 2), (3, 0), (1, 1)):
        s = DeformConvShape.jasna_propagation(batch)
        c = ctypes.byref(s.to_c())
        eff = min(chunk or 64, batch)
        slots = min(3, -(-batch // eff))
        got = lib.dcn_forward_f16_host_workspace_bytes(c, chunk)
        ws_chunk = lib.dcn_forward_f16_workspace_bytes(ctypes.byref(s.with_batch(eff).to_c()))
        assert got >= 256 + slots * (eff * per + ws_chunk), (batch, chunk)
        assert got < 256 + slots * (eff * per + 2 * ws_chunk + 4 * (1 << 20)), (batch, chunk)
    small = DeformConvShape(1, 4, 5, 5, 3, 5, 5, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)  # direct path
    assert lib.dcn_forward_f16_host_workspace_bytes(ctypes.byref(small.to_c()), 0) == 0
    s = DeformConvShape.jasna_propagation(4).to_c()
    p = ctypes.c_void_p(256)
    need = lib.dcn_forward_f16_host_workspace_bytes(ctypes.byref(s), 2)
    assert lib.dcn_forward_f16_host(ctypes.byref(s), p, p, p, p, p, p, None, 2, p, need - 1, None) == \
        _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_forward_f16_host(ctypes.byref(s), p, p, p, p, p, p, None, -1, p, need, None) == \
        _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_forward_f16_host(ctypes.byref(s), None, p, p, p, p, p, None, 2, p, need, None) == \
        _native.DCN_ERR_INVALID_ARGUMENT
    assert lib.dcn_forward_f16_host(ctypes.byref(small.to_c()), p, p, p, p, p, p, None, 0, p, need, None) == \
        _native.DCN_ERR_UNSUPPORTED


def test_temporal_prepare_argument_checks(lib):
    """dcn_temporal_prepare_f16 rejects bad extents and missing or misaligned tensors before it
    touches a device (deform_input alone may be null)."""
    p = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(257)
    args = lambda **k: [k.get(n, p) for n in ("prop", "cur", "n2", "f1", "prev")]  # noqa: E731
    call = lambda b, w, h, ins, cond=p, di=None, f2=p: lib.dcn_temporal_prepare_f16(  # noqa: E731
        b, w, h, *ins, 1, cond, di, f2, None)
    assert call(0, 64, 64, args()) == _native.DCN_ERR_INVALID_SHAPE
    assert call(1, 0, 64, args()) == _native.DCN_ERR_INVALID_SHAPE
    assert call(1, 64, -1, args()) == _native.DCN_ERR_INVALID_SHAPE
    assert call(1, 1 << 16, 1 << 16, args()) == _native.DCN_ERR_INVALID_SHAPE
    assert call(1, 64, 64, args(n2=None)) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(1, 64, 64, args(f1=odd)) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(1, 64, 64, args(), cond=None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(1, 64, 64, args(), f2=None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(1, 64, 64, args(), di=odd) == _native.DCN_ERR_INVALID_ARGUMENT


def test_temporal_slab_form_argument_checks(lib):
    """dcn_temporal_prepare_slabs_f16 and dcn_forward_f16_raw_grouped reject bad extents, frames
    the slab form does not take, missing or misaligned tensors and a short workspace before they
    touch a device; dcn_temporal_slabs_bytes is the [batch][16][H+2][W+2] x 16-byte slab size."""
    assert lib.dcn_temporal_slabs_bytes(2, 64, 64) == 2 * 16 * 66 * 66 * 16
    assert lib.dcn_temporal_slabs_bytes(1, 480, 270) == 0      # too large for the shared-memory form
    assert lib.dcn_temporal_slabs_bytes(0, 64, 64) == 0
    p = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(264)  # 8-byte aligned only
    full = 2 * 16 * 66 * 66 * 16
    args = lambda **k: [k.get(n, p) for n in ("prop", "cur", "n2", "f1", "prev")]  # noqa: E731
    call = lambda b, w, h, ins, cond=p, f2=p, ws=p, nbytes=full: lib.dcn_temporal_prepare_slabs_f16(  # noqa: E731
        b, w, h, *ins, 1, cond, f2, ws, nbytes, None)
    assert call(0, 64, 64, args()) == _native.DCN_ERR_INVALID_SHAPE
    assert call(2, 64, -1, args()) == _native.DCN_ERR_INVALID_SHAPE
    assert call(1, 480, 270, args()) == _native.DCN_ERR_UNSUPPORTED
    assert call(1, 17, 13, args()) == _native.DCN_ERR_UNSUPPORTED   # odd pixel count
    assert call(2, 64, 64, args(prop=odd)) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(2, 64, 64, args(f1=None)) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(2, 64, 64, args(), cond=odd) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(2, 64, 64, args(), ws=None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(2, 64, 64, args(), ws=odd) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(2, 64, 64, args(), nbytes=full - 1) == _native.DCN_ERR_INVALID_ARGUMENT

    s = DeformConvShape.jasna_propagation(2, 64, 64).to_c()
    need = lib.dcn_forward_f16_raw_workspace_bytes(ctypes.byref(s))
    assert need >= full
    raw_call = lambda ws=p, raw=p, nbytes=need, shape=s: lib.dcn_forward_f16_raw_grouped(  # noqa: E731
        ctypes.byref(shape), ws, raw, p, p, p, p, p, None, nbytes, None)
    bad = DeformConvShape.jasna_propagation(2, 64, 64).to_c()
    bad.batch = 0
    assert raw_call(shape=bad) == _native.DCN_ERR_INVALID_SHAPE
    assert raw_call(raw=None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert raw_call(raw=odd) == _native.DCN_ERR_INVALID_ARGUMENT
    assert raw_call(ws=None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert raw_call(nbytes=need - 1) == _native.DCN_ERR_INVALID_ARGUMENT


def test_nhwc_regroup_argument_checks(lib):
    """dcn_regroup_input_nhwc_f16 rejects direct-path shapes, missing or misaligned pointers and a
    short workspace before it touches a device."""
    s = DeformConvShape.jasna_propagation(2, 64, 64).to_c()
    need = lib.dcn_forward_f16_workspace_bytes(ctypes.byref(s))
    p = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(264)  # 8-byte aligned only
    call = lambda x=p, ws=p, nbytes=need, shape=s: lib.dcn_regroup_input_nhwc_f16(  # noqa: E731
        ctypes.byref(shape), x, ws, nbytes, None)
    direct = DeformConvShape(1, 128, 64, 64, 32, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 16).to_c()
    assert call(shape=direct) == _native.DCN_ERR_UNSUPPORTED
    assert call(x=None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(x=odd) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(ws=odd) == _native.DCN_ERR_INVALID_ARGUMENT
    assert call(nbytes=need - 1) == _native.DCN_ERR_INVALID_ARGUMENT
