"""GPU checks of the operator's error contract and helper kernels, through the C ABI:
non-finite detection (MetalNonFiniteFlagTests.swift, MetalShader.swift:454-463), the offset
transform (MetalShader.swift:817-839 vs JasnaCLI.swift:177-211), host-side argument
errors, the device error word and the reference-style benchmark."""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

import oracle
from golden_data import reference_kats
from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape, InvalidArgument, NonFiniteOutput

pytestmark = pytest.mark.gpu


def test_non_finite_flag_reference_cases(cuda_op):
    import torch

    for values, expected in reference_kats()["non_finite_flag"]["cases"]:
        vals = torch.tensor([float(v) for v in values], dtype=torch.float16, device="cuda")
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        cuda_op.flag_non_finite(vals, flag)
        torch.cuda.synchronize()
        assert int(flag.item()) == expected, values


def test_fused_epilogue_flags_non_finite_output(cuda_op):
    inp = synthetic.generate(1)
    x = inp.input.copy()
    x[1234] = np.inf  # a sample that lands on it turns the output non-finite
    with pytest.raises(NonFiniteOutput) as e:
        cuda_op.run_float16(inp.shape, x, inp.offset, inp.mask, inp.weight, inp.bias)
    assert e.value.is_recoverable_numerical_failure
    # a finite run of the same operator does not raise
    cuda_op.run_float16(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)


def test_direct_path_flags_non_finite_output(cuda_op):
    s = DeformConvShape.jasna_propagation(1, 5, 5)  # direct path
    g = synthetic.SplitMix64(5)
    arrays = [g.uniform(n, -1, 1) for n in (s.input_count, s.offset_count, s.mask_count, s.weight_count,
                                              s.output_channels)]
    arrays[3][0] = 70000.0  # overflows FP16 -> Inf weight
    with pytest.raises(NonFiniteOutput), np.errstate(over="ignore"):  # the overflow is the point
        cuda_op.run_float16(s, *arrays)


def test_offset_transform_reference_cli_case(cuda_op):
    import torch

    kat = reference_kats()["offset_transform"]
    plane = kat["plane"]
    raw, f1, f2 = (np.array(kat[k], np.float32) for k in ("raw", "flow1", "flow2"))
    off, msk = cuda_op.prepare_offsets(plane, *(torch.from_numpy(a).half().cuda() for a in (raw, f1, f2)))
    torch.cuda.synchronize()
    ref_off, ref_msk = oracle.prepare_offsets(plane, raw, f1, f2)
    err = max(np.abs(off.float().cpu().numpy() - ref_off).max(), np.abs(msk.float().cpu().numpy() - ref_msk).max())
    assert err < kat["tolerance"]  # JasnaCLI.swift:208


def test_run_dcn_offset_transform_host_arrays(cuda_op):
    """runDCNOffsetTransform's host-array form (MetalRunner.swift:469-508): the reference CLI's
    plane-7 case under its 0.005 gate (JasnaCLI.swift:177-211), the same bits as the device-tensor
    entry, and a 4096-pixel plane with raw values that saturate tanh and the sigmoid; sizes that do
    not match the plane raise InvalidShape."""
    import torch

    from jasnamacos_b200.deform_conv import InvalidShape

    kat = reference_kats()["offset_transform"]
    plane = kat["plane"]
    raw, f1, f2 = (np.array(kat[k], np.float32) for k in ("raw", "flow1", "flow2"))
    off, msk = cuda_op.run_dcn_offset_transform(plane, raw, f1, f2)
    assert off.dtype == np.float16 and off.shape == (288 * plane,) and msk.shape == (144 * plane,)
    ref_off, ref_msk = oracle.prepare_offsets(plane, raw, f1, f2)
    err = max(np.abs(off.astype(np.float32) - ref_off).max(), np.abs(msk.astype(np.float32) - ref_msk).max())
    assert err < kat["tolerance"]
    d_off, d_msk = cuda_op.prepare_offsets(plane, *(torch.from_numpy(a).half().cuda() for a in (raw, f1, f2)))
    torch.cuda.synchronize()
    assert np.array_equal(off, d_off.cpu().numpy()) and np.array_equal(msk, d_msk.cpu().numpy())

    plane = 64 * 64
    g = np.random.default_rng(21)
    f16 = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    raw, f1, f2 = f16(g.uniform(-12, 12, 432 * plane)), f16(g.uniform(-16, 16, 2 * plane)), f16(
        g.uniform(-16, 16, 2 * plane))
    off, msk = cuda_op.run_dcn_offset_transform(plane, raw, f1, f2)
    ref_off, ref_msk = oracle.prepare_offsets(plane, raw, f1, f2)
    # one FP16 rounding of offsets below 26 in magnitude (ulp 2^-6 there) and of masks in [0, 1]
    assert np.abs(off.astype(np.float32) - ref_off).max() <= 2.0 ** -6
    assert np.abs(msk.astype(np.float32) - ref_msk).max() <= 2.0 ** -11
    assert np.isfinite(off.astype(np.float32)).all() and msk.min() >= 0 and msk.max() <= 1
    with pytest.raises(InvalidShape):
        cuda_op.run_dcn_offset_transform(plane, raw[:-1], f1, f2)
    with pytest.raises(InvalidShape):
        cuda_op.run_dcn_offset_transform(0, raw[:0], f1[:0], f2[:0])


def test_misaligned_pointers_are_rejected_on_the_host(cuda_op):
    import torch

    s = DeformConvShape.jasna_propagation()
    x = torch.zeros(s.input_count, dtype=torch.float16, device="cuda")
    off_big = torch.zeros(s.offset_count + 1, dtype=torch.float16, device="cuda")
    msk = torch.zeros(s.mask_count, dtype=torch.float16, device="cuda")
    w = torch.zeros(s.weight_count, dtype=torch.float16, device="cuda")
    b = torch.zeros(64, dtype=torch.float16, device="cuda")
    packed = cuda_op.prepack(s, w)
    with pytest.raises(InvalidArgument):
        cuda_op.forward_f16(s, x, off_big[1:], msk, packed, b)  # offset rows must be 16-byte aligned
    ws = torch.zeros(cuda_op.workspace_bytes(s) // 2, dtype=torch.uint8, device="cuda")
    with pytest.raises(InvalidArgument):
        cuda_op.forward_f16(s, x, off_big[:-1], msk, packed, b, workspace=ws)  # short workspace


def test_device_error_word_is_clear(cuda_op):
    assert cuda_op.lib.dcn_device_error() == _native.DCN_OK


def test_benchmark_jasna_shape(cuda_op):
    r = cuda_op.benchmark_jasna_shape(iterations=5)
    assert r["max_difference_from_direct"] <= 0.002
    assert math.isfinite(r["checksum"]) and not r["nonfinite"]
    assert r["fused"].median > 0 and r["direct"].median > 0


def test_stream_ordering_on_a_side_stream(cuda_op):
    """Work is enqueued on the caller's stream: a side stream gives the same result."""
    import torch

    inp = synthetic.generate(1)
    s = inp.shape
    x, off, msk, w, b = [torch.from_numpy(a).cuda() for a in inp.tensors_f16()]
    packed = cuda_op.prepack(s, w)
    base = cuda_op.forward_f16(s, x, off, msk, packed, b)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        out = cuda_op.forward_f16(s, x, off, msk, packed, b, stream=side)
    side.synchronize()
    assert torch.equal(base, out)
    assert ctypes.sizeof(ctypes.c_void_p) == 8


@pytest.mark.parametrize("shape,path,splits,launches", [
    (DeformConvShape.jasna_propagation(1, 64, 64), _native.DCN_PATH_SLAB_TC, 4, 3),
    (DeformConvShape.jasna_propagation(2048, 64, 64), _native.DCN_PATH_SLAB_TC, 1, 2),
    (DeformConvShape.jasna_propagation(1, 270, 480), _native.DCN_PATH_FUSED_TC, 1, 2),
    (DeformConvShape.jasna_propagation(2, 5, 7), _native.DCN_PATH_DIRECT, 1, 1),
], ids=["one_tile_image", "config4", "config3", "direct"])
def test_launch_plan(cuda_op, shape, path, splits, launches):
    """dcn_forward_f16_plan agrees with the path query and the workspace layout: a group
    split (a reduction pass and FP32 partials past the slabs) only for batches with fewer
    128-pixel tiles than SMs, persistent grids of at most one CTA per SM."""
    import torch

    plan = cuda_op.plan(shape)
    assert plan["path"] == cuda_op.path(shape) == path
    assert plan["group_splits"] == splits and plan["launches"] == launches
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if path != _native.DCN_PATH_DIRECT:
        assert 1 <= plan["grid"] <= sms and plan["prepass_images"] == shape.batch
    if path == _native.DCN_PATH_SLAB_TC:
        slabs = shape.batch * shape.offset_groups * (shape.input_height + 2) * (shape.input_width + 2) * 16
        assert (cuda_op.workspace_bytes(shape) > (slabs + 255) // 256 * 256) == (splits > 1)


def test_bounded_wait_timeout_is_reported_and_context_survives(cuda_op):
    """The failure path of every bounded device wait, without a fault: a wait that nothing
    completes runs out after its limit, the kernel records the timeout in the device error
    word and returns, the host reads DCN_ERR_DEVICE_TIMEOUT once (the read clears it), and
    the same context then runs the operator correctly."""
    import time

    import torch

    from jasnamacos_b200.deform_conv import DeviceTimeout

    assert cuda_op.lib.dcn_check_wait_timeout(0, None) == _native.DCN_ERR_INVALID_ARGUMENT
    assert cuda_op.lib.dcn_device_error() == _native.DCN_OK
    t0 = time.perf_counter()
    assert cuda_op.lib.dcn_check_wait_timeout(100_000, None) == _native.DCN_OK  # 100 ms limit
    with pytest.raises(DeviceTimeout):
        cuda_op.device_error()  # synchronises: the wait has run out by now
    elapsed = time.perf_counter() - t0
    assert 0.09 <= elapsed < 5.0, elapsed
    assert cuda_op.lib.dcn_device_error() == _native.DCN_OK, "the error word is cleared by the read"

    inp = synthetic.generate(1)
    s = inp.shape
    x, off, msk, w, b = [torch.from_numpy(a).cuda() for a in inp.tensors_f16()]
    out = cuda_op.forward_f16(s, x, off, msk, cuda_op.prepack(s, w), b)
    torch.cuda.synchronize()
    cuda_op.device_error()
    q = inp.quantized()
    ref = oracle.run(s, q.input, q.offset, q.mask, q.weight, q.bias)
    d = np.abs(out.float().cpu().numpy() - ref)
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (float(d.max()), float(d.mean()))
