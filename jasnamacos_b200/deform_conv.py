"""Host-side mirror of the reference's deformable-convolution operator.

Mirrors, name for name where Python allows:
  * ``DeformConvShape`` -- ``struct DeformConvShape`` (Sources/JasnaMetalPoC/DeformConv.swift:3-42)
  * ``DeformConvError`` -- ``enum DeformConvError`` (DeformConv.swift:44-73)
  * ``CudaDeformConv``  -- ``final class MetalDeformConv`` (MetalRunner.swift:92-388), the
    operator the Swift host calls: ``run_float32`` (``runFloat32``, :159-185) plus the FP16
    entry points its production graph binds (gather + GEMM, FusedFourPassRecurrenceProbe.swift:609-630)
    and ``benchmark_jasna_shape`` (``benchmarkJasnaShape``, :187-388).

Every computation runs in ``libdcn_b200.so`` through its C ABI; PyTorch only provides
device memory, streams and events.  There is no CPU fallback: without the library or a
CUDA device the operator raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, fields

import numpy as np

from . import _native
from .benchmark_statistics import BenchmarkStatistics


# ----------------------------------------------------------------------------- errors


class DeformConvError(Exception):
    """Base of the operator's errors (DeformConv.swift:44-73)."""

    status = _native.DCN_ERR_LAUNCH

    @property
    def is_recoverable_numerical_failure(self) -> bool:
        """Only non-finite output is recoverable (DeformConv.swift:52-55)."""
        return False


class InvalidShape(DeformConvError):
    status = _native.DCN_ERR_INVALID_SHAPE

    def __init__(self, message: str = "Invalid deformable-convolution shape"):
        super().__init__(message)


class InvalidArrayCount(DeformConvError):
    status = _native.DCN_ERR_INVALID_COUNT

    def __init__(self, name: str, expected: int, actual: int):
        self.name, self.expected, self.actual = name, expected, actual
        super().__init__(f"{name} has {actual} elements; expected {expected}")


class DeviceUnavailable(DeformConvError):
    """The reference's `.metalUnavailable`: no usable CUDA device."""

    status = _native.DCN_ERR_NO_DEVICE

    def __init__(self, message: str = "No CUDA device is available"):
        super().__init__(message)


class Unsupported(DeformConvError):
    """The reference's `.shaderResourceMissing` / shape guards: no kernel for this case."""

    status = _native.DCN_ERR_UNSUPPORTED


class NonFiniteOutput(DeformConvError):
    status = _native.DCN_ERR_NONFINITE

    def __init__(self, message: str):
        super().__init__(f"CUDA DCNv2 produced non-finite output: {message}")

    @property
    def is_recoverable_numerical_failure(self) -> bool:
        return True


class CommandFailed(DeformConvError):
    status = _native.DCN_ERR_LAUNCH

    def __init__(self, message: str):
        super().__init__(f"CUDA command failed: {message}")


class InvalidArgument(DeformConvError):
    status = _native.DCN_ERR_INVALID_ARGUMENT


class DeviceTimeout(DeformConvError):
    status = _native.DCN_ERR_DEVICE_TIMEOUT


def raise_for_status(status: int, context: str = "") -> None:
    """Maps a dcn_status to the matching exception (no-op for DCN_OK)."""
    if status == _native.DCN_OK:
        return
    text = _native.status_string(status)
    msg = f"{context}: {text}" if context else text
    if status == _native.DCN_ERR_INVALID_SHAPE:
        raise InvalidShape(msg)
    if status == _native.DCN_ERR_NO_DEVICE:
        raise DeviceUnavailable(msg)
    if status == _native.DCN_ERR_UNSUPPORTED:
        raise Unsupported(msg)
    if status == _native.DCN_ERR_NONFINITE:
        raise NonFiniteOutput(msg)
    if status == _native.DCN_ERR_INVALID_ARGUMENT:
        raise InvalidArgument(msg)
    if status == _native.DCN_ERR_DEVICE_TIMEOUT:
        raise DeviceTimeout(msg)
    if status == _native.DCN_ERR_INVALID_COUNT:
        raise DeformConvError(msg)
    raise CommandFailed(msg)


# ----------------------------------------------------------------------------- shape


@dataclass(frozen=True)
class TemporalPreparationResult:
    """TemporalPreparationResult (MetalRunner.swift:60-65): FP16 host arrays."""
    gpu_milliseconds: float
    conditions: np.ndarray        # [196 * plane]
    deform_input: np.ndarray      # [128 * plane]
    second_order_flow: np.ndarray  # [2 * plane]


@dataclass(frozen=True)
class TemporalPreparationProbeResult:
    """TemporalPreparationProbeResult (TemporalPreparationProbe.swift:3-12)."""
    median_milliseconds: float
    minimum_milliseconds: float
    maximum_milliseconds: float
    iterations: int
    maximum_magnitude: float
    repeat_maximum_error: float
    first_order_zero_maximum_error: float
    checksum: float


@dataclass(frozen=True)
class DeformConvShape:
    """`struct DeformConvShape` (DeformConv.swift:3-42), same fields in the same order."""

    batch: int
    input_channels: int
    input_height: int
    input_width: int
    output_channels: int
    output_height: int
    output_width: int
    kernel_height: int
    kernel_width: int
    pad_height: int
    pad_width: int
    stride_height: int
    stride_width: int
    dilation_height: int
    dilation_width: int
    groups: int
    offset_groups: int

    # Derived counts (DeformConv.swift:22-27).
    @property
    def input_count(self) -> int:
        return self.batch * self.input_channels * self.input_height * self.input_width

    @property
    def output_count(self) -> int:
        return self.batch * self.output_channels * self.output_height * self.output_width

    @property
    def kernel_area(self) -> int:
        return self.kernel_height * self.kernel_width

    @property
    def offset_count(self) -> int:
        return self.batch * 2 * self.offset_groups * self.kernel_area * self.output_height * self.output_width

    @property
    def mask_count(self) -> int:
        return self.batch * self.offset_groups * self.kernel_area * self.output_height * self.output_width

    @property
    def weight_count(self) -> int:
        return self.output_channels * (self.input_channels // self.groups) * self.kernel_area

    @property
    def output_pixels(self) -> int:
        return self.batch * self.output_height * self.output_width

    def validate(self) -> None:
        """DeformConvShape.validate (DeformConv.swift:29-41), plus this build's 32-bit index limits."""
        c = self.to_c()
        raise_for_status(_native.load().dcn_shape_validate(ctypes.byref(c)))

    def validate_reference(self) -> bool:
        """The reference's own predicate only (no library needed)."""
        s = self
        return (
            s.batch > 0 and s.input_channels > 0 and s.output_channels > 0
            and s.input_height > 0 and s.input_width > 0
            and s.output_height > 0 and s.output_width > 0
            and s.kernel_height > 0 and s.kernel_width > 0
            and s.groups > 0 and s.offset_groups > 0
            and s.input_channels % s.groups == 0
            and s.output_channels % s.groups == 0
            and s.input_channels % s.offset_groups == 0
        )

    def to_c(self) -> _native.DcnShape:
        return _native.DcnShape(*[getattr(self, f.name) for f in fields(self)])

    def with_batch(self, batch: int) -> "DeformConvShape":
        values = {f.name: getattr(self, f.name) for f in fields(self)}
        values["batch"] = batch
        return DeformConvShape(**values)

    def as_tuple(self) -> tuple[int, ...]:
        return tuple(getattr(self, f.name) for f in fields(self))

    @classmethod
    def jasna_propagation(cls, batch: int = 1, height: int = 64, width: int = 64) -> "DeformConvShape":
        """BasicVSR++ propagation alignment: 128 -> 64 channels, 3x3, pad 1, 16 deformable
        groups (PropagationDeformConvShape, MetalMLProbe.swift:47-66; MetalRunner.swift:191-209)."""
        return cls(batch, 128, height, width, 64, height, width, 3, 3, 1, 1, 1, 1, 1, 1, 1, 16)


def check_counts(shape: DeformConvShape, input, offset, mask, weight, bias) -> None:
    """DeformConvCPU.require (DeformConv.swift:85-89, :140-144) for array-likes."""
    names = ("input", "offset", "mask", "weight", "bias")
    expected = (shape.input_count, shape.offset_count, shape.mask_count, shape.weight_count,
                shape.output_channels)
    for name, arr, want in zip(names, (input, offset, mask, weight, bias), expected):
        n = int(np.prod(arr.shape)) if hasattr(arr, "shape") else len(arr)
        if n != want:
            raise InvalidArrayCount(name, want, n)


# ----------------------------------------------------------------------------- operator


def _torch():
    import torch

    return torch


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(stream) -> int | None:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None


class CudaDeformConv:
    """The CUDA counterpart of `MetalDeformConv` (MetalRunner.swift:92-388).

    Device-tensor methods (``forward_*``, ``prepack``, ``flag_non_finite``,
    ``prepare_offsets``) take CUDA tensors and enqueue work on the current (or
    given) stream; host methods (``run_float32``, ``run_float16``) take numpy
    arrays, copy them to the device, run, synchronise and return numpy arrays,
    like the reference's synchronous ``runFloat32``.
    """

    def __init__(self, device: int | None = None):
        torch = _torch()
        self.lib = _native.load()
        if not torch.cuda.is_available():
            raise DeviceUnavailable()
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)

    # -- queries ---------------------------------------------------------------
    def path(self, shape: DeformConvShape) -> int:
        return self.lib.dcn_forward_f16_path(ctypes.byref(shape.to_c()))

    def plan(self, shape: DeformConvShape) -> dict:
        """dcn_forward_f16_plan: path, group splits, tiles per unit, launches per call, grid and
        images converted by the pre-pass, on this operator's device."""
        torch = _torch()
        out = _native.DcnPlan()
        with torch.cuda.device(self.device):
            st = self.lib.dcn_forward_f16_plan(ctypes.byref(shape.to_c()), ctypes.byref(out))
        raise_for_status(st, "dcn_forward_f16_plan")
        return {name: int(getattr(out, name)) for name, _ in _native.DcnPlan._fields_}

    def packed_weight_bytes(self, shape: DeformConvShape) -> int:
        return int(self.lib.dcn_packed_weight_bytes(ctypes.byref(shape.to_c())))

    def workspace_bytes(self, shape: DeformConvShape) -> int:
        return int(self.lib.dcn_forward_f16_workspace_bytes(ctypes.byref(shape.to_c())))

    def grouped_input_bytes(self, shape: DeformConvShape) -> int:
        """Bytes of the grouped input at the start of the workspace: zero-bordered slabs on the slab
        path, corner pairs on the global-gather path, 0 on the direct path."""
        path = self.path(shape)
        n, g, h, w = shape.batch, shape.offset_groups, shape.input_height, shape.input_width
        if path == _native.DCN_PATH_SLAB_TC:
            return n * g * (h + 2) * (w + 2) * 16
        if path == _native.DCN_PATH_FUSED_TC:
            return n * g * h * (w + 1) * 32
        return 0

    def raw_workspace_bytes(self, shape: DeformConvShape) -> int:
        """Scratch of forward_f16_raw; 0 when the shape has no raw form (odd group count or direct path)."""
        return int(self.lib.dcn_forward_f16_raw_workspace_bytes(ctypes.byref(shape.to_c())))

    # -- device-tensor API -----------------------------------------------------
    def _check_device(self, *tensors) -> None:
        for t in tensors:
            if t is not None and (not t.is_cuda or not t.is_contiguous()):
                raise InvalidArgument("tensors must be contiguous CUDA tensors")

    def forward_f32(self, shape, input, offset, mask, weight, bias, out=None, stream=None):
        """deform_conv2d_fp32 (MetalShader.swift:76-124) on device tensors; bit-exact with the CPU reference."""
        torch = _torch()
        check_counts(shape, input, offset, mask, weight, bias)
        if out is None:
            out = torch.empty(shape.output_count, dtype=torch.float32, device=input.device)
        self._check_device(input, offset, mask, weight, bias, out)
        with torch.cuda.device(input.device):
            st = self.lib.dcn_forward_f32(
                ctypes.byref(shape.to_c()), _ptr(input), _ptr(offset), _ptr(mask), _ptr(weight), _ptr(bias),
                _ptr(out), _stream_handle(stream))
        raise_for_status(st, "dcn_forward_f32")
        return out

    def forward_f16_direct(self, shape, input, offset, mask, weight_oihw, bias, out=None, stream=None):
        """deform_conv2d_fp16 (MetalShader.swift:126-174): FP16 storage, FP32 math, OIHW weights."""
        torch = _torch()
        check_counts(shape, input, offset, mask, weight_oihw, bias)
        if out is None:
            out = torch.empty(shape.output_count, dtype=torch.float16, device=input.device)
        self._check_device(input, offset, mask, weight_oihw, bias, out)
        with torch.cuda.device(input.device):
            st = self.lib.dcn_forward_f16_direct(
                ctypes.byref(shape.to_c()), _ptr(input), _ptr(offset), _ptr(mask), _ptr(weight_oihw),
                _ptr(bias), _ptr(out), _stream_handle(stream))
        raise_for_status(st, "dcn_forward_f16_direct")
        return out

    def prepack(self, shape, weight, layout: int = _native.DCN_WEIGHT_OIHW, stream=None):
        """Weight prepack kernel: FP32/FP16 OIHW or [ic][k][oc] -> the opaque packed FP16 weight."""
        torch = _torch()
        if int(np.prod(weight.shape)) != shape.weight_count:
            raise InvalidArrayCount("weight", shape.weight_count, int(np.prod(weight.shape)))
        dtype = {torch.float32: _native.DCN_DTYPE_F32, torch.float16: _native.DCN_DTYPE_F16}.get(weight.dtype)
        if dtype is None:
            raise InvalidArgument("weight must be float32 or float16")
        nbytes = self.packed_weight_bytes(shape)
        if nbytes == 0:
            raise InvalidShape()
        packed = torch.empty(nbytes, dtype=torch.uint8, device=weight.device)
        self._check_device(weight, packed)
        with torch.cuda.device(weight.device):
            st = self.lib.dcn_prepack_weights(ctypes.byref(shape.to_c()), _ptr(weight), dtype, layout,
                                              _ptr(packed), _stream_handle(stream))
        raise_for_status(st, "dcn_prepack_weights")
        return packed

    @staticmethod
    def _io(shape, input, input_second, out_image_channels, out_channel_offset):
        """The dcn_io of a call and the element counts of its input/output tensors."""
        if input_second is None and out_image_channels is None and out_channel_offset == 0:
            return None, shape.input_count, shape.output_count
        plane = shape.input_height * shape.input_width
        io = _native.DcnIo()
        in_count = shape.input_count
        if input_second is not None:
            first_ch = input.numel() // (shape.batch * plane)
            second_ch = input_second.numel() // (shape.batch * plane)
            if first_ch + second_ch != shape.input_channels or first_ch * shape.batch * plane != input.numel():
                raise InvalidArrayCount("input + input_second", shape.input_count,
                                        input.numel() + input_second.numel())
            io.input_second = _ptr(input_second)
            io.input_split = first_ch
            in_count = input.numel()
        out_count = shape.output_count
        if out_image_channels is not None:
            io.output_image_channels = out_image_channels
            io.output_channel_offset = out_channel_offset
            out_count = shape.batch * out_image_channels * shape.output_height * shape.output_width
        else:
            io.output_channel_offset = out_channel_offset
        return io, in_count, out_count

    def forward_f16(self, shape, input, offset, mask, packed_weight, bias, out=None, flag=None,
                    workspace=None, stream=None, input_second=None, out_image_channels=None,
                    out_channel_offset=0):
        """Fused FP16 DCNv2 (gather + tcgen05 GEMM + epilogue); replaces the reference's
        gather + SIMD-group GEMM + non-finite-flag passes (MetalShader.swift:299-463).

        `input_second` (channels [split, C) of the input, `input` then holding [0, split))
        and `out_image_channels`/`out_channel_offset` (write channels [offset, offset+OC) of
        an output tensor with that many channels per image) read and write the caller's
        tensors in place, as dcn_forward_f16_io does."""
        torch = _torch()
        io, in_count, out_count = self._io(shape, input, input_second, out_image_channels, out_channel_offset)
        for name, arr, want in (("input", input, in_count), ("offset", offset, shape.offset_count),
                                ("mask", mask, shape.mask_count), ("bias", bias, shape.output_channels)):
            if arr.numel() != want:
                raise InvalidArrayCount(name, want, arr.numel())
        if out is None:
            out = torch.empty(out_count, dtype=torch.float16, device=input.device)
        elif out.numel() != out_count:
            raise InvalidArrayCount("output", out_count, out.numel())
        ws_bytes = self.workspace_bytes(shape)
        if workspace is None and ws_bytes > 0:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=input.device)
        self._check_device(input, input_second, offset, mask, packed_weight, bias, out, flag, workspace)
        with torch.cuda.device(input.device):
            st = self.lib.dcn_forward_f16_io(
                ctypes.byref(shape.to_c()), None if io is None else ctypes.byref(io), _ptr(input), _ptr(offset),
                _ptr(mask), _ptr(packed_weight), _ptr(bias), _ptr(out), _ptr(flag), _ptr(workspace),
                0 if workspace is None else workspace.numel() * workspace.element_size(), _stream_handle(stream))
        raise_for_status(st, "dcn_forward_f16")
        return out

    def regroup_input(self, shape, input, workspace=None, stream=None):
        """NCHW FP16 -> the fused kernel's [N][C/8][H][W][8] layout (the pre-pass of forward_f16)."""
        torch = _torch()
        ws_bytes = self.workspace_bytes(shape)
        if ws_bytes == 0:
            raise Unsupported("shape does not take the fused path")
        if workspace is None:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=input.device)
        self._check_device(input, workspace)
        st = self.lib.dcn_regroup_input_f16(ctypes.byref(shape.to_c()), _ptr(input), _ptr(workspace),
                                            workspace.numel() * workspace.element_size(), _stream_handle(stream))
        raise_for_status(st, "dcn_regroup_input_f16")
        return workspace

    def regroup_input_nhwc(self, shape, input_nhwc, workspace=None, stream=None):
        """regroup_input for a channels-last input [N][H][W][C] FP16 (dcn_regroup_input_nhwc_f16):
        the same grouped bytes at the start of the workspace."""
        torch = _torch()
        ws_bytes = self.workspace_bytes(shape)
        if ws_bytes == 0:
            raise Unsupported("shape does not take a tensor-core path")
        if workspace is None:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=input_nhwc.device)
        self._check_device(input_nhwc, workspace)
        st = self.lib.dcn_regroup_input_nhwc_f16(ctypes.byref(shape.to_c()), _ptr(input_nhwc), _ptr(workspace),
                                                 workspace.numel() * workspace.element_size(),
                                                 _stream_handle(stream))
        raise_for_status(st, "dcn_regroup_input_nhwc_f16")
        return workspace

    def forward_f16_grouped(self, shape, input_grouped, offset, mask, packed_weight, bias, out=None, flag=None,
                            stream=None):
        """The fused gather + tcgen05 kernel alone, on an input already in the grouped layout."""
        torch = _torch()
        if out is None:
            out = torch.empty(shape.output_count, dtype=torch.float16, device=offset.device)
        self._check_device(input_grouped, offset, mask, packed_weight, bias, out, flag)
        st = self.lib.dcn_forward_f16_grouped(
            ctypes.byref(shape.to_c()), _ptr(input_grouped), _ptr(offset), _ptr(mask), _ptr(packed_weight),
            _ptr(bias), _ptr(out), _ptr(flag), _stream_handle(stream))
        raise_for_status(st, "dcn_forward_f16_grouped")
        return out

    def forward_f16_raw(self, shape, input, raw, flow1, flow2, packed_weight, bias, out=None, flag=None,
                        workspace=None, stream=None, input_second=None, out_image_channels=None,
                        out_channel_offset=0):
        """Offset producer + DCNv2 in one operator: `raw` is the offset network's output
        [N][3*G*9][Ho][Wo] (residues, then mask logits), flows [N][2][Ho][Wo] in (x, y) order;
        replaces prepare_dcn_offsets_fp16 (MetalShader.swift:817-839) followed by the convolution.
        The tensor-plumbing arguments are those of forward_f16 (dcn_forward_f16_raw_io)."""
        torch = _torch()
        io, in_count, out_count = self._io(shape, input, input_second, out_image_channels, out_channel_offset)
        gka = shape.offset_groups * shape.kernel_area
        plane = shape.output_height * shape.output_width
        for name, arr, want in (("input", input, in_count), ("raw", raw, shape.batch * 3 * gka * plane),
                                ("flow1", flow1, shape.batch * 2 * plane), ("flow2", flow2, shape.batch * 2 * plane),
                                ("bias", bias, shape.output_channels)):
            if arr.numel() != want:
                raise InvalidArrayCount(name, want, arr.numel())
        if out is None:
            out = torch.empty(out_count, dtype=torch.float16, device=input.device)
        elif out.numel() != out_count:
            raise InvalidArrayCount("output", out_count, out.numel())
        ws_bytes = self.raw_workspace_bytes(shape)
        if ws_bytes == 0:
            raise Unsupported("shape does not take a tensor-core path with an even deformable-group count")
        if workspace is None:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=input.device)
        self._check_device(input, input_second, raw, flow1, flow2, packed_weight, bias, out, flag, workspace)
        with torch.cuda.device(input.device):
            st = self.lib.dcn_forward_f16_raw_io(
                ctypes.byref(shape.to_c()), None if io is None else ctypes.byref(io), _ptr(input), _ptr(raw),
                _ptr(flow1), _ptr(flow2), _ptr(packed_weight),
                _ptr(bias), _ptr(out), _ptr(flag), _ptr(workspace), workspace.numel() * workspace.element_size(),
                _stream_handle(stream))
        raise_for_status(st, "dcn_forward_f16_raw")
        return out

    def forward_f16_raw_grouped(self, shape, workspace, raw, flow1, flow2, packed_weight, bias, out=None, flag=None,
                                stream=None):
        """The raw form (offset transform fused) on an input already in the grouped layout at the
        start of `workspace` (from regroup_input or temporal_prepare_slabs): forward_f16_raw
        without its pre-pass."""
        torch = _torch()
        if out is None:
            out = torch.empty(shape.output_count, dtype=torch.float16, device=raw.device)
        self._check_device(workspace, raw, flow1, flow2, packed_weight, bias, out, flag)
        st = self.lib.dcn_forward_f16_raw_grouped(
            ctypes.byref(shape.to_c()), _ptr(workspace), _ptr(raw), _ptr(flow1), _ptr(flow2), _ptr(packed_weight),
            _ptr(bias), _ptr(out), _ptr(flag), workspace.numel() * workspace.element_size(), _stream_handle(stream))
        raise_for_status(st, "dcn_forward_f16_raw_grouped")
        return out

    def flag_non_finite(self, values, flag, stream=None):
        """flag_non_finite_fp16 (MetalShader.swift:454-463)."""
        self._check_device(values, flag)
        st = self.lib.dcn_flag_non_finite_f16(_ptr(values), values.numel(), _ptr(flag), _stream_handle(stream))
        raise_for_status(st, "dcn_flag_non_finite_f16")
        return flag

    def prepare_offsets(self, plane: int, raw, flow1, flow2, offset=None, mask=None, stream=None):
        """prepare_dcn_offsets_fp16 (MetalShader.swift:817-839; MetalRunner.swift:469-508)."""
        torch = _torch()
        if raw.numel() != 432 * plane or flow1.numel() != 2 * plane or flow2.numel() != 2 * plane:
            raise InvalidShape()
        if offset is None:
            offset = torch.empty(288 * plane, dtype=torch.float16, device=raw.device)
        if mask is None:
            mask = torch.empty(144 * plane, dtype=torch.float16, device=raw.device)
        self._check_device(raw, flow1, flow2, offset, mask)
        st = self.lib.dcn_prepare_offsets_f16(plane, _ptr(raw), _ptr(flow1), _ptr(flow2), _ptr(offset),
                                              _ptr(mask), _stream_handle(stream))
        raise_for_status(st, "dcn_prepare_offsets_f16")
        return offset, mask

    def temporal_prepare(self, width: int, height: int, feat_prop, feat_current, feat_n2, flow1, previous_flow,
                         has_second_order: bool, batch: int = 1, conditions=None, deform_input=None,
                         with_deform_input: bool = True, flow2=None, stream=None):
        """accumulate_second_order_flow_fp16 + assemble_temporal_alignment_fp16
        (MetalShader.swift:736-813) on device FP16 tensors for `batch` frames, through
        dcn_temporal_prepare_f16.  Returns (conditions [batch*196*plane], deform_input
        [batch*128*plane] or None when `with_deform_input` is false, flow2 [batch*2*plane])."""
        torch = _torch()
        plane = width * height
        if width <= 0 or height <= 0 or batch <= 0:
            raise InvalidShape()
        for t, ch in ((feat_prop, 64), (feat_current, 64), (feat_n2, 64), (flow1, 2), (previous_flow, 2)):
            if t.numel() != batch * ch * plane:
                raise InvalidShape()
        dev = feat_prop.device
        if conditions is None:
            conditions = torch.empty(batch * 196 * plane, dtype=torch.float16, device=dev)
        if deform_input is None and with_deform_input:
            deform_input = torch.empty(batch * 128 * plane, dtype=torch.float16, device=dev)
        if flow2 is None:
            flow2 = torch.empty(batch * 2 * plane, dtype=torch.float16, device=dev)
        tensors = [feat_prop, feat_current, feat_n2, flow1, previous_flow, conditions, flow2]
        self._check_device(*tensors, *([deform_input] if deform_input is not None else []))
        st = self.lib.dcn_temporal_prepare_f16(batch, width, height, *[_ptr(t) for t in tensors[:5]],
                                               1 if has_second_order else 0, _ptr(conditions),
                                               _ptr(deform_input) if deform_input is not None else None,
                                               _ptr(flow2), _stream_handle(stream))
        raise_for_status(st, "dcn_temporal_prepare_f16")
        return conditions, deform_input, flow2

    def temporal_slabs_bytes(self, width: int, height: int, batch: int = 1) -> int:
        """Bytes of the deform input in the DCN's slab layout (0: the frame does not take that form)."""
        return int(self.lib.dcn_temporal_slabs_bytes(batch, width, height))

    def temporal_prepare_slabs(self, width: int, height: int, feat_prop, feat_current, feat_n2, flow1,
                               previous_flow, has_second_order: bool, batch: int = 1, workspace=None,
                               conditions=None, flow2=None, stream=None):
        """temporal_prepare with the deform input written in the DCN's slab layout at the start of
        `workspace` (dcn_temporal_prepare_slabs_f16); by default a new workspace of the size the DCN
        of DeformConvShape.jasna_propagation(batch, height, width) takes, which forward_f16_grouped
        and forward_f16_raw_grouped then read without a pre-pass.  Returns (conditions, workspace,
        flow2).  Raises Unsupported for frames the slab form does not take."""
        torch = _torch()
        plane = width * height
        if width <= 0 or height <= 0 or batch <= 0:
            raise InvalidShape()
        for t, ch in ((feat_prop, 64), (feat_current, 64), (feat_n2, 64), (flow1, 2), (previous_flow, 2)):
            if t.numel() != batch * ch * plane:
                raise InvalidShape()
        dev = feat_prop.device
        if workspace is None:
            need = max(self.temporal_slabs_bytes(width, height, batch),
                       self.workspace_bytes(DeformConvShape.jasna_propagation(batch, height, width)))
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        if conditions is None:
            conditions = torch.empty(batch * 196 * plane, dtype=torch.float16, device=dev)
        if flow2 is None:
            flow2 = torch.empty(batch * 2 * plane, dtype=torch.float16, device=dev)
        tensors = [feat_prop, feat_current, feat_n2, flow1, previous_flow, conditions, flow2, workspace]
        self._check_device(*tensors)
        st = self.lib.dcn_temporal_prepare_slabs_f16(batch, width, height, *[_ptr(t) for t in tensors[:5]],
                                                     1 if has_second_order else 0, _ptr(conditions), _ptr(flow2),
                                                     _ptr(workspace), workspace.numel() * workspace.element_size(),
                                                     _stream_handle(stream))
        raise_for_status(st, "dcn_temporal_prepare_slabs_f16")
        return conditions, workspace, flow2

    def device_error(self) -> None:
        """Raises DeviceTimeout if a kernel's bounded device-side wait expired since the last check."""
        raise_for_status(self.lib.dcn_device_error(), "device error word")

    def host_workspace_bytes(self, shape: DeformConvShape, chunk_images: int = 0) -> int:
        """Device staging memory of forward_f16_host (dcn_forward_f16_host_workspace_bytes)."""
        return int(self.lib.dcn_forward_f16_host_workspace_bytes(ctypes.byref(shape.to_c()), chunk_images))

    def forward_f16_host(self, shape, input_host, offset_host, mask_host, packed_weight, bias, out_host,
                         chunk_images: int = 0, workspace=None, stream=None, check: bool = True) -> int:
        """End-to-end FP16 operator on HOST buffers through dcn_forward_f16_host: the library
        cuts the batch into chunks of images and pipelines each chunk's host->device copies,
        kernels and device->host copy on its own streams (up to three chunks in flight).  Host
        tensors should be pinned (torch pin_memory) for the copies to overlap.  Synchronises
        the stream, reads the non-finite flag (a 4-byte device->host copy inside the call) and
        returns it; raises NonFiniteOutput if it is set and `check`."""
        torch = _torch()
        dev = packed_weight.device
        for name, arr, want in (("input", input_host, shape.input_count), ("offset", offset_host, shape.offset_count),
                                ("mask", mask_host, shape.mask_count), ("output", out_host, shape.output_count)):
            if arr.numel() != want:
                raise InvalidArrayCount(name, want, arr.numel())
            if arr.is_cuda or arr.dtype != torch.float16 or not arr.is_contiguous():
                raise InvalidArgument(f"{name} must be a contiguous FP16 host tensor")
        ws_bytes = self.host_workspace_bytes(shape, chunk_images)
        if ws_bytes == 0:
            raise Unsupported("shape does not take a tensor-core path")
        if workspace is None:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        self._check_device(packed_weight, bias, workspace)
        flag_host = ctypes.c_uint32(0xFFFFFFFF)
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        with torch.cuda.device(dev):
            st = self.lib.dcn_forward_f16_host(
                ctypes.byref(shape.to_c()), _ptr(input_host), _ptr(offset_host), _ptr(mask_host), _ptr(packed_weight),
                _ptr(bias), _ptr(out_host), ctypes.addressof(flag_host), chunk_images, _ptr(workspace),
                workspace.numel() * workspace.element_size(), s.cuda_stream or None)
            raise_for_status(st, "dcn_forward_f16_host")
            s.synchronize()
        value = int(flag_host.value)
        if check and value & _native.DCN_FLAG_NONFINITE:
            raise NonFiniteOutput("Inf/NaN in the DCNv2 output")
        return value

    # -- host-array API (synchronous, like the reference) -------------------------
    def run_float32(self, shape: DeformConvShape, input, offset, mask, weight, bias) -> np.ndarray:
        """`runFloat32(shape:input:offset:mask:weight:bias:)` (MetalRunner.swift:159-185)."""
        torch = _torch()
        shape.validate()
        check_counts(shape, input, offset, mask, weight, bias)
        dev = self.device

        def up(a):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32).reshape(-1)).to(dev)

        out = self.forward_f32(shape, up(input), up(offset), up(mask), up(weight), up(bias))
        torch.cuda.synchronize(dev)
        self.device_error()
        return out.cpu().numpy()

    def run_float16(self, shape: DeformConvShape, input, offset, mask, weight, bias,
                    weight_layout: int = _native.DCN_WEIGHT_OIHW) -> np.ndarray:
        """FP16 operator on host arrays: prepack + fused (or direct) kernel + non-finite check.
        Raises NonFiniteOutput (the only recoverable error) if any output is Inf/NaN."""
        torch = _torch()
        shape.validate()
        check_counts(shape, input, offset, mask, weight, bias)
        dev = self.device

        def up(a):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16).reshape(-1)).to(dev)

        packed = self.prepack(shape, up(weight), weight_layout)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        out = self.forward_f16(shape, up(input), up(offset), up(mask), packed, up(bias), flag=flag)
        torch.cuda.synchronize(dev)
        self.device_error()
        if int(flag.item()) & _native.DCN_FLAG_NONFINITE:
            raise NonFiniteOutput("Inf/NaN in the DCNv2 output")
        return out.cpu().numpy()

    def run_dcn_offset_transform(self, plane: int, raw, flow1, flow2) -> tuple[np.ndarray, np.ndarray]:
        """`runDCNOffsetTransform(plane:raw:flow1:flow2:)` (MetalRunner.swift:469-508): the offset
        network's raw output (432 channels of `plane` pixels) and the two flows (2 channels each) as
        FP16 host arrays in; the DCN offsets (288 channels, 10*tanh(raw) plus the flow, y first)
        and the mask (144 channels, sigmoid(raw)) out as FP16 host arrays.  Sizes that do not match
        `plane` raise InvalidShape, as the reference throws invalidShape."""
        torch = _torch()
        arrays = [np.ascontiguousarray(a, dtype=np.float16).reshape(-1) for a in (raw, flow1, flow2)]
        if plane <= 0 or [a.size for a in arrays] != [432 * plane, 2 * plane, 2 * plane]:
            raise InvalidShape()
        dev = self.device
        offset, mask = self.prepare_offsets(plane, *(torch.from_numpy(a).to(dev) for a in arrays))
        torch.cuda.synchronize(dev)
        self.device_error()
        return offset.cpu().numpy(), mask.cpu().numpy()

    def run_temporal_preparation(self, width: int, height: int, feat_prop, feat_current, feat_n2, flow1,
                                 previous_flow, has_second_order: bool) -> "TemporalPreparationResult":
        """`runTemporalPreparation(width:height:featProp:featCurrent:featN2:flow1:previousFlow:
        hasSecondOrder:)` (MetalRunner.swift:510-582): one frame of FP16 host arrays in, the
        conditions, the deform input and the second-order flow out (FP16 host arrays), with the
        GPU time of the call."""
        torch = _torch()
        plane = width * height
        arrays = [np.ascontiguousarray(a, dtype=np.float16).reshape(-1)
                  for a in (feat_prop, feat_current, feat_n2, flow1, previous_flow)]
        if width <= 0 or height <= 0 or [a.size for a in arrays] != [64 * plane] * 3 + [2 * plane] * 2:
            raise InvalidShape()
        dev = self.device
        ins = [torch.from_numpy(a).to(dev) for a in arrays]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        cond, di, flow2 = self.temporal_prepare(width, height, *ins, has_second_order)
        end.record()
        end.synchronize()
        self.device_error()
        return TemporalPreparationResult(float(start.elapsed_time(end)), cond.cpu().numpy(), di.cpu().numpy(),
                                         flow2.cpu().numpy())

    def verify_temporal_preparation(self, backward_flow, forward_flow) -> TemporalPreparationProbeResult:
        """`verifyTemporalPreparation(runner:backwardFlow:forwardFlow:)`
        (TemporalPreparationProbe.swift:14-101): 64x64 frames built with the probe's feature
        formula, each direction's flow used as both flow1 and the previous flow; two warm-up
        passes, then eight timed passes (backward + forward, GPU time each), then one first-order
        pass with zero feat_n2.  Raises CommandFailed, as the probe throws, unless the conditions
        are finite and not all tiny, the timed passes repeat within 0.001 and the first-order
        second-order flow is exactly zero."""
        torch = _torch()
        w = h = 64
        plane = w * h
        arrays = [np.ascontiguousarray(a, dtype=np.float16).reshape(-1) for a in (backward_flow, forward_flow)]
        if any(a.size != 2 * plane for a in arrays):
            raise InvalidShape()

        def features(seed):
            i = np.arange(64 * plane, dtype=np.int64)
            return ((((i * 37 + seed) % 509).astype(np.float32) / np.float32(508) - np.float32(0.5))
                    * np.float32(0.5)).astype(np.float16)

        dev = self.device
        up = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
        feat_prop, feat_current, feat_n2 = up(features(17)), up(features(31)), up(features(47))
        zero = torch.zeros(64 * plane, dtype=torch.float16, device=dev)
        flows = [up(a) for a in arrays]

        def execute(second_order):
            outs, ms = [], 0.0
            for flow in flows:
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                res = self.temporal_prepare(w, h, feat_prop, feat_current, feat_n2 if second_order else zero,
                                            flow, flow, second_order)
                end.record()
                end.synchronize()
                ms += float(start.elapsed_time(end))
                outs.append(res)
            self.device_error()
            return ms, outs

        execute(True)
        execute(True)
        first_ms, first = execute(True)
        samples, last = [first_ms], first
        for _ in range(1, 8):
            ms, last = execute(True)
            samples.append(ms)
        _, first_order = execute(False)
        samples.sort()
        max_mag = rep = zero_err = 0.0
        checksum = 0.0
        for d in range(2):
            cur = last[d][0].float().cpu().numpy()
            if not np.isfinite(cur).all():
                raise CommandFailed("temporal preparation produced a non-finite condition")
            max_mag = max(max_mag, float(np.abs(cur).max()))
            rep = max(rep, float(np.abs(first[d][0].float().cpu().numpy() - cur).max()))
            checksum += float(cur[::4099].astype(np.float64).sum())
            zero_err = max(zero_err, float(first_order[d][2].float().abs().max().item()))
        if not (max_mag > 0.001 and rep <= 0.001 and zero_err == 0.0):
            raise CommandFailed(f"temporal preparation validation failed (max={max_mag}, repeat={rep}, "
                                f"zero={zero_err})")
        return TemporalPreparationProbeResult(samples[len(samples) // 2], samples[0], samples[-1], len(samples),
                                              max_mag, rep, zero_err, checksum)

    # -- benchmark (benchmarkJasnaShape) ----------------------------------------
    def benchmark_jasna_shape(self, iterations: int = 20, weight_set=None, seed: int = 0x4A41534E41):
        """`benchmarkJasnaShape` (MetalRunner.swift:187-388): the Jasna propagation shape in FP16,
        direct kernel vs the fused tensor-core kernel, 2 warm-ups + `iterations` timed runs each
        (CUDA events), cross-variant gate <= 0.002 (MetalRunner.swift:350-354), checksum of every
        257th output (:335-337).  Inputs: U(-1,1) input, U(-0.25,0.25) offsets, U(0.25,0.75) mask,
        U(-0.02,0.02) weight/bias (:210-234), drawn from this package's seeded generator."""
        from . import synthetic

        torch = _torch()
        shape = DeformConvShape.jasna_propagation()
        rng = synthetic.SplitMix64(seed)
        dev = self.device
        to16 = lambda a: torch.from_numpy(a.astype(np.float16)).to(dev)  # noqa: E731
        x = to16(rng.uniform(shape.input_count, -1.0, 1.0))
        off = to16(rng.uniform(shape.offset_count, -0.25, 0.25))
        msk = to16(rng.uniform(shape.mask_count, 0.25, 0.75))
        if weight_set is not None:
            packed_ickoc, bias_np = weight_set.arrays()
            w_oihw = to16(np.transpose(packed_ickoc.reshape(128, 9, 64), (2, 0, 1)).reshape(-1))
            bias = to16(bias_np)
        else:
            w_oihw = to16(rng.uniform(shape.weight_count, -0.02, 0.02))
            bias = to16(rng.uniform(shape.output_channels, -0.02, 0.02))
        packed = self.prepack(shape, w_oihw)
        out_direct = torch.empty(shape.output_count, dtype=torch.float16, device=dev)
        out_fused = torch.empty_like(out_direct)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        ws = torch.empty(max(self.workspace_bytes(shape), 1), dtype=torch.uint8, device=dev)

        def timed(fn):
            samples = []
            for _ in range(2):
                fn()
            for _ in range(max(iterations, 1)):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn()
                b.record()
                b.synchronize()
                samples.append(a.elapsed_time(b))
            return BenchmarkStatistics.from_samples(samples)

        direct_stats = timed(lambda: self.forward_f16_direct(shape, x, off, msk, w_oihw, bias, out=out_direct))
        fused_stats = timed(lambda: self.forward_f16(shape, x, off, msk, packed, bias, out=out_fused, flag=flag,
                                                     workspace=ws))
        torch.cuda.synchronize(dev)
        self.device_error()
        diff = (out_fused.float() - out_direct.float()).abs().max().item()
        if not diff <= 0.002:
            raise CommandFailed(f"fused FP16 result differs from the direct kernel by {diff}")
        if direct_stats is None or fused_stats is None:
            raise CommandFailed("invalid DCNv2 benchmark samples")
        checksum = float(out_fused[::257].double().sum().item())
        return {
            "direct": direct_stats,
            "fused": fused_stats,
            "iterations": len(fused_stats.samples),
            "checksum": checksum,
            "max_difference_from_direct": diff,
            "nonfinite": bool(int(flag.item()) & _native.DCN_FLAG_NONFINITE),
        }
