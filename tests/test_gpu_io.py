"""GPU: tensor plumbing of dcn_forward_f16_io / dcn_forward_f16_raw_io -- the input read
from two tensors in place of the deformInput = [feat_prop, feat_n2] concatenation
(assemble_temporal_alignment_fp16, MetalShader.swift:769-813) and the output written into a
channel slot of a wider tensor in place of the backbone-input copy
(assemble_temporal_backbone_fp16, MetalShader.swift:903-929).

Each case runs the same inputs through the plain entry point (one concatenated input, a
plain output) and through the plumbing entry point, on every path: the written slot must
equal the plain output bit for bit, the other channels must keep their contents (filled with
+Inf, which also checks that the non-finite flag looks only at the slot), and the plain output
is checked against the CPU oracle."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape, InvalidArgument

pytestmark = pytest.mark.gpu

F16_MAX_ABS = 2e-2
F16_MEAN_ABS = 2e-3

CASES = [
    # shape, expected path, input split, output channels per image, output channel offset
    (DeformConvShape.jasna_propagation(3, 64, 64), _native.DCN_PATH_SLAB_TC, 64, 192, 128),
    (DeformConvShape.jasna_propagation(1, 64, 96), _native.DCN_PATH_FUSED_TC, 64, 128, 64),
    (DeformConvShape.jasna_propagation(2, 5, 7), _native.DCN_PATH_DIRECT, 37, 96, 17),
]


def _inputs(shape, seed):
    g = synthetic.SplitMix64(seed)
    x = synthetic.quantize_f16(g.normal(shape.input_count))
    off = synthetic.quantize_f16(g.normal(shape.offset_count, 0.0, 4.0))
    msk = synthetic.quantize_f16(synthetic.sigmoid(g.normal(shape.mask_count)))
    w, b = synthetic.weights(shape, seed + 1)
    return x, off, msk, synthetic.quantize_f16(w), synthetic.quantize_f16(b)


def _split(x, shape, split):
    import torch

    v = x.view(shape.batch, shape.input_channels, -1)
    return v[:, :split].contiguous().view(-1), v[:, split:].contiguous().view(-1)


@pytest.mark.parametrize("shape,path,split,out_ch,out_off", CASES, ids=["slab", "global_gather", "direct"])
def test_split_input_and_output_slot_match_plain_call(cuda_op, shape, path, split, out_ch, out_off, host_threads):
    import torch

    assert cuda_op.path(shape) == path
    x, off, msk, w, b = _inputs(shape, 901)
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    xd, offd, mskd, wd, bd = dev(x), dev(off), dev(msk), dev(w), dev(b)
    packed = cuda_op.prepack(shape, wd)
    plain = cuda_op.forward_f16(shape, xd, offd, mskd, packed, bd)

    first, second = _split(xd, shape, split)
    plane = shape.output_height * shape.output_width
    big = torch.full((shape.batch, out_ch, plane), float("inf"), dtype=torch.float16, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    cuda_op.forward_f16(shape, first, offd, mskd, packed, bd, out=big.view(-1), flag=flag, input_second=second,
                        out_image_channels=out_ch, out_channel_offset=out_off)
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert int(flag.item()) == 0, "the flag must only look at the written slot"
    slot = big[:, out_off:out_off + shape.output_channels]
    assert torch.equal(slot.reshape(-1), plain), "slot differs from the plain call"
    rest = torch.cat([big[:, :out_off], big[:, out_off + shape.output_channels:]], dim=1)
    assert bool(torch.isinf(rest).all()), "channels outside the slot were written"

    ref = oracle.run(shape, x, off, msk, w, b, threads=host_threads)
    d = np.abs(plain.float().cpu().numpy() - ref)
    assert d.max() <= F16_MAX_ABS and d.mean() <= F16_MEAN_ABS, (float(d.max()), float(d.mean()))


def test_raw_form_with_split_input_and_output_slot(cuda_op):
    import torch

    shape = DeformConvShape.jasna_propagation(2, 64, 64)
    plane = shape.output_height * shape.output_width
    x, _, _, w, b = _inputs(shape, 902)
    g = synthetic.SplitMix64(903)
    raw = synthetic.quantize_f16(g.normal(shape.batch * 432 * plane))
    f1 = synthetic.quantize_f16(g.uniform(shape.batch * 2 * plane, -16, 16))
    f2 = synthetic.quantize_f16(g.uniform(shape.batch * 2 * plane, -16, 16))
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    xd, wd, bd = dev(x), dev(w), dev(b)
    packed = cuda_op.prepack(shape, wd)
    plain = cuda_op.forward_f16_raw(shape, xd, dev(raw), dev(f1), dev(f2), packed, bd)
    first, second = _split(xd, shape, 64)
    big = torch.full((shape.batch, 192, plane), float("inf"), dtype=torch.float16, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    cuda_op.forward_f16_raw(shape, first, dev(raw), dev(f1), dev(f2), packed, bd, out=big.view(-1), flag=flag,
                            input_second=second, out_image_channels=192, out_channel_offset=64)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    assert torch.equal(big[:, 64:128].reshape(-1), plain)
    assert bool(torch.isinf(big[:, :64]).all()) and bool(torch.isinf(big[:, 128:]).all())


def test_plumbing_arguments_are_validated(cuda_op):
    import torch

    shape = DeformConvShape.jasna_propagation(1, 64, 64)
    x, off, msk, w, b = _inputs(shape, 904)
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    xd, offd, mskd, bd = dev(x), dev(off), dev(msk), dev(b)
    packed = cuda_op.prepack(shape, dev(w))
    # A tensor-core path needs the split on a deformable-group boundary (8 channels).
    first, second = _split(xd, shape, 60)
    with pytest.raises(InvalidArgument):
        cuda_op.forward_f16(shape, first, offd, mskd, packed, bd, input_second=second)
    # The slot must fit in the output tensor.
    with pytest.raises(InvalidArgument):
        cuda_op.forward_f16(shape, xd, offd, mskd, packed, bd,
                            out=torch.empty(shape.output_count * 2, dtype=torch.float16, device="cuda"),
                            out_image_channels=128, out_channel_offset=65)
