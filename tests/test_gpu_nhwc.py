"""GPU: channels-last input for the tensor-core paths (dcn_regroup_input_nhwc_f16).

The reference's tensors are NCHW (S/DeformConv.swift:110-132); a host that keeps [N][H][W][C]
features calls this pre-pass and then dcn_forward_f16_grouped / dcn_forward_f16_raw_grouped.  The
grouped bytes it writes must equal what dcn_regroup_input_f16 writes for the same values in NCHW
(slab layout and corner-pair layout, borders included, into a workspace filled with 0xA5 first),
and the operator's output must be bit-identical to dcn_forward_f16 on the NCHW tensor."""

from __future__ import annotations

import numpy as np
import pytest

from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape, InvalidArgument, Unsupported

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,h,w,path", [(3, 64, 64, _native.DCN_PATH_SLAB_TC), (2, 40, 24, _native.DCN_PATH_SLAB_TC),
                                        (1, 96, 120, _native.DCN_PATH_FUSED_TC)],
                         ids=["slab_64x64x3", "slab_40x24x2_split", "pairs_96x120"])
def test_nhwc_input_matches_nchw(cuda_op, n, h, w, path):
    import torch

    shape = DeformConvShape.jasna_propagation(n, h, w)
    assert cuda_op.path(shape) == path
    g = torch.Generator(device="cuda").manual_seed(n * 1000 + h + w)
    x = torch.randn(shape.input_count, generator=g, device="cuda").half()
    x_nhwc = x.view(n, 128, h, w).permute(0, 2, 3, 1).contiguous().view(-1)
    off = (torch.rand(shape.offset_count, generator=g, device="cuda") * 24 - 12).half()
    msk = torch.rand(shape.mask_count, generator=g, device="cuda").half()
    wt, b = synthetic.weights(shape, 3)
    packed = cuda_op.prepack(shape, torch.from_numpy(wt).half().cuda())
    bias = torch.from_numpy(b).half().cuda()
    ref_ws = cuda_op.regroup_input(shape, x)
    ws = torch.full_like(ref_ws, 0xA5)
    cuda_op.regroup_input_nhwc(shape, x_nhwc, workspace=ws)
    grouped = (n * 16 * (h + 2) * (w + 2) * 16 if path == _native.DCN_PATH_SLAB_TC
               else n * 16 * h * (w + 1) * 32)
    torch.cuda.synchronize()
    assert torch.equal(ws[:grouped], ref_ws[:grouped])
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = cuda_op.forward_f16(shape, x, off, msk, packed, bias, flag=flag)
    got = cuda_op.forward_f16_grouped(shape, ws, off, msk, packed, bias, flag=flag)
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert int(flag.item()) == 0
    assert torch.equal(got, want)
    assert np.isfinite(got.float().cpu().numpy()).all()


def test_nhwc_rejections(cuda_op):
    import torch

    direct = DeformConvShape(1, 128, 8, 8, 32, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 16)
    with pytest.raises(Unsupported):
        cuda_op.regroup_input_nhwc(direct, torch.zeros(direct.input_count, dtype=torch.float16, device="cuda"),
                                   workspace=torch.empty(1 << 16, dtype=torch.uint8, device="cuda"))
    shape = DeformConvShape.jasna_propagation(1, 64, 64)
    buf = torch.zeros(shape.input_count + 8, dtype=torch.float16, device="cuda")
    with pytest.raises(InvalidArgument):  # 2-byte offset: not 16-byte aligned
        cuda_op.regroup_input_nhwc(shape, buf[1:1 + shape.input_count])
