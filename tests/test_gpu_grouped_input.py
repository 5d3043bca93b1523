"""GPU: the grouped input form of the slab path, written by the caller.

dcn_forward_f16_grouped takes the input already in the slab layout that the regroup pre-pass
of dcn_forward_f16 would produce: [N][C/8][H+2][W+2][8] FP16, element (n, g, y+1, x+1, c) =
input[n][8g+c][y][x], with a one-pixel ring of zeros.  An upstream kernel that writes its
features in this layout (the reference's assemble_temporal_alignment_fp16 writes the DCN
input, Sources/JasnaMetalPoC/MetalShader.swift:769-813) removes the pre-pass from the
operator.  Here the layout is built with plain torch ops from the NCHW input -- not with the
library's regroup kernel -- and the result must equal dcn_forward_f16 bit for bit and pass
the FP16 gates against the CPU oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import _native, synthetic

pytestmark = pytest.mark.gpu


def slab_layout(x, n, c, h, w):
    """NCHW FP16 -> zero-bordered per-group slabs [N][C/8][H+2][W+2][8] (torch ops only)."""
    import torch

    t = x.view(n, c // 8, 8, h, w).permute(0, 1, 3, 4, 2)  # [N][G][H][W][8]
    out = torch.zeros(n, c // 8, h + 2, w + 2, 8, dtype=x.dtype, device=x.device)
    out[:, :, 1:h + 1, 1:w + 1, :] = t
    return out.reshape(-1)


@pytest.mark.parametrize("batch,h,w", [(160, 64, 64), (2, 16, 24)], ids=["160_tiles", "2x16x24_split"])
def test_caller_written_slabs_match_the_operator(cuda_op, batch, h, w):
    import torch

    from jasnamacos_b200.deform_conv import DeformConvShape

    shape = DeformConvShape.jasna_propagation(batch, h, w)
    assert cuda_op.path(shape) == _native.DCN_PATH_SLAB_TC
    x, off, msk, wt, b = synthetic.device_batch(shape, 16.0, seed=91, device="cuda")
    w16 = torch.from_numpy(wt).cuda().half()
    b16 = torch.from_numpy(b).cuda().half()
    packed = cuda_op.prepack(shape, w16)
    ref_dev = cuda_op.forward_f16(shape, x, off, msk, packed, b16)
    ws = torch.zeros(cuda_op.workspace_bytes(shape), dtype=torch.uint8, device="cuda")
    slabs = slab_layout(x, batch, 128, h, w)
    assert slabs.numel() * 2 <= ws.numel()
    ws[:slabs.numel() * 2].copy_(slabs.view(torch.uint8))
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = cuda_op.forward_f16_grouped(shape, ws, off, msk, packed, b16, flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    assert torch.equal(got, ref_dev)
    per = shape.with_batch(1)
    t = batch - 1
    ref = oracle.run(per, x[t * per.input_count:(t + 1) * per.input_count].float().cpu().numpy(),
                     off[t * per.offset_count:(t + 1) * per.offset_count].float().cpu().numpy(),
                     msk[t * per.mask_count:(t + 1) * per.mask_count].float().cpu().numpy(),
                     w16.float().cpu().numpy(), b16.float().cpu().numpy())
    d = np.abs(got[t * per.output_count:(t + 1) * per.output_count].float().cpu().numpy() - ref)
    assert float(d.max()) <= 2e-2 and float(d.mean()) <= 2e-3
