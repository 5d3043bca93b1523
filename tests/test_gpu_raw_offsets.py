"""GPU: the offset producer fused into the convolution (dcn_forward_f16_raw) against the
reference chain -- prepare_dcn_offsets_fp16 (MetalShader.swift:817-839, restated in the oracle)
with its FP16 outputs, then the DCNv2 oracle -- and against the two-step GPU chain
(dcn_prepare_offsets_f16 + dcn_forward_f16), on the slab path (64x64 tiles) and on the
global-gather path (a 64x96 image, too large for a shared-memory slab)."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu


def _case(shape: DeformConvShape, seed: int):
    g = synthetic.SplitMix64(seed)
    plane = shape.output_height * shape.output_width
    n = shape.batch
    x = synthetic.quantize_f16(g.normal(shape.input_count))
    raw = synthetic.quantize_f16(g.normal(n * 432 * plane))
    flow1 = synthetic.quantize_f16(g.uniform(n * 2 * plane, -16, 16))
    flow2 = synthetic.quantize_f16(g.uniform(n * 2 * plane, -16, 16))
    w, b = synthetic.weights(shape, seed + 1)
    return x, raw, flow1, flow2, synthetic.quantize_f16(w), synthetic.quantize_f16(b)


@pytest.mark.parametrize("shape,path", [
    (DeformConvShape.jasna_propagation(3, 64, 64), _native.DCN_PATH_SLAB_TC),
    (DeformConvShape.jasna_propagation(1, 64, 96), _native.DCN_PATH_FUSED_TC),
], ids=["slab", "global_gather"])
def test_raw_offsets_match_reference_chain(cuda_op, shape, path, host_threads):
    import torch

    assert cuda_op.path(shape) == path
    plane = shape.output_height * shape.output_width
    x, raw, f1, f2, w, b = _case(shape, 77)
    # Reference chain on the CPU: the offset transform per image, FP16 intermediates, the oracle DCN.
    offs, msks = [], []
    for i in range(shape.batch):
        o, m = oracle.prepare_offsets(plane, raw[i * 432 * plane:(i + 1) * 432 * plane],
                                      f1[i * 2 * plane:(i + 1) * 2 * plane], f2[i * 2 * plane:(i + 1) * 2 * plane])
        offs.append(synthetic.quantize_f16(o))
        msks.append(synthetic.quantize_f16(m))
    off, msk = np.concatenate(offs), np.concatenate(msks)
    ref = oracle.run(shape, x, off, msk, w, b, threads=host_threads)

    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    packed = cuda_op.prepack(shape, dev(w))
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    fused = cuda_op.forward_f16_raw(shape, dev(x), dev(raw), dev(f1), dev(f2), packed, dev(b), flag=flag)
    # Two-step GPU chain: the reference's offset kernel per frame, then the operator.
    o_dev = torch.empty(shape.offset_count, dtype=torch.float16, device="cuda")
    m_dev = torch.empty(shape.mask_count, dtype=torch.float16, device="cuda")
    for i in range(shape.batch):
        cuda_op.prepare_offsets(plane, dev(raw[i * 432 * plane:(i + 1) * 432 * plane]),
                                dev(f1[i * 2 * plane:(i + 1) * 2 * plane]), dev(f2[i * 2 * plane:(i + 1) * 2 * plane]),
                                offset=o_dev[i * 288 * plane:(i + 1) * 288 * plane],
                                mask=m_dev[i * 144 * plane:(i + 1) * 144 * plane])
    two_step = cuda_op.forward_f16(shape, dev(x), o_dev, m_dev, packed, dev(b))
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert int(flag.item()) == 0
    fused_np = fused.float().cpu().numpy()
    d = np.abs(fused_np - ref)
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (float(d.max()), float(d.mean()))
    d2 = np.abs(fused_np - two_step.float().cpu().numpy())
    assert d2.mean() <= 2e-3 and d2.max() <= 2e-2, (float(d2.max()), float(d2.mean()))


def test_raw_entry_rejects_direct_shapes(cuda_op):
    from jasnamacos_b200.deform_conv import Unsupported

    import torch

    s = DeformConvShape.jasna_propagation(1, 5, 5)  # direct path
    z = torch.zeros(1, dtype=torch.float16, device="cuda")
    with pytest.raises((Unsupported, Exception)):
        cuda_op.forward_f16_raw(s, torch.zeros(s.input_count, dtype=torch.float16, device="cuda"),
                                torch.zeros(432 * 25, dtype=torch.float16, device="cuda"),
                                torch.zeros(50, dtype=torch.float16, device="cuda"),
                                torch.zeros(50, dtype=torch.float16, device="cuda"), z, z)
