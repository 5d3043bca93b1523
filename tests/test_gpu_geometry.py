"""GPU: convolution geometry on the tensor-core paths.  The sampling position of tap (ky, kx)
at output (oy, ox) is (oy*stride - pad + ky*dilation + dy, ox*stride - pad + kx*dilation + dx)
(DeformConv.swift:110-121); both tensor-core kernels take any stride, padding and dilation,
the slab kernel 3x3 kernels and the global-gather kernel any kernel size up to 144
(group, tap) pairs.  Each case is checked against the CPU oracle with the FP16 gates."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu

SLAB, PAIRS = _native.DCN_PATH_SLAB_TC, _native.DCN_PATH_FUSED_TC


def _shape(n, h, w, k, pad, stride, dil, og=16):
    """8 input channels per deformable group (the tensor-core class), 64 output channels."""
    kh, kw = k
    ho = (h + 2 * pad[0] - dil[0] * (kh - 1) - 1) // stride[0] + 1
    wo = (w + 2 * pad[1] - dil[1] * (kw - 1) - 1) // stride[1] + 1
    return DeformConvShape(n, 8 * og, h, w, 64, ho, wo, kh, kw, pad[0], pad[1], stride[0], stride[1], dil[0],
                           dil[1], 1, og)


CASES = [
    ("slab_stride2", _shape(2, 32, 32, (3, 3), (1, 1), (2, 2), (1, 1)), SLAB),
    ("slab_pad2_dil2", _shape(1, 40, 40, (3, 3), (2, 2), (1, 1), (2, 2)), SLAB),
    ("slab_stride2_dil2_pad0", _shape(3, 36, 36, (3, 3), (0, 0), (2, 2), (2, 2)), SLAB),
    ("slab_asymmetric", _shape(2, 24, 46, (3, 3), (2, 0), (1, 2), (1, 3)), SLAB),
    ("pairs_stride2", _shape(1, 64, 96, (3, 3), (1, 1), (2, 2), (1, 1)), PAIRS),
    ("pairs_5x5_og5", _shape(1, 72, 80, (5, 5), (2, 2), (1, 1), (1, 1), og=5), PAIRS),
    ("pairs_1x1", _shape(1, 72, 80, (1, 1), (0, 0), (1, 1), (1, 1)), PAIRS),
]


@pytest.mark.parametrize("name,shape,path", CASES, ids=[c[0] for c in CASES])
def test_tensor_core_geometry_matches_oracle(cuda_op, name, shape, path, host_threads):
    assert shape.output_height > 0 and shape.output_width > 0
    assert (shape.output_height * shape.output_width) % 8 == 0, name
    assert cuda_op.path(shape) == path, name
    g = synthetic.SplitMix64(sum(name.encode()) * 7919)
    x = synthetic.quantize_f16(g.normal(shape.input_count))
    off = synthetic.quantize_f16(g.uniform(shape.offset_count, -5.0, 5.0))
    msk = synthetic.quantize_f16(g.uniform(shape.mask_count, 0.0, 1.0))
    w, b = synthetic.weights(shape, 3)
    w, b = synthetic.quantize_f16(w), synthetic.quantize_f16(b)
    ref = oracle.run(shape, x, off, msk, w, b, threads=host_threads)
    out = cuda_op.run_float16(shape, x, off, msk, w, b).astype(np.float32)
    d = np.abs(out - ref)
    assert np.isfinite(out).all(), name
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (name, float(d.max()), float(d.mean()))
