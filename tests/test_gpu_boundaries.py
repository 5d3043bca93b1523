"""GPU: hand-made sampling positions at the image boundary on both tensor-core paths, against
the CPU oracle.

Every (pixel, deformable group, tap) gets an offset that puts its sample on one of a few
absolute positions per axis: just outside (-1.5, -1), straddling the first row or column
(-0.75, -0.5), exactly on integer rows/columns (0, the last one), straddling the last one
(H-0.5), on or past the far edge (H, H+0.25), and one interior point.  These are the cases of
bilinear() in DeformConv.swift:146-165 where corners drop out one by one (zero padding per
corner, floor of negative positions); the slab kernel reads them from its zero-bordered
slabs, the global-gather kernel from its zero-padded corner pairs.  The targets are multiples
of 1/4, so every offset (target minus the pixel's base position) is exact in FP16 and the
oracle sees the very same positions."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu


def _targets(extent: int) -> np.ndarray:
    return np.array([-1.5, -1.0, -0.75, -0.5, 0.0, extent - 1.0, extent - 0.5, extent, extent + 0.25,
                     extent / 2.0 + 0.25], dtype=np.float64)


def _boundary_offsets(shape: DeformConvShape, seed: int) -> np.ndarray:
    """Offsets [N][2*G*9][Ho][Wo] that put every sample on a boundary target of each axis."""
    rng = np.random.default_rng(seed)
    n, g, ka = shape.batch, shape.offset_groups, shape.kernel_area
    ho, wo = shape.output_height, shape.output_width
    oy, ox = np.meshgrid(np.arange(ho), np.arange(wo), indexing="ij")
    off = np.empty((n, g, ka, 2, ho, wo), dtype=np.float64)
    ty_set, tx_set = _targets(shape.input_height), _targets(shape.input_width)
    for k in range(ka):
        ky, kx = divmod(k, shape.kernel_width)
        base_y = oy * shape.stride_height - shape.pad_height + ky * shape.dilation_height
        base_x = ox * shape.stride_width - shape.pad_width + kx * shape.dilation_width
        ty = rng.choice(ty_set, size=(n, g, ho, wo))
        tx = rng.choice(tx_set, size=(n, g, ho, wo))
        off[:, :, k, 0] = ty - base_y
        off[:, :, k, 1] = tx - base_x
    flat = off.reshape(-1).astype(np.float32)
    assert np.array_equal(flat.astype(np.float16).astype(np.float32), flat), "offsets must be exact in FP16"
    return flat


@pytest.mark.parametrize("shape,path", [
    (DeformConvShape.jasna_propagation(2, 64, 64), _native.DCN_PATH_SLAB_TC),
    (DeformConvShape.jasna_propagation(1, 64, 96), _native.DCN_PATH_FUSED_TC),
], ids=["slab", "global_gather"])
def test_boundary_positions_match_oracle(cuda_op, shape, path, host_threads):
    import torch

    assert cuda_op.path(shape) == path
    g = synthetic.SplitMix64(4711)
    x = synthetic.quantize_f16(g.normal(shape.input_count))
    msk = synthetic.quantize_f16(g.uniform(shape.mask_count, 0.25, 1.0))
    w, b = synthetic.weights(shape, 4712)
    w, b = synthetic.quantize_f16(w), synthetic.quantize_f16(b)
    off = _boundary_offsets(shape, 4713)
    ref = oracle.run(shape, x, off, msk, w, b, threads=host_threads)
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    out = cuda_op.forward_f16(shape, dev(x), dev(off), dev(msk), cuda_op.prepack(shape, dev(w)), dev(b))
    torch.cuda.synchronize()
    cuda_op.device_error()
    d = np.abs(out.float().cpu().numpy() - ref)
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (float(d.max()), float(d.mean()))
    # The FP32 path on the same positions is bit-identical to the oracle.
    out32 = cuda_op.run_float32(shape, x, off, msk, w, b)
    assert np.array_equal(out32, ref), "FP32 path differs from the oracle on boundary positions"
