"""GPU: a property of every output at the benchmark's full size (config 4: 2048 FP16 tiles of
128x64x64, flow U(-16,16), the offsets, masks and weights bench.py times).

The operator is linear in its input for fixed offsets, masks and weights
(S/DeformConv.swift:98-136: each output is bias + a sum of weight x mask x bilinear(input)
terms).  Two inputs are drawn on a 1/64 grid in [-1, 1), so they and their sum are exact in FP16.
Every one of the 2048 tiles must then satisfy out(a + b) - bias = (out(a) - bias) + (out(b) - bias)
within the FP16 gates that the oracle comparisons use (max abs <= 2e-2, mean abs <= 2e-3).  A tile
whose output were corrupted would break this, wherever it sits in the batch; the oracle tests
sample 128 of the same tiles."""

from __future__ import annotations

import pytest

from jasnamacos_b200 import synthetic

pytestmark = pytest.mark.gpu

TILES = 2048


def test_config4_linearity_on_every_tile(cuda_op):
    import torch

    shape, _, x, off, msk, w, b = synthetic.bench_inputs(4, 0, 1, "cuda", TILES)
    assert shape.batch == TILES
    del x
    packed = cuda_op.prepack(shape, torch.from_numpy(w).cuda().half())
    bias = torch.from_numpy(b).cuda().half()
    g = torch.Generator(device="cuda").manual_seed(64)
    grid = lambda: (torch.randint(-64, 64, (shape.input_count,), generator=g, device="cuda",  # noqa: E731
                                  dtype=torch.int16).half() / 64)
    xa, xb = grid(), grid()
    xab = xa + xb  # exact: multiples of 1/64 in [-2, 2)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = [cuda_op.forward_f16(shape, t, off, msk, packed, bias, flag=flag) for t in (xa, xb, xab)]
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert int(flag.item()) == 0
    bias_f = bias.float().view(1, 64, 1)
    ya, yb, yab = (o.float().view(TILES, 64, -1) - bias_f for o in outs)
    d = (yab - (ya + yb)).abs()
    per_tile_max = d.amax(dim=(1, 2))
    per_tile_mean = d.mean(dim=(1, 2))
    worst = int(per_tile_max.argmax())
    assert float(per_tile_max.max()) <= 2e-2, (worst, float(per_tile_max.max()))
    assert float(per_tile_mean.max()) <= 2e-3, (int(per_tile_mean.argmax()), float(per_tile_mean.max()))
    # the property is not empty: the outputs are far from zero on every tile
    assert float(yab.abs().mean(dim=(1, 2)).min()) > 1e-2
