"""GPU: the slab kernel's deformable-group split for batches with fewer 128-pixel tiles than
the B200 has SMs (one 64x64 image: 32 tiles, 16 groups split 4 ways; two images: 2 ways; the
2x16x24 smoke shape: 6 tiles, 16 ways), with its fixed-order reduction pass.

Each split batch is checked against the CPU oracle (FP16 gates), against the same images
computed inside a batch large enough not to split (the two differ only in the FP32 summation
order, so by at most one FP16 rounding step), for run-to-run identity, and with the output
written into a channel slot (the reduction pass writes the output and the flag)."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu

F16_MAX_ABS = 2e-2
F16_MEAN_ABS = 2e-3


def _slab_bytes(shape):
    return shape.batch * shape.offset_groups * (shape.input_height + 2) * (shape.input_width + 2) * 16


@pytest.mark.parametrize("n,h,w,splits", [(1, 64, 64, 4), (2, 64, 64, 2), (2, 16, 24, 16)],
                         ids=["1x64x64", "2x64x64", "2x16x24"])
def test_split_batch_matches_oracle_and_unsplit_batch(cuda_op, n, h, w, splits, host_threads):
    import torch

    big = DeformConvShape.jasna_propagation(8 if h == 64 else 32, h, w)  # fills the GPU: no split
    shape = big.with_batch(n)
    lib = _native.load()
    assert cuda_op.path(shape) == _native.DCN_PATH_SLAB_TC
    plane = h * w
    extra = cuda_op.workspace_bytes(shape) - _slab_bytes(shape)
    assert extra == splits * n * 64 * plane * 4, "the workspace must hold the FP32 partial sums"
    assert cuda_op.workspace_bytes(big) == _slab_bytes(big), "the large batch must not split"
    del lib

    inputs = synthetic.generate(2, tiles=range(big.batch), batch=big.batch) if h == 64 else None
    if inputs is None:
        g = synthetic.SplitMix64(1234)
        arrays = [synthetic.quantize_f16(a) for a in (
            g.normal(big.input_count), g.uniform(big.offset_count, -6, 6), g.uniform(big.mask_count, 0, 1))]
        w_, b_ = synthetic.weights(big, 99)
        x, off, msk, wt, bias = arrays + [synthetic.quantize_f16(w_), synthetic.quantize_f16(b_)]
    else:
        x, off, msk, wt, bias = inputs.input, inputs.offset, inputs.mask, inputs.weight, inputs.bias
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).astype(np.float16)).cuda()  # noqa: E731
    packed = cuda_op.prepack(big, dev(wt))
    bd = dev(bias)
    full = cuda_op.forward_f16(big, dev(x), dev(off), dev(msk), packed, bd)

    xs = x[:shape.input_count]
    offs = off[:shape.offset_count]
    msks = msk[:shape.mask_count]
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    split1 = cuda_op.forward_f16(shape, dev(xs), dev(offs), dev(msks), packed, bd, flag=flag)
    split2 = cuda_op.forward_f16(shape, dev(xs), dev(offs), dev(msks), packed, bd)
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert int(flag.item()) == 0
    assert torch.equal(split1, split2), "split results must be identical run to run"

    ref = oracle.run(shape, xs, offs, msks, wt, bias, threads=host_threads)
    d = np.abs(split1.float().cpu().numpy() - ref)
    assert d.max() <= F16_MAX_ABS and d.mean() <= F16_MEAN_ABS, (float(d.max()), float(d.mean()))
    # Against the unsplit batch: FP32 partial sums in another order, then one FP16 rounding.
    e = (split1.float() - full[:shape.output_count].float()).abs()
    assert float(e.max()) <= 2e-3, float(e.max())
    assert float((e > 0).float().mean()) < 0.05


def test_split_batch_into_output_slot_and_raw_form(cuda_op):
    import torch

    shape = DeformConvShape.jasna_propagation(1, 64, 64)
    plane = 64 * 64
    g = synthetic.SplitMix64(4321)
    x = synthetic.quantize_f16(g.normal(shape.input_count))
    raw = synthetic.quantize_f16(g.normal(432 * plane))
    f1 = synthetic.quantize_f16(g.uniform(2 * plane, -16, 16))
    f2 = synthetic.quantize_f16(g.uniform(2 * plane, -16, 16))
    w_, b_ = synthetic.weights(shape, 5)
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    packed = cuda_op.prepack(shape, dev(synthetic.quantize_f16(w_)))
    bd = dev(synthetic.quantize_f16(b_))
    xd = dev(x)
    plain = cuda_op.forward_f16_raw(shape, xd, dev(raw), dev(f1), dev(f2), packed, bd)
    slot = torch.full((1, 192, plane), float("inf"), dtype=torch.float16, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    first, second = xd[:64 * plane].contiguous(), xd[64 * plane:].contiguous()
    cuda_op.forward_f16_raw(shape, first, dev(raw), dev(f1), dev(f2), packed, bd, out=slot.view(-1), flag=flag,
                            input_second=second, out_image_channels=192, out_channel_offset=128)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0, "the flag must only look at the written slot"
    assert torch.equal(slot[0, 128:].reshape(-1), plain)
    assert bool(torch.isinf(slot[0, :128]).all())
    # The raw form against the two-step chain on the same split shape.
    o = torch.empty(288 * plane, dtype=torch.float16, device="cuda")
    m = torch.empty(144 * plane, dtype=torch.float16, device="cuda")
    cuda_op.prepare_offsets(plane, dev(raw), dev(f1), dev(f2), offset=o, mask=m)
    two = cuda_op.forward_f16(shape, xd, o, m, packed, bd)
    d = (two.float() - plain.float()).abs()
    assert float(d.max()) <= F16_MAX_ABS and float(d.mean()) <= F16_MEAN_ABS


_NO_SPLIT_CHILD = """
import numpy as np, torch
from jasnamacos_b200 import synthetic
from jasnamacos_b200.deform_conv import CudaDeformConv, DeformConvShape
op = CudaDeformConv(0)
big = DeformConvShape.jasna_propagation(6)
one = big.with_batch(1)
x, off, msk, w, b = synthetic.device_batch(big, 16.0, seed=11, device="cuda")
packed = op.prepack(big, torch.from_numpy(w).cuda().half())
b16 = torch.from_numpy(b).cuda().half()
assert op.workspace_bytes(one) == 16 * 66 * 66 * 16
full = op.forward_f16(big, x, off, msk, packed, b16)
t = 3
alone = op.forward_f16(one, x[t * one.input_count:(t + 1) * one.input_count],
                       off[t * one.offset_count:(t + 1) * one.offset_count],
                       msk[t * one.mask_count:(t + 1) * one.mask_count], packed, b16)
torch.cuda.synchronize()
assert torch.equal(alone, full[t * one.output_count:(t + 1) * one.output_count])
print("bit-identical")
"""


def test_split_off_makes_images_batch_independent():
    """With DCN_B200_GROUP_SPLIT=0 (a child process: the switch is read once) an image run
    alone equals the same image inside a larger batch bit for bit."""
    repo = Path(__file__).resolve().parents[1]
    env = dict(os.environ, DCN_B200_GROUP_SPLIT="0", PYTHONPATH=str(repo))
    r = subprocess.run([sys.executable, "-c", _NO_SPLIT_CHILD], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "bit-identical" in r.stdout
