"""GPU: dcn_forward_f16_host, the operator on host buffers (the reference's host-array
contract, MetalDeformConv.runFloat32, Sources/JasnaMetalPoC/MetalRunner.swift:159-185).

The library cuts the batch into chunks and pipelines each chunk's copies and kernels on its
own streams.  Chunks of 32 tiles are large enough that the slab kernel does not split the
deformable groups, so their tiles must equal the device-resident dcn_forward_f16 result of
the whole batch bit for bit; the short last chunk (2 tiles, group-split) is checked against
the CPU oracle under the FP16 gates, and so is a sample of the full chunks.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu


def test_host_entry_matches_device_entry_and_oracle(cuda_op):
    import torch

    shape = DeformConvShape.jasna_propagation(98)  # chunks of 32: 32, 32, 32, 2
    x, off, msk, w, b = synthetic.device_batch(shape, 16.0, seed=77, device="cuda")
    w16 = torch.from_numpy(w).cuda().half()
    b16 = torch.from_numpy(b).cuda().half()
    packed = cuda_op.prepack(shape, w16)
    ref_dev = cuda_op.forward_f16(shape, x, off, msk, packed, b16)
    pin = lambda t: torch.empty(t.numel(), dtype=t.dtype, pin_memory=True).copy_(t)  # noqa: E731
    hx, hoff, hmsk = pin(x), pin(off), pin(msk)
    hout = torch.full((shape.output_count,), float("nan"), dtype=torch.float16, pin_memory=True)
    for _ in range(2):  # the second call reuses the library's streams and the same workspace
        flag = cuda_op.forward_f16_host(shape, hx, hoff, hmsk, packed, b16, hout, chunk_images=32)
        assert flag == 0
    per = shape.with_batch(1)
    full = 96 * per.output_count
    assert torch.equal(hout[:full], ref_dev[:full].cpu())
    tiles = [0, 31, 32, 63, 95, 96, 97]
    ref = oracle.run(per.with_batch(len(tiles)),
                     np.concatenate([x[t * per.input_count:(t + 1) * per.input_count].float().cpu().numpy()
                                     for t in tiles]),
                     np.concatenate([off[t * per.offset_count:(t + 1) * per.offset_count].float().cpu().numpy()
                                     for t in tiles]),
                     np.concatenate([msk[t * per.mask_count:(t + 1) * per.mask_count].float().cpu().numpy()
                                     for t in tiles]),
                     w16.float().cpu().numpy(), b16.float().cpu().numpy(), threads=oracle.host_threads())
    got = np.concatenate([hout[t * per.output_count:(t + 1) * per.output_count].float().numpy() for t in tiles])
    d = np.abs(got - ref)
    assert np.isfinite(d).all()
    assert float(d.max()) <= 2e-2 and float(d.mean()) <= 2e-3, (float(d.max()), float(d.mean()))


def test_host_entry_reports_nonfinite_output(cuda_op):
    import torch

    from jasnamacos_b200.deform_conv import NonFiniteOutput

    shape = DeformConvShape.jasna_propagation(3)
    x, off, msk, w, _ = synthetic.device_batch(shape, 16.0, seed=78, device="cuda")
    packed = cuda_op.prepack(shape, torch.from_numpy(w).cuda().half())
    inf_bias = torch.full((64,), float("inf"), dtype=torch.float16, device="cuda")
    pin = lambda t: torch.empty(t.numel(), dtype=t.dtype, pin_memory=True).copy_(t)  # noqa: E731
    hout = torch.empty(shape.output_count, dtype=torch.float16, pin_memory=True)
    with pytest.raises(NonFiniteOutput):
        cuda_op.forward_f16_host(shape, pin(x), pin(off), pin(msk), packed, inf_bias, hout, chunk_images=2)
    assert cuda_op.forward_f16_host(shape, pin(x), pin(off), pin(msk), packed, inf_bias, hout, chunk_images=2,
                                    check=False) & 1
