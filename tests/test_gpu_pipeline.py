"""GPU: the host-buffer pipeline (dcn_forward_f16_host through forward_f16_host: chunks of
images copied in, convolved and copied out on the library's own streams) returns exactly what
the device-resident operator returns, and large batches are deterministic run to run with no
device-side timeout recorded."""

from __future__ import annotations

import pytest

from jasnamacos_b200 import synthetic

pytestmark = pytest.mark.gpu


def _batch(cuda_op, n, seed):
    import torch

    shape = synthetic.config_shape(4, batch=n)
    x, off, msk, w, b = synthetic.device_batch(shape, 16.0, seed=seed, device="cuda")
    w16 = torch.from_numpy(w).cuda().half()
    b16 = torch.from_numpy(b).cuda().half()
    return shape, x, off, msk, cuda_op.prepack(shape, w16), b16


def test_host_pipeline_matches_device_resident(cuda_op):
    import torch

    shape, x, off, msk, packed, b16 = _batch(cuda_op, 192, seed=11)
    ref = cuda_op.forward_f16(shape, x, off, msk, packed, b16)
    torch.cuda.synchronize()
    hx, hoff, hmsk = (t.cpu().pin_memory() for t in (x, off, msk))
    hout = torch.empty(shape.output_count, dtype=torch.float16).pin_memory()
    for chunk in (64, 50, 192):
        hout.zero_()
        assert cuda_op.forward_f16_host(shape, hx, hoff, hmsk, packed, b16, hout, chunk_images=chunk) == 0
        got = hout.cuda()
        bad = int((got != ref).sum().item())
        assert bad == 0, f"chunk {chunk}: {bad} outputs differ, max {float((got.float() - ref.float()).abs().max())}"
    cuda_op.device_error()


def test_large_batch_determinism(cuda_op):
    import torch

    shape, x, off, msk, packed, b16 = _batch(cuda_op, 1024, seed=12)
    outs = [cuda_op.forward_f16(shape, x, off, msk, packed, b16) for _ in range(3)]
    torch.cuda.synchronize()
    cuda_op.device_error()
    for o in outs[1:]:
        bad = int((o != outs[0]).sum().item())
        assert bad == 0, f"{bad} outputs differ between identical runs"
