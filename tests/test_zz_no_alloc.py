"""GPU: dcn_forward_f16_static_scratch, the entry point for callers that cannot allocate
device memory when they run the convolution (its scratch lives in a fixed 16 MiB array
inside the library), called through the C ABI and compared with dcn_forward_f16 given a
caller workspace, on two calls in a row with different inputs.  Both entry points run the
same kernels on the same inputs in the same order, so the outputs must be identical bit for
bit; the first call's output is also checked against the CPU oracle, the device's free
memory must not change across the second call, and the sticky device error word must stay
clear.  Collected last on purpose (file name), and self-contained, so it passes alone in a
fresh process or after the rest."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu

F16_MAX_ABS = 2e-2
F16_MEAN_ABS = 2e-3


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("batch", [4, 1], ids=["4_tiles", "1_tile_group_split"])
def test_static_scratch_matches_workspace_entry_point_twice(batch):
    """Four 64x64 tiles (slabs only) and one tile, whose 16 deformable groups are split across
    SMs with their FP32 partial sums kept in the static scratch too."""
    import torch

    import oracle

    assert torch.cuda.is_available()
    lib = _native.load()
    shape = DeformConvShape.jasna_propagation(batch=batch)
    c_shape = shape.to_c()
    assert lib.dcn_static_scratch_bytes() == 16 << 20
    w, b = synthetic.weights(shape, 21)
    w16 = torch.from_numpy(w).cuda().half()
    b16 = torch.from_numpy(b).cuda().half()
    packed = torch.empty(lib.dcn_packed_weight_bytes(ctypes.byref(c_shape)), dtype=torch.uint8, device="cuda")
    assert lib.dcn_prepack_weights(ctypes.byref(c_shape), _p(w16), _native.DCN_DTYPE_F16, _native.DCN_WEIGHT_OIHW,
                                   _p(packed), None) == _native.DCN_OK
    ws_bytes = lib.dcn_forward_f16_workspace_bytes(ctypes.byref(c_shape))
    assert ws_bytes <= lib.dcn_static_scratch_bytes()
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")

    # Everything both calls need is allocated before the first call, so that the free-memory
    # reading around the second call sees only what the entry point itself might allocate.
    calls = []
    for seed in (31, 32):  # two calls in a row, different inputs
        x, off, msk, _, _ = synthetic.device_batch(shape, 16.0, seed=seed, device="cuda")
        calls.append(dict(x=x, off=off, msk=msk,
                          ref=torch.empty(shape.output_count, dtype=torch.float16, device="cuda"),
                          out=torch.full((shape.output_count,), float("nan"), dtype=torch.float16, device="cuda"),
                          flag=torch.zeros(1, dtype=torch.int32, device="cuda")))
    torch.cuda.synchronize()
    for call, c in enumerate(calls):
        st = lib.dcn_forward_f16(ctypes.byref(c_shape), _p(c["x"]), _p(c["off"]), _p(c["msk"]), _p(packed),
                                 _p(b16), _p(c["ref"]), None, _p(ws), ws_bytes, None)
        assert st == _native.DCN_OK
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = lib.dcn_forward_f16_static_scratch(ctypes.byref(c_shape), _p(c["x"]), _p(c["off"]), _p(c["msk"]),
                                                _p(packed), _p(b16), _p(c["out"]), _p(c["flag"]), None)
        assert st == _native.DCN_OK, _native.status_string(st)
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        if call == 1:  # the first call on a device may load the library's module (the array itself)
            assert free_after == free_before, (free_before, free_after)
        assert int(c["flag"].item()) == 0
        assert torch.equal(c["out"], c["ref"]), f"call {call}: static-scratch output differs from dcn_forward_f16"
    assert lib.dcn_device_error() == _native.DCN_OK

    # One oracle check (first call): the shared output is also right, not just repeatable.
    c = calls[0]
    ref = oracle.run(shape, c["x"].float().cpu().numpy(), c["off"].float().cpu().numpy(),
                     c["msk"].float().cpu().numpy(), w16.float().cpu().numpy(), b16.float().cpu().numpy(),
                     threads=oracle.host_threads())
    d = np.abs(c["out"].float().cpu().numpy() - ref)
    assert np.isfinite(d).all()
    assert float(d.max()) <= F16_MAX_ABS and float(d.mean()) <= F16_MEAN_ABS, (float(d.max()), float(d.mean()))


def test_static_scratch_rejects_problems_beyond_its_size():
    lib = _native.load()
    big = DeformConvShape.jasna_propagation(batch=20)  # 20 tiles need more than 16 MiB on either path
    c_big = big.to_c()
    assert lib.dcn_forward_f16_workspace_bytes(ctypes.byref(c_big)) > lib.dcn_static_scratch_bytes()
    p = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    st = lib.dcn_forward_f16_static_scratch(ctypes.byref(c_big), p, p, p, p, p, p, None, None)
    assert st == _native.DCN_ERR_SCRATCH_TOO_SMALL
    assert b"static scratch" in lib.dcn_status_string(st)
