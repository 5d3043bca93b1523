"""GPU: the operator captured in a CUDA graph.

A call is two or three kernels, the later ones launched with programmatic dependent launch
(their CTAs start while the previous kernel runs and wait in griddepcontrol.wait before any
global access).  Stream capture turns those launches into programmatic graph edges; this
checks that graph replays give exactly the eager results, for each launch chain: the slab
kernel with its group split and reduction pass (one 64x64 image), the slab kernel alone (a
batch of 64x64 tiles) and the global-gather kernel in its raw-input form (a 64x96 image).
Each graph is replayed on new inputs copied into the captured buffers."""

from __future__ import annotations

import pytest

from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu


def _capture(fn):
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()  # warm-up outside the graph (tensor-map encoder, device attributes)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


@pytest.mark.parametrize("batch,h,w,path,launches", [
    (1, 64, 64, _native.DCN_PATH_SLAB_TC, 3),
    (40, 64, 64, _native.DCN_PATH_SLAB_TC, 2),
], ids=["split_with_reduction", "slab"])
def test_graph_replay_matches_eager(cuda_op, batch, h, w, path, launches):
    import torch

    shape = DeformConvShape.jasna_propagation(batch, h, w)
    assert cuda_op.path(shape) == path and cuda_op.plan(shape)["launches"] == launches
    x, off, msk, wt, b = synthetic.device_batch(shape, 16.0, seed=501, device="cuda")
    packed = cuda_op.prepack(shape, torch.from_numpy(wt).cuda().half())
    bias = torch.from_numpy(b).cuda().half()
    ws = torch.empty(cuda_op.workspace_bytes(shape), dtype=torch.uint8, device="cuda")
    out = torch.empty(shape.output_count, dtype=torch.float16, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    graph = _capture(lambda: cuda_op.forward_f16(shape, x, off, msk, packed, bias, out=out, flag=flag,
                                                 workspace=ws))
    for seed in (502, 503, 504):
        x2, off2, msk2, _, _ = synthetic.device_batch(shape, 16.0, seed=seed, device="cuda")
        want = cuda_op.forward_f16(shape, x2, off2, msk2, packed, bias)
        x.copy_(x2)
        off.copy_(off2)
        msk.copy_(msk2)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        cuda_op.device_error()
        assert torch.equal(out, want), f"graph replay differs from the eager call (seed {seed})"
    assert int(flag.item()) == 0


def test_graph_replay_raw_form_global_gather(cuda_op):
    import torch

    shape = DeformConvShape.jasna_propagation(1, 64, 96)
    assert cuda_op.path(shape) == _native.DCN_PATH_FUSED_TC
    x, _, _, wt, b = synthetic.device_batch(shape, 16.0, seed=601, device="cuda")
    packed = cuda_op.prepack(shape, torch.from_numpy(wt).cuda().half())
    bias = torch.from_numpy(b).cuda().half()
    raw, f1, f2 = synthetic.device_raw_batch(shape, 16.0, seed=602, device="cuda")
    ws = torch.empty(cuda_op.raw_workspace_bytes(shape), dtype=torch.uint8, device="cuda")
    out = torch.empty(shape.output_count, dtype=torch.float16, device="cuda")
    graph = _capture(lambda: cuda_op.forward_f16_raw(shape, x, raw, f1, f2, packed, bias, out=out, workspace=ws))
    for seed in (603, 604):
        raw2, g1, g2 = synthetic.device_raw_batch(shape, 16.0, seed=seed, device="cuda")
        want = cuda_op.forward_f16_raw(shape, x, raw2, g1, g2, packed, bias)
        raw.copy_(raw2)
        f1.copy_(g1)
        f2.copy_(g2)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        cuda_op.device_error()
        assert torch.equal(out, want), f"graph replay differs from the eager call (seed {seed})"
