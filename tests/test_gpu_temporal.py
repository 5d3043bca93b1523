"""GPU: dcn_temporal_prepare_f16, the temporal preparation in front of the DCN
(runTemporalPreparation, MetalRunner.swift:510-582; kernels MetalShader.swift:736-813), against the
oracle's restatement (oracle.temporal_prepare, pinned in tests/test_oracle_temporal.py).

The kernel uses the reference's sampling arithmetic with one IEEE rounding per operation, so every
output must equal the oracle's bit for bit: on the reference CLI's own 3x3 case
(JasnaCLI.swift:227-316, also under its 0.004 gate), on the 64x64 frames of the reference's
temporal probe (TemporalPreparationProbe.swift:14-101: its feature formula, its repeat and
first-order-zero checks), batched, with and without the deform-input copy, and on a 270x480
frame whose flows leave the frame on every side.  The slab form (dcn_temporal_prepare_slabs_f16)
writes the deform input in the DCN's own layout, which the DCN then reads without its pre-pass.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.test_oracle_temporal import cli_inputs

pytestmark = pytest.mark.gpu


def _probe_features(plane: int, seed: int) -> np.ndarray:
    """features(seed:) of TemporalPreparationProbe.swift:23-27, FP16-rounded."""
    i = np.arange(64 * plane, dtype=np.int64)
    v = (((i * 37 + seed) % 509).astype(np.float32) / np.float32(508) - np.float32(0.5)) * np.float32(0.5)
    return v.astype(np.float16).astype(np.float32)


def _flows(plane: int, lim: float, seed: int) -> np.ndarray:
    g = np.random.default_rng(seed)
    return g.uniform(-lim, lim, 2 * plane).astype(np.float16).astype(np.float32)


def test_cli_case_bit_exact(cuda_op):
    ins = cli_inputs()
    res = cuda_op.run_temporal_preparation(3, 3, *ins, True)
    cond, di, flow2 = oracle.temporal_prepare(3, 3, *ins, True)
    assert np.array_equal(res.second_order_flow.astype(np.float32), flow2)
    assert np.array_equal(res.conditions.astype(np.float32), cond)
    assert np.array_equal(res.deform_input.astype(np.float32), di)
    got = np.concatenate([res.second_order_flow, res.conditions, res.deform_input]).astype(np.float32)
    assert np.abs(got - np.concatenate([flow2, cond, di])).max() < 0.004  # JasnaCLI.swift:296
    assert res.gpu_milliseconds >= 0.0
    # first-order run (JasnaCLI.swift:300-313): the second-order flow is exactly zero
    fp, fc, _, f1, prev = ins
    first = cuda_op.run_temporal_preparation(3, 3, fp, fc, np.zeros(64 * 9, np.float32), f1, prev, False)
    assert not np.any(first.second_order_flow)


@pytest.mark.parametrize("second_order", [True, False], ids=["second_order", "first_order"])
def test_probe_frames_batched_bit_exact(cuda_op, second_order):
    """Three 64x64 frames in one call (the probe's features, flows up to +-16 px), compared frame by
    frame with the oracle; the same call without the deform-input copy gives the same conditions
    and flow; repeated calls are identical (the probe's repeat check)."""
    import torch

    w = h = 64
    plane = w * h
    frames = 3
    ins = {k: [] for k in ("prop", "cur", "n2", "f1", "prev")}
    for f in range(frames):
        ins["prop"].append(_probe_features(plane, 17 + f))
        ins["cur"].append(_probe_features(plane, 31 + f))
        ins["n2"].append(_probe_features(plane, 47 + f) if second_order else np.zeros(64 * plane, np.float32))
        ins["f1"].append(_flows(plane, 16.0, 100 + f))
        ins["prev"].append(_flows(plane, 16.0, 200 + f))
    dev = {k: torch.from_numpy(np.concatenate(v).astype(np.float16)).cuda() for k, v in ins.items()}
    args = (w, h, dev["prop"], dev["cur"], dev["n2"], dev["f1"], dev["prev"], second_order)
    cond, di, flow2 = cuda_op.temporal_prepare(*args, batch=frames)
    cond2, none, flow2b = cuda_op.temporal_prepare(*args, batch=frames, with_deform_input=False)
    again, _, _ = cuda_op.temporal_prepare(*args, batch=frames)
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert none is None
    assert torch.equal(cond, cond2) and torch.equal(flow2, flow2b) and torch.equal(cond, again)
    cond_h, di_h, flow2_h = (t.float().cpu().numpy() for t in (cond, di, flow2))
    for f in range(frames):
        want = oracle.temporal_prepare(w, h, ins["prop"][f], ins["cur"][f], ins["n2"][f], ins["f1"][f],
                                       ins["prev"][f], second_order)
        assert np.array_equal(cond_h[f * 196 * plane:(f + 1) * 196 * plane], want[0]), f
        assert np.array_equal(di_h[f * 128 * plane:(f + 1) * 128 * plane], want[1]), f
        assert np.array_equal(flow2_h[f * 2 * plane:(f + 1) * 2 * plane], want[2]), f
    assert np.abs(cond_h).max() > 0.001                       # TemporalPreparationProbe.swift:86
    if not second_order:
        assert not np.any(flow2_h)                            # :88, the first-order flow is zero


def test_large_frame_bit_exact(cuda_op):
    """One 270x480 frame (the size of benchmark config 3) with flows up to +-40 px."""
    import torch

    w, h = 480, 270
    plane = w * h
    g = np.random.default_rng(9)
    f16 = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    prop, cur, n2 = (f16(g.standard_normal(64 * plane)) for _ in range(3))
    f1, prev = _flows(plane, 40.0, 1), _flows(plane, 40.0, 2)
    res = cuda_op.temporal_prepare(w, h, *(torch.from_numpy(a.astype(np.float16)).cuda()
                                           for a in (prop, cur, n2, f1, prev)), True)
    torch.cuda.synchronize()
    want = oracle.temporal_prepare(w, h, prop, cur, n2, f1, prev, True)
    for got, exp in zip(res, want):
        assert np.array_equal(got.float().cpu().numpy(), exp)


def test_chain_into_the_raw_form_dcn(cuda_op, host_threads):
    """The alignment step as the reference chains it (S/FusedFourPassRecurrenceProbe.swift:609-630):
    the temporal preparation's flow1/flow2 and deform input feed the raw-form DCN (offset transform
    fused).  The DCN reading the concatenated deform input and the DCN reading feat_prop and feat_n2
    as two tensors (dcn_io, no concatenation) give the same bits; both match the CPU chain
    (oracle temporal preparation -> oracle offset transform -> oracle DCN) under the FP16 gates."""
    import torch

    from jasnamacos_b200 import synthetic
    from jasnamacos_b200.deform_conv import DeformConvShape

    w = h = 64
    plane = w * h
    frames = 2
    shape = DeformConvShape.jasna_propagation(frames, h, w)
    g = np.random.default_rng(31)
    f16 = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    prop, cur, n2 = (f16(g.standard_normal(frames * 64 * plane)) for _ in range(3))
    f1, prev = _flows(frames * plane, 8.0, 3), _flows(frames * plane, 8.0, 4)
    raw = f16(g.standard_normal(frames * 432 * plane))
    wt, b = synthetic.weights(shape, 5)
    wt, b = f16(wt), f16(b)
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    prop_d, n2_d = dev(prop), dev(n2)
    cond, di, flow2 = cuda_op.temporal_prepare(w, h, prop_d, dev(cur), n2_d, dev(f1), dev(prev), True, batch=frames)
    packed = cuda_op.prepack(shape, dev(wt))
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    concat = cuda_op.forward_f16_raw(shape, di, dev(raw), dev(f1), flow2, packed, dev(b), flag=flag)
    # two tensors, per image [64][H][W] each: the DCN input split at channel 64
    split = cuda_op.forward_f16_raw(shape, prop_d, dev(raw), dev(f1), flow2, packed, dev(b), flag=flag,
                                    input_second=n2_d)
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert int(flag.item()) == 0
    assert torch.equal(concat, split)
    got = concat.float().cpu().numpy()
    for f in range(frames):
        sl = lambda a, c: a[f * c * plane:(f + 1) * c * plane]  # noqa: E731
        _, di_ref, flow2_ref = oracle.temporal_prepare(w, h, sl(prop, 64), sl(cur, 64), sl(n2, 64), sl(f1, 2),
                                                       sl(prev, 2), True)
        assert np.array_equal(flow2[f * 2 * plane:(f + 1) * 2 * plane].float().cpu().numpy(), flow2_ref)
        off, msk = oracle.prepare_offsets(plane, sl(raw, 432), sl(f1, 2), flow2_ref)
        one = shape.with_batch(1)
        ref = oracle.run(one, di_ref, f16(off), f16(msk), wt, b, threads=host_threads)
        d = np.abs(got[f * one.output_count:(f + 1) * one.output_count] - ref)
        assert d.max() <= 2e-2 and d.mean() <= 2e-3, (f, float(d.max()), float(d.mean()))


@pytest.mark.parametrize("w,h", [(44, 30), (70, 50), (300, 20), (17, 13)],
                         ids=["44x30", "70x50", "300x20_wide", "17x13_odd_plane"])
def test_irregular_frames_bit_exact(cuda_op, w, h):
    """Frame sizes whose width does not divide the staged kernel's 256-thread stride (its rows and
    columns advance by stepping, not division), one wider than 256 pixels, and an odd pixel count
    (which takes the global-memory form): three frames each, against the oracle."""
    import torch

    plane = w * h
    frames = 3
    g = np.random.default_rng(w * 1000 + h)
    f16 = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    prop, cur, n2 = (f16(g.standard_normal(frames * 64 * plane)) for _ in range(3))
    f1, prev = _flows(frames * plane, 12.0, w), _flows(frames * plane, 12.0, h)
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    cond, di, flow2 = cuda_op.temporal_prepare(w, h, dev(prop), dev(cur), dev(n2), dev(f1), dev(prev), True,
                                               batch=frames)
    torch.cuda.synchronize()
    cuda_op.device_error()
    got = [t.float().cpu().numpy() for t in (cond, di, flow2)]
    for f in range(frames):
        sl = lambda a, c: a[f * c * plane:(f + 1) * c * plane]  # noqa: E731
        want = oracle.temporal_prepare(w, h, sl(prop, 64), sl(cur, 64), sl(n2, 64), sl(f1, 2), sl(prev, 2), True)
        for a, b, c in zip(got, want, (196, 128, 2)):
            assert np.array_equal(sl(a, c), b), (w, h, f, c)


def test_verify_temporal_preparation_probe(cuda_op):
    """verify_temporal_preparation mirrors the reference's probe (TemporalPreparationProbe.swift:
    14-101): eight timed bidirectional passes that repeat exactly, conditions that are not all tiny,
    and an exactly zero second-order flow on the first-order pass; a flow with a NaN makes the
    conditions non-finite, which the probe reports as a failed command.  (A NaN position floors
    to 0, inside the frame, so no load leaves its buffer.)"""
    from jasnamacos_b200.deform_conv import CommandFailed

    plane = 64 * 64
    backward, forward = _flows(plane, 4.0, 7), _flows(plane, 4.0, 8)
    res = cuda_op.verify_temporal_preparation(backward, forward)
    assert res.iterations == 8
    assert res.repeat_maximum_error == 0.0 and res.first_order_zero_maximum_error == 0.0
    assert res.maximum_magnitude > 0.001 and np.isfinite(res.checksum)
    assert 0.0 < res.minimum_milliseconds <= res.median_milliseconds <= res.maximum_milliseconds
    bad = backward.copy()
    bad[123] = np.nan
    with pytest.raises(CommandFailed):
        cuda_op.verify_temporal_preparation(bad, forward)


@pytest.mark.parametrize("w,h,frames", [(64, 64, 1), (48, 32, 2), (46, 28, 3), (64, 64, 40)],
                         ids=["64x64x1_split4", "48x32x2_split4", "46x28x3_width_not_4k", "64x64x40"])
def test_slab_form_feeds_the_dcn_without_a_prepass(cuda_op, w, h, frames):
    """dcn_temporal_prepare_slabs_f16 writes the deform input straight into the DCN's slab layout:
    into a workspace filled with 0xA5 first, its slab bytes (zero ring included) equal what
    dcn_regroup_input_f16 makes of the NCHW deform input, its conditions and flow2 equal
    dcn_temporal_prepare_f16's (which match the oracle bit for bit), and the DCN reading those
    slabs without a pre-pass (dcn_forward_f16_raw_grouped, dcn_forward_f16_grouped) gives the
    same bits as the DCN regrouping the NCHW deform input itself.  Small batches take the
    group-split form, whose partial sums follow the slabs in the same workspace."""
    import torch

    from jasnamacos_b200 import _native, synthetic
    from jasnamacos_b200.deform_conv import DeformConvShape

    plane = w * h
    g = np.random.default_rng(w * 100 + h + frames)
    f16 = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    dev = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    prop, cur, n2 = (f16(g.standard_normal(frames * 64 * plane)) for _ in range(3))
    f1, prev = _flows(frames * plane, 12.0, w + 1), _flows(frames * plane, 12.0, h + 2)
    args = (w, h, dev(prop), dev(cur), dev(n2), dev(f1), dev(prev), True)
    shape = DeformConvShape.jasna_propagation(frames, h, w)
    assert cuda_op.path(shape) == _native.DCN_PATH_SLAB_TC
    cond, di, flow2 = cuda_op.temporal_prepare(*args, batch=frames)
    ref_ws = cuda_op.regroup_input(shape, di)
    ws = torch.full((cuda_op.workspace_bytes(shape),), 0xA5, dtype=torch.uint8, device="cuda")
    cond_s, ws_out, flow2_s = cuda_op.temporal_prepare_slabs(*args, batch=frames, workspace=ws)
    torch.cuda.synchronize()
    cuda_op.device_error()
    n = cuda_op.temporal_slabs_bytes(w, h, frames)
    assert ws_out is ws and n == frames * 16 * (h + 2) * (w + 2) * 16
    assert torch.equal(cond, cond_s) and torch.equal(flow2, flow2_s)
    assert torch.equal(ws[:n], ref_ws[:n])
    want = oracle.temporal_prepare(w, h, prop[:64 * plane], cur[:64 * plane], n2[:64 * plane], f1[:2 * plane],
                                   prev[:2 * plane], True)
    assert np.array_equal(cond_s[:196 * plane].float().cpu().numpy(), want[0])

    wt, b = synthetic.weights(shape, 7)
    packed, bias = cuda_op.prepack(shape, dev(f16(wt))), dev(f16(b))
    raw = dev(f16(g.standard_normal(frames * 432 * plane)))
    f1_d = dev(f1)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    want_raw = cuda_op.forward_f16_raw(shape, di, raw, f1_d, flow2, packed, bias, flag=flag)
    got_raw = cuda_op.forward_f16_raw_grouped(shape, ws, raw, f1_d, flow2_s, packed, bias, flag=flag)
    off = torch.empty(frames * 288 * plane, dtype=torch.float16, device="cuda")
    msk = torch.empty(frames * 144 * plane, dtype=torch.float16, device="cuda")
    for i in range(frames):
        cuda_op.prepare_offsets(plane, raw[i * 432 * plane:(i + 1) * 432 * plane], f1_d[i * 2 * plane:(i + 1) * 2 * plane],
                                flow2[i * 2 * plane:(i + 1) * 2 * plane], offset=off[i * 288 * plane:(i + 1) * 288 * plane],
                                mask=msk[i * 144 * plane:(i + 1) * 144 * plane])
    want_off = cuda_op.forward_f16(shape, di, off, msk, packed, bias, flag=flag)
    got_off = cuda_op.forward_f16_grouped(shape, ws, off, msk, packed, bias, flag=flag)
    torch.cuda.synchronize()
    cuda_op.device_error()
    assert int(flag.item()) == 0
    assert torch.equal(got_raw, want_raw)
    assert torch.equal(got_off, want_off)
    assert torch.equal(ws[:n], ref_ws[:n])  # the DCN read the slabs without changing them


def test_slab_form_rejects_frames_it_does_not_take(cuda_op):
    """Frames the slab form does not take (too large for the shared-memory kernel, an odd pixel
    count) raise Unsupported, and a workspace shorter than the slabs raises InvalidArgument."""
    import torch

    from jasnamacos_b200.deform_conv import InvalidArgument, Unsupported

    def inputs(w, h):
        plane = w * h
        z = lambda c: torch.zeros(c * plane, dtype=torch.float16, device="cuda")  # noqa: E731
        return (w, h, z(64), z(64), z(64), z(2), z(2), True)

    assert cuda_op.temporal_slabs_bytes(480, 270) == 0
    with pytest.raises(Unsupported):
        cuda_op.temporal_prepare_slabs(*inputs(480, 270), workspace=torch.empty(1 << 20, dtype=torch.uint8,
                                                                                 device="cuda"))
    with pytest.raises(Unsupported):
        cuda_op.temporal_prepare_slabs(*inputs(17, 13), workspace=torch.empty(1 << 20, dtype=torch.uint8,
                                                                               device="cuda"))
    short = torch.empty(cuda_op.temporal_slabs_bytes(64, 64) - 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(InvalidArgument):
        cuda_op.temporal_prepare_slabs(*inputs(64, 64), workspace=short)
