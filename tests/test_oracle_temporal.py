"""CPU: the oracle's restatement of runTemporalPreparation (MetalRunner.swift:510-582:
accumulate_second_order_flow_fp16 + assemble_temporal_alignment_fp16, MetalShader.swift:736-813).

Pinned three ways:
* the reference's own self-check (JasnaCLI.swift:227-316): its 3x3 frame built from the same
  integer formulas, its expectations recomputed here in numpy float32 in the order the Swift code
  writes them (`sampleZero`, :213-225), compared bit for bit, under its 0.004 gate as well; and
  its first-order run, whose second-order flow must be exactly zero (:300-313);
* PyTorch's grid_sample (bilinear, zero padding, align_corners=True), which the reference kernel
  says it follows (MetalShader.swift:736-738), as an independent implementation of the warps;
* the deform input, which must be [feat_prop, feat_n2] unchanged.
"""

from __future__ import annotations

import numpy as np

import oracle


def cli_inputs(plane: int = 9):
    """The reference CLI's temporal inputs (JasnaCLI.swift:228-242), FP16-rounded."""
    f16 = lambda a: np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)  # noqa: E731
    i64 = np.arange(64 * plane, dtype=np.int64)
    i2 = np.arange(2 * plane, dtype=np.int64)
    feat_prop = f16(((i64 * 11) % 71).astype(np.float32) / np.float32(50) - np.float32(0.7))
    feat_current = f16(((i64 * 17) % 83).astype(np.float32) / np.float32(60) - np.float32(0.6))
    feat_n2 = f16(((i64 * 23) % 97).astype(np.float32) / np.float32(70) - np.float32(0.65))
    flow1 = f16(((i2 * 7) % 19).astype(np.float32) / np.float32(20) - np.float32(0.4))
    previous = f16(((i2 * 5) % 17).astype(np.float32) / np.float32(25) - np.float32(0.3))
    return feat_prop, feat_current, feat_n2, flow1, previous


def _sample_zero(values, base, h, w, y, x):
    """sampleZero of JasnaCLI.swift:213-225 in float32, operation by operation."""
    y, x = np.float32(y), np.float32(x)
    y0, x0 = int(np.floor(y)), int(np.floor(x))
    ly, lx = np.float32(y - np.float32(y0)), np.float32(x - np.float32(x0))

    def v(yy, xx):
        return values[base + yy * w + xx] if 0 <= yy < h and 0 <= xx < w else np.float32(0)

    one = np.float32(1)
    t0 = np.float32(np.float32(v(y0, x0) * (one - ly)) * (one - lx))
    t1 = np.float32(np.float32(v(y0, x0 + 1) * (one - ly)) * lx)
    t2 = np.float32(np.float32(v(y0 + 1, x0) * ly) * (one - lx))
    t3 = np.float32(np.float32(v(y0 + 1, x0 + 1) * ly) * lx)
    return np.float32(np.float32(np.float32(t0 + t1) + t2) + t3)


def cli_expectations(w, h, feat_prop, feat_current, feat_n2, flow1, previous):
    """The expectations of JasnaCLI.swift:248-290, restated."""
    plane = w * h
    h16 = lambda v: np.float32(np.float16(v))  # noqa: E731
    flow2 = np.zeros(2 * plane, dtype=np.float32)
    for c in range(2):
        for s in range(plane):
            y, x = s // w, s % w
            warped = _sample_zero(previous, c * plane, h, w, np.float32(y) + flow1[plane + s], np.float32(x) + flow1[s])
            flow2[c * plane + s] = h16(np.float32(flow1[c * plane + s] + warped))
    cond = np.zeros(196 * plane, dtype=np.float32)
    for c in range(196):
        for s in range(plane):
            y, x = s // w, s % w
            if c < 64:
                v = _sample_zero(feat_prop, c * plane, h, w, np.float32(y) + flow1[plane + s], np.float32(x) + flow1[s])
            elif c < 128:
                v = feat_current[(c - 64) * plane + s]
            elif c < 192:
                v = _sample_zero(feat_n2, (c - 128) * plane, h, w, np.float32(y) + flow2[plane + s],
                                 np.float32(x) + flow2[s])
            elif c < 194:
                v = flow1[(c - 192) * plane + s]
            else:
                v = flow2[(c - 194) * plane + s]
            cond[c * plane + s] = h16(v)
    return cond, np.concatenate([feat_prop, feat_n2]), flow2


def test_cli_selfcheck_case_bit_exact():
    ins = cli_inputs()
    cond, di, flow2 = oracle.temporal_prepare(3, 3, *ins, True)
    e_cond, e_di, e_flow2 = cli_expectations(3, 3, *ins)
    assert np.array_equal(flow2, e_flow2)
    assert np.array_equal(cond, e_cond)
    assert np.array_equal(di, e_di)
    # the reference's own gate on the same case (JasnaCLI.swift:292-299)
    err = np.abs(np.concatenate([flow2, cond, di]) - np.concatenate([e_flow2, e_cond, e_di])).max()
    assert err < 0.004
    assert np.abs(flow2).max() > 0.05 and np.abs(cond).max() > 0.5  # the case is not trivial


def test_first_order_flow_is_exactly_zero():
    feat_prop, feat_current, _, flow1, previous = cli_inputs()
    zeros = np.zeros(64 * 9, dtype=np.float32)
    cond, di, flow2 = oracle.temporal_prepare(3, 3, feat_prop, feat_current, zeros, flow1, previous, False)
    assert np.array_equal(flow2, np.zeros(18, dtype=np.float32))  # JasnaCLI.swift:300-313
    assert np.array_equal(cond[128 * 9:192 * 9], zeros)            # warp of zeros by a zero flow
    assert np.array_equal(cond[194 * 9:], np.zeros(18, dtype=np.float32))


def test_warps_match_torch_grid_sample():
    """The two feature warps and the flow warp equal grid_sample(bilinear, zeros,
    align_corners=True) up to FP32 rounding order, on a 13x17 frame with flows that leave the
    frame on every side."""
    import torch
    import torch.nn.functional as F

    w, h = 17, 13
    plane = w * h
    rng = np.random.default_rng(5)
    f16 = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    feat_prop = f16(rng.standard_normal(64 * plane))
    feat_current = f16(rng.standard_normal(64 * plane))
    feat_n2 = f16(rng.standard_normal(64 * plane))
    flow1 = f16(rng.uniform(-6, 6, 2 * plane))
    previous = f16(rng.uniform(-3, 3, 2 * plane))
    cond, di, flow2 = oracle.temporal_prepare(w, h, feat_prop, feat_current, feat_n2, flow1, previous, True)

    def warp(img, flow):  # img [C][h][w], flow [2][h][w] in (x, y) pixels
        ys, xs = np.meshgrid(np.arange(h, dtype=np.float64), np.arange(w, dtype=np.float64), indexing="ij")
        gx = (xs + flow[0]) * 2 / (w - 1) - 1
        gy = (ys + flow[1]) * 2 / (h - 1) - 1
        grid = torch.from_numpy(np.stack([gx, gy], -1)[None])
        out = F.grid_sample(torch.from_numpy(img.astype(np.float64))[None], grid, mode="bilinear",
                            padding_mode="zeros", align_corners=True)
        return out[0].numpy()

    f1 = flow1.reshape(2, h, w).astype(np.float64)
    f2 = flow2.reshape(2, h, w).astype(np.float64)
    want_flow2 = flow1.reshape(2, h, w) + warp(previous.reshape(2, h, w), f1)
    assert np.abs(flow2.reshape(2, h, w) - want_flow2).max() <= 4e-3  # one FP16 rounding of values < 9
    want_prop = warp(feat_prop.reshape(64, h, w), f1)
    want_n2 = warp(feat_n2.reshape(64, h, w), f2)
    c = cond.reshape(196, h, w)
    assert np.abs(c[:64] - want_prop).max() <= 4e-3
    assert np.abs(c[128:192] - want_n2).max() <= 4e-3
    assert np.array_equal(c[64:128], feat_current.reshape(64, h, w))
    assert np.array_equal(c[192:194], flow1.reshape(2, h, w))
    assert np.array_equal(c[194:], flow2.reshape(2, h, w))
    assert np.array_equal(di, np.concatenate([feat_prop, feat_n2]))
