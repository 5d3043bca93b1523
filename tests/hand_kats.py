"""Known answers derived by hand from the reference's DCNv2 definition, independent of the oracle.

`DeformConvCPU.run` (Sources/JasnaMetalPoC/DeformConv.swift:75-138) computes
    out[n, oc, oy, ox] = bias[oc] + sum_{ic, ky, kx} bilinear(in[n, ic], y, x) * mask * w[oc, ic, ky, kx]
with y = oy*sh - ph + ky*dh + offset[n, 2*(g*KA + k)], x = ... + offset[n, 2*(g*KA + k) + 1],
g = ic / (C / offsetGroups), mask = mask[n, g*KA + k], and `bilinear` (:146-165) taking
floor(y), floor(x), the fractions ly, lx and the four corners, each corner outside the image
contributing zero.  The reference's own test (Tests/JasnaMetalPoCTests/DeformConvCPUTests.swift:4-33)
checks only a 1x1 kernel with zero offsets.  The cases below add what it leaves out -- fractional
positions, corners outside the image on every side, positions in (-1, 0), two offset groups with
their own offsets and masks, stride, padding -- with every value a short dyadic fraction, so each
expected output is exact in binary32 and was worked out by hand (the arithmetic is in each case's
`why`).  They pin the oracle (tests/test_oracle_hand_kats.py) and the GPU paths
(tests/test_gpu_hand_kats.py) to the definition itself, not to each other.
"""

from __future__ import annotations

import numpy as np

from jasnamacos_b200.deform_conv import DeformConvShape


def _shape(n, c, h, w, oc, ho, wo, kh, kw, ph, pw, sh, sw, dh, dw, g, og):
    return DeformConvShape(n, c, h, w, oc, ho, wo, kh, kw, ph, pw, sh, sw, dh, dw, g, og)


def cases():
    out = []

    # 1. Fractional position inside the image.  in = [[1, 2], [4, 8]], 1x1 kernel, every pixel
    #    offset by (dy, dx) = (0.5, 0.25), mask 1, weight 1, bias 0.
    #    (0,0): y=0.5, x=0.25: 0.5*0.75*1 + 0.5*0.25*2 + 0.5*0.75*4 + 0.5*0.25*8 = 0.375+0.25+1.5+1 = 3.125
    #    (0,1): x=1.25: corners (0,1)=2, (0,2)=0, (1,1)=8, (1,2)=0 -> 0.5*0.75*2 + 0.5*0.75*8 = 0.75+3 = 3.75
    #    (1,0): y=1.5: rows 1 and 2 (2 is outside) -> 0.5*0.75*4 + 0.5*0.25*8 = 1.5+1 = 2.5
    #    (1,1): y=1.5, x=1.25: only corner (1,1)=8 inside -> 0.5*0.75*8 = 3
    s = _shape(1, 1, 2, 2, 1, 2, 2, 1, 1, 0, 0, 1, 1, 1, 1, 1, 1)
    off = np.array([0.5] * 4 + [0.25] * 4, np.float32)  # channel 0 = dy plane, channel 1 = dx plane
    out.append(dict(name="fractional_inside", shape=s, input=np.array([1, 2, 4, 8], np.float32), offset=off,
                    mask=np.ones(4, np.float32), weight=np.ones(1, np.float32), bias=np.zeros(1, np.float32),
                    expected=np.array([3.125, 3.75, 2.5, 3.0], np.float32), why="see comment 1"))

    # 2. Positions in (-1, 0): floor gives -1, the row/column -1 corners are zero.
    #    Same input, offsets (dy, dx) = (-0.25, -0.5) everywhere, mask 0.5, weight 2, bias 1.
    #    mask*weight = 1 per sample, then + bias.
    #    (0,0): y=-0.25 -> y0=-1 (ly=0.75), x=-0.5 -> x0=-1 (lx=0.5): only corner (0,0)=1 inside, with
    #           weight ly*lx = 0.375 -> 0.375 + 1 = 1.375
    #    (0,1): y0=-1 (ly=0.75), x=0.5 -> x0=0 (lx=0.5): corners (0,0)=1, (0,1)=2 with 0.75*0.5 each
    #           -> 0.375*3 + 1 = 2.125
    #    (1,0): y=0.75 -> y0=0 (ly=0.75), x0=-1 (lx=0.5): corners (0,0)=1 w 0.25*0.5, (1,0)=4 w 0.75*0.5
    #           -> 0.125 + 1.5 + 1 = 2.625
    #    (1,1): y0=0 (0.75), x0=0 (0.5): 0.125*1 + 0.125*2 + 0.375*4 + 0.375*8 = 0.125+0.25+1.5+3 = 4.875
    #           + 1 = 5.875
    off = np.array([-0.25] * 4 + [-0.5] * 4, np.float32)
    out.append(dict(name="negative_fractions", shape=s, input=np.array([1, 2, 4, 8], np.float32), offset=off,
                    mask=np.full(4, 0.5, np.float32), weight=np.full(1, 2.0, np.float32),
                    bias=np.ones(1, np.float32),
                    expected=np.array([1.375, 2.125, 2.625, 5.875], np.float32), why="see comment 2"))

    # 3. Two offset groups (one channel each), each with its own offset and mask; 1x1 kernel, one
    #    output channel with weights (1, 2), bias 0.  Image 1x2 (H=1, W=2).
    #    channel 0 = [1, 3] (group 0): dx = +0.5 everywhere, mask 1
    #    channel 1 = [5, 7] (group 1): dx = -1 everywhere (whole-pixel shift left), mask 0.25
    #    px 0: g0 x=0.5 -> 0.5*1 + 0.5*3 = 2;  g1 x=-1 -> corner x0=-1 outside, x1=0 with lx=0 -> 0
    #          -> 2*1 + 0*0.25*2 = 2
    #    px 1: g0 x=1.5 -> 0.5*3 + 0 = 1.5;  g1 x=0 -> 5 -> 1.5 + 5*0.25*2 = 4
    #    offset layout [2*g*KA + 2*k (+1)] per group: g0 dy, g0 dx, g1 dy, g1 dx planes.
    s3 = _shape(1, 2, 1, 2, 1, 1, 2, 1, 1, 0, 0, 1, 1, 1, 1, 1, 2)
    off3 = np.array([0, 0, 0.5, 0.5, 0, 0, -1, -1], np.float32)
    msk3 = np.array([1, 1, 0.25, 0.25], np.float32)
    out.append(dict(name="two_offset_groups", shape=s3, input=np.array([1, 3, 5, 7], np.float32), offset=off3,
                    mask=msk3, weight=np.array([1, 2], np.float32), bias=np.zeros(1, np.float32),
                    expected=np.array([2.0, 4.0], np.float32), why="see comment 3"))

    # 4. 3x3 kernel, pad 1, stride 2 on a 3x3 image of ones, zero offsets except tap (1,1) which
    #    moves by (dy, dx) = (0.5, 0.5); weights 1, mask 1, bias 0.  Output 2x2 (Ho = (3+2-3)/2+1).
    #    out(oy,ox) samples rows 2*oy-1+ky, cols 2*ox-1+kx.  With zero offsets each in-image tap
    #    gives 1.  Output (0,0): taps at rows -1..1, cols -1..1: 4 in-image taps (rows 0..1 x cols
    #    0..1), but the centre tap (0,0) moves to (0.5, 0.5): corners (0,0),(0,1),(1,0),(1,1) all
    #    inside, each 0.25 -> 1, so the sum stays 4.
    #    Output (1,1): rows 1..3, cols 1..3: in-image taps rows 1..2 x cols 1..2 = 4; centre tap
    #    (2,2) moves to (2.5, 2.5): only corner (2,2) inside, weight 0.25 -> 4 - 1 + 0.25 = 3.25.
    #    Output (0,1): rows -1..1, cols 1..3: in-image rows 0..1 x cols 1..2 = 4 taps; centre (0,2)
    #    -> (0.5, 2.5): corners (0,2) and (1,2) inside, 0.25 each -> 4 - 1 + 0.5 = 3.5.  By symmetry
    #    (1,0) = 3.5.
    s4 = _shape(1, 1, 3, 3, 1, 2, 2, 3, 3, 1, 1, 2, 2, 1, 1, 1, 1)
    off4 = np.zeros(2 * 9 * 4, np.float32)
    centre = 4  # tap k = ky*3 + kx = 4
    off4[(2 * centre) * 4:(2 * centre + 1) * 4] = 0.5      # dy plane of tap 4
    off4[(2 * centre + 1) * 4:(2 * centre + 2) * 4] = 0.5  # dx plane of tap 4
    out.append(dict(name="stride2_pad1_centre_tap", shape=s4, input=np.ones(9, np.float32), offset=off4,
                    mask=np.ones(9 * 4, np.float32), weight=np.ones(9, np.float32), bias=np.zeros(1, np.float32),
                    expected=np.array([4.0, 3.5, 3.5, 3.25], np.float32), why="see comment 4"))
    return out
