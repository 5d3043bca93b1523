"""CPU oracle checks: pinned to the reference's known answers, then cross-checked.

The oracle is the checker for every GPU parity test, so it is validated first:
  * the reference's own DCNv2 known-answer test (DeformConvCPUTests.swift:4-33),
  * the committed golden fixtures (made with the literal oracle, torchvision-checked),
  * the memoised form is bit-identical to the literal loop,
  * torchvision.ops.deform_conv2d agrees on random shapes (secondary reference),
  * SplitMix64 reproduces SeededGenerator's constants (DeformConv.swift:168-181),
  * the offset transform matches the reference CLI's own check (JasnaCLI.swift:177-211).
"""

from __future__ import annotations

import math

import numpy as np
import pytest

import oracle
from golden_data import golden_cases, reference_kats
from jasnamacos_b200 import synthetic
from jasnamacos_b200.deform_conv import DeformConvShape


def test_reference_kat_one_by_one_convolution():
    kat = reference_kats()["deform_conv_1x1"]
    shape = DeformConvShape(*kat["shape"])
    out = oracle.run(shape, kat["input"], kat["offset"], kat["mask"], kat["weight"], kat["bias"], fast=False)
    assert out.tolist() == kat["expected"]  # exact, as `#expect(output == [2, 3, 4, 5])`


@pytest.mark.parametrize("case", list(golden_cases()), ids=lambda c: c[0])
def test_golden_fixtures_literal_and_fast(case):
    name, shape, x, off, msk, w, b, expected = case
    literal = oracle.run(shape, x, off, msk, w, b, fast=False)
    fast = oracle.run(shape, x, off, msk, w, b, fast=True)
    assert np.array_equal(literal.view(np.uint32), expected.view(np.uint32)), name
    assert np.array_equal(fast.view(np.uint32), expected.view(np.uint32)), name


def test_far_offsets_give_bias():
    for name, shape, x, off, msk, w, b, expected in golden_cases():
        if name == "far_offsets":
            per = shape.output_height * shape.output_width
            assert np.array_equal(expected.reshape(shape.output_channels, per),
                                  np.repeat(b[:, None], per, axis=1))


def _random_shape(rng: np.random.Generator) -> DeformConvShape:
    groups = int(rng.choice([1, 2]))
    og = int(rng.choice([1, 2, 4]))
    cin = int(np.lcm(groups, og) * rng.integers(1, 3))
    cout = groups * int(rng.integers(1, 4))
    kh, kw = int(rng.integers(1, 4)), int(rng.integers(1, 4))
    ph, pw = int(rng.integers(0, 3)), int(rng.integers(0, 3))
    sh, sw = int(rng.integers(1, 3)), int(rng.integers(1, 3))
    dh, dw = int(rng.integers(1, 3)), int(rng.integers(1, 3))
    h, w = int(rng.integers(3, 10)), int(rng.integers(3, 10))
    ho = max(1, (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1)
    wo = max(1, (w + 2 * pw - dw * (kw - 1) - 1) // sw + 1)
    return DeformConvShape(int(rng.integers(1, 3)), cin, h, w, cout, ho, wo, kh, kw, ph, pw, sh, sw, dh, dw,
                           groups, og)


def test_fast_equals_literal_random_shapes():
    rng = np.random.default_rng(1234)
    for i in range(25):
        shape = _random_shape(rng)
        gen = synthetic.SplitMix64(100 + i)
        arrays = [gen.uniform(n, -1, 1) for n in (shape.input_count,)] + [
            gen.uniform(shape.offset_count, -3, 3), gen.uniform(shape.mask_count, 0, 1),
            gen.uniform(shape.weight_count, -0.5, 0.5), gen.uniform(shape.output_channels, -0.1, 0.1)]
        a = oracle.run(shape, *arrays, fast=False)
        b = oracle.run(shape, *arrays, fast=True, threads=2)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), shape


def test_torchvision_cross_check_random_shapes():
    torch = pytest.importorskip("torch")
    torchvision = pytest.importorskip("torchvision")
    rng = np.random.default_rng(99)
    for i in range(10):
        s = _random_shape(rng)
        gen = synthetic.SplitMix64(500 + i)
        x = gen.uniform(s.input_count, -1, 1)
        off = gen.uniform(s.offset_count, -4, 4)
        msk = gen.uniform(s.mask_count, 0, 1)
        w = gen.uniform(s.weight_count, -0.5, 0.5)
        b = gen.uniform(s.output_channels, -0.1, 0.1)
        ours = oracle.run(s, x, off, msk, w, b)
        tv = torchvision.ops.deform_conv2d(
            torch.from_numpy(x).view(s.batch, s.input_channels, s.input_height, s.input_width),
            torch.from_numpy(off).view(s.batch, -1, s.output_height, s.output_width),
            torch.from_numpy(w).view(s.output_channels, s.input_channels // s.groups, s.kernel_height,
                                     s.kernel_width),
            torch.from_numpy(b), stride=(s.stride_height, s.stride_width), padding=(s.pad_height, s.pad_width),
            dilation=(s.dilation_height, s.dilation_width),
            mask=torch.from_numpy(msk).view(s.batch, -1, s.output_height, s.output_width)).numpy().reshape(-1)
        assert np.abs(ours - tv).max() <= 1e-5, s


def test_validate_matches_reference_rules():
    good = DeformConvShape.jasna_propagation()
    assert oracle.validate(good) and good.validate_reference()
    bad = [
        good.with_batch(0),
        DeformConvShape(1, 128, 64, 64, 64, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 3, 16),  # 128 % 3
        DeformConvShape(1, 128, 64, 64, 64, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 3),   # 128 % 3 offset groups
        DeformConvShape(1, 128, 64, 64, 65, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 2, 16),  # 65 % 2
        DeformConvShape(1, 128, 64, 64, 64, 64, 64, 0, 3, 1, 1, 1, 1, 1, 1, 1, 16),
    ]
    for s in bad:
        assert not oracle.validate(s) and not s.validate_reference()


def test_splitmix64_matches_seeded_generator_constants():
    # Independent restatement in Python integers (DeformConv.swift:175-181).
    def ref(seed, count):
        state = 0x9E3779B97F4A7C15 if seed == 0 else seed
        out = []
        mask = (1 << 64) - 1
        for _ in range(count):
            state = (state + 0x9E3779B97F4A7C15) & mask
            z = state
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
            out.append(z ^ (z >> 31))
        return out

    for seed in (0, 0xC0FFEE, 0x4A41534E41):
        want = ref(seed, 16)
        assert oracle.splitmix64_sequence(seed, 16) == want
        assert [int(v) for v in synthetic.SplitMix64(seed).next_u64(16)] == want


def test_offset_transform_matches_reference_cli_check():
    kat = reference_kats()["offset_transform"]
    plane = kat["plane"]
    raw, f1, f2 = (np.array(kat[k], np.float32) for k in ("raw", "flow1", "flow2"))
    offset, mask = oracle.prepare_offsets(plane, raw, f1, f2)
    # The reference CLI's own expectation (JasnaCLI.swift:186-207), restated independently.
    err = 0.0
    for ch in range(288):
        for sp in range(plane):
            i = ch * plane + sp
            flow = f1 if ch < 144 else f2
            fc = 1 if (ch % 144) % 2 == 0 else 0
            err = max(err, abs(10 * math.tanh(raw[i]) + flow[fc * plane + sp] - offset[i]))
    for ch in range(144):
        for sp in range(plane):
            err = max(err, abs(1 / (1 + math.exp(-raw[(ch + 288) * plane + sp])) - mask[ch * plane + sp]))
    assert err < 1e-5
