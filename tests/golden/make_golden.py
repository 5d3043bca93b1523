"""Generates the DCNv2 golden fixtures in this directory.

* ``reference_kats.json`` -- known-answer data copied from the reference's own tests
  (read as text): the 1x1 deformable convolution of
  Tests/JasnaMetalPoCTests/DeformConvCPUTests.swift:4-33 and the statistics case of
  Tests/JasnaMetalPoCTests/BenchmarkStatisticsTests.swift:5-20, plus the deterministic
  offset-transform vectors of the reference CLI self-test (Sources/JasnaMetalPoC/JasnaCLI.swift:177-182).
* ``dcn_golden.npz`` + ``dcn_golden.json`` -- small seeded DCNv2 cases computed with the
  literal CPU oracle (the restatement of DeformConvCPU.run, DeformConv.swift:75-166), each
  cross-checked here against torchvision.ops.deform_conv2d (max abs diff <= 1e-5) before it
  is written.  FP16 cases store inputs already quantised to FP16 (widened to FP32).

Run from the repository root: ``python tests/golden/make_golden.py``.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402
from jasnamacos_b200 import synthetic  # noqa: E402
from jasnamacos_b200.deform_conv import DeformConvShape  # noqa: E402


def kats() -> dict:
    # JasnaCLI.swift:177-182: raw[i] = Float16(Float((i*13) % 101)/50 - 1), plane 7;
    # flow1[i] = Float16(Float(i)/20 - 0.25); flow2[i] = Float16(0.3 - Float(i)/30).
    plane = 7
    raw = [float(np.float16(((i * 13) % 101) / 50 - 1)) for i in range(432 * plane)]
    flow1 = [float(np.float16(i / 20 - 0.25)) for i in range(2 * plane)]
    flow2 = [float(np.float16(0.3 - i / 30)) for i in range(2 * plane)]
    return {
        "deform_conv_1x1": {
            "source": "Tests/JasnaMetalPoCTests/DeformConvCPUTests.swift:4-33",
            "shape": [1, 1, 2, 2, 1, 2, 2, 1, 1, 0, 0, 1, 1, 1, 1, 1, 1],
            "input": [1, 2, 3, 4],
            "offset": [0.0] * 8,
            "mask": [0.5] * 4,
            "weight": [2],
            "bias": [1],
            "expected": [2, 3, 4, 5],
        },
        "benchmark_statistics": {
            "source": "Tests/JasnaMetalPoCTests/BenchmarkStatisticsTests.swift:5-20",
            "samples": [4, 1, 3, 2],
            "sorted": [1, 2, 3, 4],
            "minimum": 1,
            "maximum": 4,
            "median": 2.5,
            "mean": 2.5,
            "standard_deviation_squared": 1.25,
            "percentile10": 1.3,
            "percentile90": 3.7,
            "tolerance": 1e-12,
            "rejected": [[], [1, "inf"]],
        },
        "non_finite_flag": {
            "source": "Tests/JasnaMetalPoCTests/MetalNonFiniteFlagTests.swift:50-52",
            "cases": [[[0, 1, -2, 0.5], 0], [[0, "inf", 1], 1], [[0, "nan", 1], 1]],
        },
        "offset_transform": {
            "source": "Sources/JasnaMetalPoC/JasnaCLI.swift:177-211",
            "plane": plane,
            "raw": raw,
            "flow1": flow1,
            "flow2": flow2,
            "tolerance": 0.005,
        },
    }


def boundary_case():
    """1x1 kernel over a 4x4 image; offsets place samples at y/x in (-1,0), exactly on the
    last row/column, beyond the edge, on integers and at negative fractions."""
    s = DeformConvShape(1, 1, 4, 4, 1, 4, 4, 1, 1, 0, 0, 1, 1, 1, 1, 1, 1)
    x = np.arange(16, dtype=np.float32) * 0.25 - 1.0
    dy = np.array([-0.5, -1.0, 0.0, 3.0, -0.25, 2.0, 0.75, 1.5, -1.75, 0.5, -3.5, 0.999,
                   -0.001, 4.0, -4.0, 0.5], dtype=np.float32)
    dx = np.array([0.5, -0.5, 3.0, -0.25, 1.0, -1.0, 2.5, -2.0, 0.25, 0.0, 1.75, -0.999,
                   0.001, -4.0, 4.0, -0.5], dtype=np.float32)
    off = np.stack([dy, dx]).astype(np.float32).reshape(-1)
    msk = np.linspace(0.1, 1.0, 16, dtype=np.float32)
    return s, x, off, msk, np.array([1.5], np.float32), np.array([0.25], np.float32)


def seeded_case(shape: DeformConvShape, seed: int, offset_range: float, fp16: bool = False):
    rng = synthetic.SplitMix64(seed)
    x = rng.uniform(shape.input_count, -1.0, 1.0)
    off = rng.uniform(shape.offset_count, -offset_range, offset_range)
    msk = rng.uniform(shape.mask_count, 0.1, 0.9)
    w = rng.uniform(shape.weight_count, -0.2, 0.2)
    b = rng.uniform(shape.output_channels, -0.1, 0.1)
    arrays = [x, off, msk, w, b]
    if fp16:
        arrays = [synthetic.quantize_f16(a) for a in arrays]
    return (shape, *arrays)


def cases():
    S = DeformConvShape
    yield "cli_selftest_shape", seeded_case(S(1, 2, 5, 5, 3, 5, 5, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1), 0xC0FFEE, 0.4)
    yield "boundary_positions", boundary_case()
    yield "groups2_og4", seeded_case(S(1, 8, 6, 7, 4, 6, 7, 3, 3, 1, 1, 1, 1, 1, 1, 2, 4), 11, 2.5)
    yield "stride2_dil2", seeded_case(S(2, 4, 9, 11, 6, 5, 6, 3, 3, 2, 2, 2, 2, 2, 2, 1, 2), 12, 1.5)
    yield "far_offsets", seeded_case(S(1, 4, 5, 5, 2, 5, 5, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1), 13, 0.0)
    yield "kernel_1x3_pad0_1", seeded_case(S(1, 6, 5, 8, 5, 5, 8, 1, 3, 0, 1, 1, 1, 1, 1, 1, 3), 14, 3.0)
    yield "jasna_8x8_fp16", seeded_case(S.jasna_propagation(1, 8, 8), 15, 3.0, fp16=True)
    yield "jasna_ragged_12x20_fp16", seeded_case(S.jasna_propagation(2, 12, 20), 16, 6.0, fp16=True)


def torchvision_check(shape, x, off, msk, w, b, out):
    import torch
    import torchvision

    s = shape
    tv = torchvision.ops.deform_conv2d(
        torch.from_numpy(x).view(s.batch, s.input_channels, s.input_height, s.input_width),
        torch.from_numpy(off).view(s.batch, -1, s.output_height, s.output_width),
        torch.from_numpy(w).view(s.output_channels, s.input_channels // s.groups, s.kernel_height, s.kernel_width),
        torch.from_numpy(b),
        stride=(s.stride_height, s.stride_width),
        padding=(s.pad_height, s.pad_width),
        dilation=(s.dilation_height, s.dilation_width),
        mask=torch.from_numpy(msk).view(s.batch, -1, s.output_height, s.output_width),
    ).numpy().reshape(-1)
    return float(np.abs(tv - out).max())


def main() -> None:
    (HERE / "reference_kats.json").write_text(json.dumps(kats(), indent=1) + "\n")
    meta, arrays = {}, {}
    for name, (shape, x, off, msk, w, b) in cases():
        if name == "far_offsets":
            off = np.full(shape.offset_count, 50.0, np.float32)
            off[1::2] = -50.0
        out = oracle.run(shape, x, off, msk, w, b, fast=False)
        diff = torchvision_check(shape, x, off, msk, w, b, out)
        assert diff <= 1e-5, (name, diff)
        meta[name] = {"shape": list(shape.as_tuple()), "torchvision_max_abs_diff": diff}
        # FP16 cases are stored as float16 (exact: they were quantised before the oracle ran).
        in_dtype = np.float16 if name.endswith("_fp16") else np.float32
        for key, arr in (("input", x), ("offset", off), ("mask", msk), ("weight", w), ("bias", b)):
            arrays[f"{name}/{key}"] = np.asarray(arr, dtype=in_dtype)
        arrays[f"{name}/output"] = np.asarray(out, dtype=np.float32)
    np.savez_compressed(HERE / "dcn_golden.npz", **arrays)
    (HERE / "dcn_golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {len(meta)} cases")


if __name__ == "__main__":
    main()
