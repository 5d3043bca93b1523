"""Host-side logic that needs no GPU: errors, shapes, statistics, weight files, generators."""

from __future__ import annotations

import math

import numpy as np
import pytest

from golden_data import reference_kats
from jasnamacos_b200 import synthetic, weights
from jasnamacos_b200.benchmark_statistics import BenchmarkStatistics
from jasnamacos_b200.deform_conv import (
    CommandFailed,
    DeformConvShape,
    DeviceUnavailable,
    InvalidArrayCount,
    InvalidShape,
    NonFiniteOutput,
    Unsupported,
    check_counts,
)


def test_only_non_finite_output_is_recoverable():
    # DeformConvCPUTests.swift:35-41
    assert NonFiniteOutput("overflow").is_recoverable_numerical_failure
    assert not InvalidShape().is_recoverable_numerical_failure
    assert not DeviceUnavailable().is_recoverable_numerical_failure
    assert not Unsupported("missing").is_recoverable_numerical_failure
    assert not CommandFailed("device lost").is_recoverable_numerical_failure


def test_benchmark_statistics_even_sample_set():
    kat = reference_kats()["benchmark_statistics"]
    st = BenchmarkStatistics.from_samples(kat["samples"])
    assert list(st.samples) == kat["sorted"]
    assert st.minimum == kat["minimum"] and st.maximum == kat["maximum"]
    assert st.median == kat["median"] and st.mean == kat["mean"]
    assert abs(st.standard_deviation - math.sqrt(kat["standard_deviation_squared"])) < kat["tolerance"]
    assert abs(st.percentile10 - kat["percentile10"]) < kat["tolerance"]
    assert abs(st.percentile90 - kat["percentile90"]) < kat["tolerance"]


def test_benchmark_statistics_rejects_empty_and_nonfinite():
    assert BenchmarkStatistics.from_samples([]) is None
    assert BenchmarkStatistics.from_samples([1, math.inf]) is None
    assert BenchmarkStatistics.from_samples([1, math.nan]) is None
    one = BenchmarkStatistics.from_samples([3.0])
    assert one.median == one.percentile10 == one.percentile90 == 3.0


def test_shape_counts_match_reference_formulas():
    s = DeformConvShape.jasna_propagation()
    assert s.input_count == 128 * 64 * 64
    assert s.offset_count == 2 * 16 * 9 * 64 * 64
    assert s.mask_count == 16 * 9 * 64 * 64
    assert s.weight_count == 64 * 128 * 9
    assert s.output_count == 64 * 64 * 64
    g = DeformConvShape(2, 8, 5, 6, 4, 5, 6, 3, 3, 1, 1, 1, 1, 1, 1, 2, 4)
    assert g.weight_count == 4 * 4 * 9


def test_check_counts_names_the_short_array():
    s = DeformConvShape(1, 1, 2, 2, 1, 2, 2, 1, 1, 0, 0, 1, 1, 1, 1, 1, 1)
    check_counts(s, [1, 2, 3, 4], [0] * 8, [0.5] * 4, [2], [1])
    with pytest.raises(InvalidArrayCount) as e:
        check_counts(s, [1, 2, 3], [0] * 8, [0.5] * 4, [2], [1])
    assert e.value.name == "input" and e.value.expected == 4 and e.value.actual == 3
    with pytest.raises(InvalidArrayCount) as e:
        check_counts(s, [1, 2, 3, 4], [0] * 8, [0.5] * 4, [2], [1, 1])
    assert e.value.name == "bias"


def test_weight_set_round_trip(tmp_path):
    rng = synthetic.SplitMix64(7)
    sets = {}
    for i, d in enumerate(weights.DIRECTIONS):
        w = rng.uniform(64 * 128 * 9, -0.1, 0.1).reshape(64, 128, 3, 3)
        b = rng.uniform(64, -0.1, 0.1)
        sets[d] = (w, b)
    manifest = weights.write_weight_sets(tmp_path, sets)
    assert manifest["format"] == weights.FORMAT
    loaded = weights.load_deform_conv_weight_sets(tmp_path)
    assert [s.direction for s in loaded] == list(weights.DIRECTIONS)
    for s in loaded:
        assert len(s.data) == weights.EXPECTED_BYTES == 147_584
        w, b = sets[s.direction]
        assert np.array_equal(s.oihw(), w.astype(np.float16))
        packed, bias = s.arrays()
        # [ic][k][oc] element (ic=5, k=7, oc=3) is OIHW (3, 5, 7//3, 7%3).
        assert packed[(5 * 9 + 7) * 64 + 3] == np.float16(w[3, 5, 2, 1])
        assert np.array_equal(bias, b.astype(np.float16))


def test_weight_set_rejects_wrong_size(tmp_path):
    p = tmp_path / "backward_1.dcnfp16"
    p.write_bytes(b"\0" * 100)
    with pytest.raises(weights.WeightFileError):
        weights.DeformConvWeightSet.from_file("backward_1", p)


def test_synthetic_generators_are_deterministic_and_distributed():
    a = synthetic.generate(1, tiles=[3])
    b = synthetic.generate(1, tiles=[3])
    assert np.array_equal(a.input, b.input) and np.array_equal(a.offset, b.offset)
    two = synthetic.generate(2, tiles=[0, 5])
    five = synthetic.generate(2, tiles=[5])
    per = five.shape.input_count
    assert np.array_equal(two.input[per:], five.input)  # tile 5 is the same wherever it is generated
    x = synthetic.SplitMix64(1).normal(200_000)
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01
    u = synthetic.SplitMix64(2).uniform(200_000, -16, 16)
    assert u.min() >= -16 and u.max() < 16 and abs(float(u.mean())) < 0.1
    # config 2: dy channel = residue + flow_y, so (offset - 10*tanh) is one value per pixel.
    s = two.shape
    plane = s.output_height * s.output_width
    off = two.offset[: s.offset_count // 2].reshape(144, 2, plane)
    assert np.all(np.abs(off) <= 26.5)


def test_jasna_shape_matches_reference_benchmark_shape():
    s = DeformConvShape.jasna_propagation()
    assert s.as_tuple() == (1, 128, 64, 64, 64, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 16)
