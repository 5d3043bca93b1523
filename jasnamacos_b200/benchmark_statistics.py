"""Benchmark sample statistics (mirrors Sources/JasnaMetalPoC/BenchmarkStatistics.swift:3-44)."""

from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class BenchmarkStatistics:
    """Sorted samples with min/max/median/mean, population standard deviation and
    linearly interpolated 10th/90th percentiles (BenchmarkStatistics.swift:13-43)."""

    samples: tuple[float, ...]
    minimum: float
    maximum: float
    median: float
    mean: float
    standard_deviation: float
    percentile10: float
    percentile90: float

    @classmethod
    def from_samples(cls, values) -> "BenchmarkStatistics | None":
        """Returns None for an empty or non-finite sample set (the Swift `init?`)."""
        values = [float(v) for v in values]
        if not values or not all(math.isfinite(v) for v in values):
            return None
        ordered = sorted(values)
        count = len(ordered)
        total = 0.0
        for v in ordered:  # summed in sorted order, as `sorted.reduce(0, +)`
            total += v
        mean = total / count
        if count % 2 == 0:
            upper = count // 2
            median = (ordered[upper - 1] + ordered[upper]) / 2
        else:
            median = ordered[count // 2]
        variance = 0.0
        for v in ordered:
            d = v - mean
            variance += d * d
        variance /= count
        return cls(
            samples=tuple(ordered),
            minimum=ordered[0],
            maximum=ordered[-1],
            median=median,
            mean=mean,
            standard_deviation=math.sqrt(variance),
            percentile10=_percentile(0.10, ordered),
            percentile90=_percentile(0.90, ordered),
        )


def _percentile(fraction: float, ordered: list[float]) -> float:
    """Linear interpolation between the neighbouring order statistics (BenchmarkStatistics.swift:36-43)."""
    if len(ordered) <= 1:
        return ordered[0]
    position = fraction * (len(ordered) - 1)
    lower = math.floor(position)
    upper = math.ceil(position)
    weight = position - lower
    return ordered[lower] * (1 - weight) + ordered[upper] * weight
