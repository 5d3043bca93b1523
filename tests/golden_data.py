"""Loader for the committed golden fixtures under tests/golden/."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from jasnamacos_b200.deform_conv import DeformConvShape

GOLDEN = Path(__file__).resolve().parent / "golden"


def reference_kats() -> dict:
    return json.loads((GOLDEN / "reference_kats.json").read_text())


def golden_cases():
    """Yields (name, shape, input, offset, mask, weight, bias, expected_output), float32 arrays."""
    meta = json.loads((GOLDEN / "dcn_golden.json").read_text())
    data = np.load(GOLDEN / "dcn_golden.npz")
    for name, info in meta.items():
        shape = DeformConvShape(*info["shape"])
        arrays = [data[f"{name}/{k}"].astype(np.float32) for k in ("input", "offset", "mask", "weight", "bias", "output")]
        yield (name, shape, *arrays)
