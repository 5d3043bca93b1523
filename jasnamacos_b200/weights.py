"""The reference's ``.dcnfp16`` DCNv2 weight files.

Format (Sources/JasnaMetalPoC/DeformConvWeights.swift:4-37, written by
tools/export_deform_weights.py:41-61): little-endian FP16 weight in
``[input_channel][kernel_element][output_channel]`` order (128 x 9 x 64), then FP16
bias[64]; 147,584 bytes per file, one file per propagation direction.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

WEIGHT_ELEMENTS = 128 * 9 * 64
BIAS_ELEMENTS = 64
EXPECTED_BYTES = (WEIGHT_ELEMENTS + BIAS_ELEMENTS) * 2
DIRECTIONS = ("backward_1", "forward_1", "backward_2", "forward_2")
FORMAT = "jasna-metal-dcnv2-fp16-v1"


class WeightFileError(ValueError):
    pass


@dataclass(frozen=True)
class DeformConvWeightSet:
    """One direction's packed weight + bias (DeformConvWeightSet, DeformConvWeights.swift:4-37)."""

    direction: str
    data: bytes

    def __post_init__(self):
        if len(self.data) != EXPECTED_BYTES:
            raise WeightFileError(f"{self.direction} has {len(self.data)} bytes; expected {EXPECTED_BYTES}")

    @classmethod
    def from_file(cls, direction: str, path: str | Path) -> "DeformConvWeightSet":
        data = Path(path).read_bytes()
        if len(data) != EXPECTED_BYTES:
            raise WeightFileError(f"{Path(path).name} has {len(data)} bytes; expected {EXPECTED_BYTES}")
        return cls(direction, data)

    def arrays(self) -> tuple[np.ndarray, np.ndarray]:
        """(weight [128*9*64] in [ic][k][oc] order, bias [64]), both float16."""
        values = np.frombuffer(self.data, dtype="<f2")
        return values[:WEIGHT_ELEMENTS].copy(), values[WEIGHT_ELEMENTS:].copy()

    def oihw(self) -> np.ndarray:
        """The weight unpacked to OIHW [64][128][3][3] (MetalRunner.swift:223-231)."""
        packed, _ = self.arrays()
        return np.ascontiguousarray(np.transpose(packed.reshape(128, 9, 64), (2, 0, 1))).reshape(64, 128, 3, 3)


def load_deform_conv_weight_sets(directory: str | Path) -> list[DeformConvWeightSet]:
    """loadDeformConvWeightSets (DeformConvWeights.swift:39-46)."""
    directory = Path(directory)
    return [DeformConvWeightSet.from_file(d, directory / f"{d}.dcnfp16") for d in DIRECTIONS]


def pack_weight_set(weight_oihw: np.ndarray, bias: np.ndarray) -> bytes:
    """The exporter's packing (tools/export_deform_weights.py:45-48): OIHW (64,128,3,3)
    -> [ic][k][oc] FP16, followed by the FP16 bias."""
    weight_oihw = np.asarray(weight_oihw)
    bias = np.asarray(bias)
    if weight_oihw.shape != (64, 128, 3, 3) or bias.shape != (64,):
        raise WeightFileError(f"unexpected shapes: {weight_oihw.shape}, {bias.shape}")
    packed = np.transpose(weight_oihw.reshape(64, 128, 9), (1, 2, 0)).astype("<f2")
    return packed.tobytes(order="C") + bias.astype("<f2").tobytes(order="C")


def write_weight_sets(directory: str | Path, sets: dict[str, tuple[np.ndarray, np.ndarray]]) -> dict:
    """Writes `<direction>.dcnfp16` files plus a sha256 manifest (export_deform_weights.py:49-61)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    manifest: dict = {
        "format": FORMAT,
        "layout": "weight[input_channel,kernel_element,output_channel], then bias[output_channel]",
        "directions": {},
    }
    for direction, (w, b) in sets.items():
        payload = pack_weight_set(w, b)
        out = directory / f"{direction}.dcnfp16"
        out.write_bytes(payload)
        manifest["directions"][direction] = {
            "file": out.name,
            "bytes": len(payload),
            "weight_elements": WEIGHT_ELEMENTS,
            "bias_elements": BIAS_ELEMENTS,
            "sha256": hashlib.sha256(payload).hexdigest(),
        }
    (directory / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest
