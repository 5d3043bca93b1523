"""The CPU oracle against known answers worked out by hand from the reference's DCNv2 definition
(tests/hand_kats.py): fractional positions, corners outside the image, positions in (-1, 0), two
offset groups with their own offsets and masks, stride and padding.  Exact, bit for bit."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from hand_kats import cases


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
@pytest.mark.parametrize("fast", [False, True], ids=["literal", "memoised"])
def test_oracle_hand_kat(case, fast):
    out = oracle.run(case["shape"], case["input"], case["offset"], case["mask"], case["weight"], case["bias"],
                     fast=fast)
    assert np.array_equal(out, case["expected"]), (case["name"], out.tolist(), case["expected"].tolist())
