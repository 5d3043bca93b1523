"""GPU: the hand-derived known answers (tests/hand_kats.py) through the C ABI.  Every value is a
short dyadic fraction, so both the FP32 path and the FP16 path (FP16 storage, FP32 sums, one
rounding to FP16) must return them exactly."""

from __future__ import annotations

import numpy as np
import pytest

from hand_kats import cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_gpu_hand_kat(cuda_op, case):
    args = (case["shape"], case["input"], case["offset"], case["mask"], case["weight"], case["bias"])
    out32 = cuda_op.run_float32(*args)
    assert np.array_equal(out32, case["expected"]), ("fp32", out32.tolist())
    out16 = cuda_op.run_float16(*args).astype(np.float32)
    assert np.array_equal(out16, case["expected"]), ("fp16", out16.tolist())
