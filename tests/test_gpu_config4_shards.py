"""GPU: oracle parity on the benchmarked config-4 data itself, sampled across every shard.

bench.py times config 4 (2048 FP16 tiles of 128x64x64, flow U(-16,16)) with rank r of N
owning tiles shard_range(2048, r, N), generated on its GPU by synthetic.bench_inputs (tile t
from its own seed 1000 + t) and convolved as one dcn_forward_f16 call over the whole shard.
This test rebuilds those shards on one GPU for the 1-GPU layout (one 2048-tile batch) and the
8-GPU layout (eight 256-tile shards), runs each exactly as the bench does, and compares 128
tiles spread over the eight ranges of shard_range(2048, r, 8) -- 16 per range, the first and
last tile of each included -- with the CPU restatement of DeformConvCPU.run
(Sources/JasnaMetalPoC/DeformConv.swift:75-138) under the FP16 gates (max abs <= 2e-2, mean
abs <= 2e-3 against the FP32 oracle on the same FP16 inputs).  The two layouts hold the same
tiles, so their outputs for the sample must also agree bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from jasnamacos_b200 import sharding, synthetic

pytestmark = pytest.mark.gpu

F16_MAX_ABS = 2e-2
F16_MEAN_ABS = 2e-3
TILES = 2048


_LAYOUT_OUTPUTS: dict[int, np.ndarray] = {}


@pytest.mark.parametrize("world", [1, 8], ids=["1gpu_layout", "8gpu_layout"])
def test_config4_benchmarked_shards_match_oracle(cuda_op, world):
    import torch

    sample = sharding.sample_tiles(TILES, 8, 16)
    assert len(sample) == 128
    per = synthetic.config_shape(4, batch=1)
    checked = []
    worst_max, sum_abs, count = 0.0, 0.0, 0
    outputs = {}
    packed = b16 = w16 = None
    for rank in range(world):
        shape, first, x, off, msk, w, b = synthetic.bench_inputs(4, rank, world, "cuda", TILES)
        if packed is None:
            w16 = torch.from_numpy(w).cuda().half()
            b16 = torch.from_numpy(b).cuda().half()
            packed = cuda_op.prepack(shape, w16)
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        out = cuda_op.forward_f16(shape, x, off, msk, packed, b16, flag=flag)
        torch.cuda.synchronize()
        assert int(flag.item()) == 0
        mine = [t - first for t in sample if first <= t < first + shape.batch]
        idx = torch.tensor(mine, device="cuda")
        sub = per.with_batch(len(mine))

        def rows(t, count):
            return t.view(shape.batch, count).index_select(0, idx).float().cpu().numpy().reshape(-1)

        ref = oracle.run(sub, rows(x, per.input_count), rows(off, per.offset_count), rows(msk, per.mask_count),
                         w16.float().cpu().numpy(), b16.float().cpu().numpy(), threads=oracle.host_threads())
        got = rows(out, per.output_count)
        d = np.abs(got - ref).reshape(len(mine), -1)
        assert np.isfinite(d).all(), f"rank {rank}: non-finite output"
        for j, t in enumerate(mine):
            assert float(d[j].max()) <= F16_MAX_ABS, (world, rank, first + t, float(d[j].max()))
        worst_max = max(worst_max, float(d.max()))
        sum_abs += float(d.sum())
        count += d.size
        checked += [first + t for t in mine]
        for j, t in enumerate(mine):
            outputs[first + t] = got.reshape(len(mine), -1)[j]
        del x, off, msk, out
        torch.cuda.empty_cache()
    assert sorted(checked) == sample  # every sampled tile, in every shard range, was compared
    assert sum_abs / count <= F16_MEAN_ABS, (world, sum_abs / count)
    assert worst_max <= F16_MAX_ABS
    _LAYOUT_OUTPUTS[world] = np.stack([outputs[t] for t in sample])
    if len(_LAYOUT_OUTPUTS) == 2:  # both layouts ran in this session: same tiles, same bits
        assert np.array_equal(_LAYOUT_OUTPUTS[1], _LAYOUT_OUTPUTS[8])
