"""GPU parity against the CPU oracle (the restatement of DeformConvCPU.run,
Sources/JasnaMetalPoC/DeformConv.swift:75-166), every call through the C ABI.

Gates (the operator's numerical contract):
  * FP32 path: bit-identical to the oracle (which implies max relative error <= 1e-5,
    denominator max(|ref|, 1e-6) as JasnaCLI.swift:105).
  * FP16 path: max abs <= 2e-2 and mean abs <= 2e-3 against the FP32 oracle run on the
    same FP16-quantised inputs; fused vs direct FP16 kernel <= 0.002 (MetalRunner.swift:350-354).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from golden_data import golden_cases, reference_kats
from jasnamacos_b200 import _native, synthetic
from jasnamacos_b200.deform_conv import DeformConvShape

pytestmark = pytest.mark.gpu

F16_MAX_ABS = 2e-2
F16_MEAN_ABS = 2e-3
F32_MAX_REL = 1e-5
FUSED_VS_DIRECT = 2e-3


def assert_bit_exact(out, ref, label=""):
    out = np.asarray(out, np.float32).reshape(-1)
    ref = np.asarray(ref, np.float32).reshape(-1)
    rel = np.abs(out - ref) / np.maximum(np.abs(ref), 1e-6)
    assert float(rel.max()) <= F32_MAX_REL, f"{label}: max rel {rel.max()}"
    mism = np.flatnonzero(out.view(np.uint32) != ref.view(np.uint32))
    # +0 and -0 compare equal in the reference's float comparison; treat them as equal.
    mism = mism[~((out[mism] == 0) & (ref[mism] == 0))]
    assert mism.size == 0, f"{label}: {mism.size} outputs differ, first at {mism[:5]}"


def assert_f16_gates(out, ref, label=""):
    d = np.abs(np.asarray(out, np.float32).reshape(-1) - np.asarray(ref, np.float32).reshape(-1))
    assert np.isfinite(d).all(), label
    assert float(d.max()) <= F16_MAX_ABS, f"{label}: max abs {d.max()}"
    assert float(d.mean()) <= F16_MEAN_ABS, f"{label}: mean abs {d.mean()}"
    return float(d.max()), float(d.mean())


# ------------------------------------------------------------------------- FP32


def test_f32_reference_kat(cuda_op):
    kat = reference_kats()["deform_conv_1x1"]
    shape = DeformConvShape(*kat["shape"])
    out = cuda_op.run_float32(shape, np.array(kat["input"]), np.array(kat["offset"]), np.array(kat["mask"]),
                              np.array(kat["weight"]), np.array(kat["bias"]))
    assert out.tolist() == kat["expected"]


@pytest.mark.parametrize("case", list(golden_cases()), ids=lambda c: c[0])
def test_f32_golden_bit_exact(cuda_op, case):
    name, shape, x, off, msk, w, b, expected = case
    out = cuda_op.run_float32(shape, x, off, msk, w, b)
    assert_bit_exact(out, expected, name)


def _random_shape(rng):
    groups = int(rng.choice([1, 2]))
    og = int(rng.choice([1, 2, 4]))
    cin = int(np.lcm(groups, og) * rng.integers(1, 4))
    cout = groups * int(rng.integers(1, 40))
    kh, kw = int(rng.integers(1, 4)), int(rng.integers(1, 4))
    ph, pw = int(rng.integers(0, 3)), int(rng.integers(0, 3))
    sh, sw = int(rng.integers(1, 3)), int(rng.integers(1, 3))
    dh, dw = int(rng.integers(1, 3)), int(rng.integers(1, 3))
    h, w = int(rng.integers(3, 20)), int(rng.integers(3, 20))
    ho = max(1, (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1)
    wo = max(1, (w + 2 * pw - dw * (kw - 1) - 1) // sw + 1)
    return DeformConvShape(int(rng.integers(1, 4)), cin, h, w, cout, ho, wo, kh, kw, ph, pw, sh, sw, dh, dw,
                           groups, og)


def test_f32_random_shapes_bit_exact(cuda_op):
    rng = np.random.default_rng(4321)
    for i in range(30):
        s = _random_shape(rng)
        g = synthetic.SplitMix64(900 + i)
        arrays = [g.uniform(s.input_count, -1, 1), g.uniform(s.offset_count, -6, 6),
                  g.uniform(s.mask_count, 0, 1), g.uniform(s.weight_count, -0.5, 0.5),
                  g.uniform(s.output_channels, -0.1, 0.1)]
        ref = oracle.run(s, *arrays)
        out = cuda_op.run_float32(s, *arrays)
        assert_bit_exact(out, ref, str(s))


def test_f32_config0_bit_exact(cuda_op):
    inp = synthetic.generate(0)
    ref = oracle.run(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    out = cuda_op.run_float32(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    assert_bit_exact(out, ref, "config 0")


# ------------------------------------------------------------------------- FP16


def test_f16_config1_fused_gates(cuda_op):
    inp = synthetic.generate(1)
    assert cuda_op.path(inp.shape) == _native.DCN_PATH_SLAB_TC  # 64x64 tiles: shared-memory slab kernel
    ref = oracle.run(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    out = cuda_op.run_float16(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    assert out.dtype == np.float16
    assert_f16_gates(out, ref, "config 1 fused")


def test_f16_config1_direct_gates_and_fused_vs_direct(cuda_op):
    import torch

    inp = synthetic.generate(1)
    s = inp.shape
    ref = oracle.run(s, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    x, off, msk, w, b = [torch.from_numpy(a).cuda() for a in inp.tensors_f16()]
    direct = cuda_op.forward_f16_direct(s, x, off, msk, w, b)
    fused = cuda_op.forward_f16(s, x, off, msk, cuda_op.prepack(s, w), b)
    torch.cuda.synchronize()
    direct, fused = direct.float().cpu().numpy(), fused.float().cpu().numpy()
    assert_f16_gates(direct, ref, "config 1 direct")
    assert np.abs(direct - ref).max() <= 1e-3  # FP32 math, one FP16 rounding
    assert float(np.abs(fused - direct).max()) <= FUSED_VS_DIRECT


@pytest.mark.parametrize("case", [c for c in golden_cases() if c[0].endswith("_fp16")], ids=lambda c: c[0])
def test_f16_golden_fixtures(cuda_op, case):
    name, shape, x, off, msk, w, b, expected = case
    out = cuda_op.run_float16(shape, x, off, msk, w, b)
    assert_f16_gates(out, expected, name)


@pytest.mark.parametrize("case", [c for c in golden_cases() if not c[0].endswith("_fp16")],
                         ids=lambda c: c[0])
def test_f16_direct_path_generic_shapes(cuda_op, case):
    """Shapes outside the fused kernel's class take the direct FP16 kernel."""
    name, shape, x, off, msk, w, b, _ = case
    q = [synthetic.quantize_f16(a) for a in (x, off, msk, w, b)]
    ref = oracle.run(shape, *q)
    out = cuda_op.run_float16(shape, *q)
    assert_f16_gates(out, ref, name)


def test_f16_config2_sampled_tiles(cuda_op, host_threads):
    tiles = [0, 37, 91, 127]
    inp = synthetic.generate(2, tiles=tiles)
    ref = oracle.run(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias, threads=host_threads)
    out = cuda_op.run_float16(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    assert_f16_gates(out, ref, "config 2 tiles")


def test_f16_config2_full_batch_properties(cuda_op):
    """Full N=128 batch: per-tile independence (tiles t..t+4 of the batch == the same five
    tiles run alone, bit for bit; five tiles are 160 128-pixel tiles, enough that the batch is
    not group-split), run-to-run determinism, finite outputs, and oracle parity on two tiles."""
    import torch

    shape = synthetic.config_shape(2)
    x, off, msk, w, b = synthetic.device_batch(shape, 16.0, seed=7, device="cuda")
    w16 = torch.from_numpy(w).cuda().half()
    b16 = torch.from_numpy(b).cuda().half()
    packed = cuda_op.prepack(shape, w16)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    out1 = cuda_op.forward_f16(shape, x, off, msk, packed, b16, flag=flag)
    out2 = cuda_op.forward_f16(shape, x, off, msk, packed, b16, flag=flag)
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)
    assert int(flag.item()) == 0
    one = shape.with_batch(1)
    five = shape.with_batch(5)
    per_in, per_off, per_msk, per_out = one.input_count, one.offset_count, one.mask_count, one.output_count
    assert cuda_op.workspace_bytes(five) == 5 * 16 * 66 * 66 * 16  # slabs only: no group split
    for t in (0, 63, 123):
        alone = cuda_op.forward_f16(five, x[t * per_in:(t + 5) * per_in], off[t * per_off:(t + 5) * per_off],
                                    msk[t * per_msk:(t + 5) * per_msk], packed, b16)
        torch.cuda.synchronize()
        assert torch.equal(alone, out1[t * per_out:(t + 5) * per_out])
    for t in (5, 120):
        xs = x[t * per_in:(t + 1) * per_in].float().cpu().numpy()
        os_ = off[t * per_off:(t + 1) * per_off].float().cpu().numpy()
        ms = msk[t * per_msk:(t + 1) * per_msk].float().cpu().numpy()
        ref = oracle.run(one, xs, os_, ms, w16.float().cpu().numpy(), b16.float().cpu().numpy())
        assert_f16_gates(out1[t * per_out:(t + 1) * per_out].float().cpu().numpy(), ref, f"tile {t}")


def test_f16_config3_large_frame(cuda_op):
    inp = synthetic.generate(3)
    ref = oracle.run(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    out = cuda_op.run_float16(inp.shape, inp.input, inp.offset, inp.mask, inp.weight, inp.bias)
    assert_f16_gates(out, ref, "config 3")


def test_prepack_sources_agree(cuda_op, tmp_path):
    """OIHW FP32, OIHW FP16 and the reference's [ic][k][oc] .dcnfp16 layout pack to the same bytes."""
    import torch

    from jasnamacos_b200 import weights

    s = DeformConvShape.jasna_propagation()
    w, b = synthetic.weights(s, 3)
    w16 = w.astype(np.float16)
    weights.write_weight_sets(tmp_path, {"backward_1": (w16.reshape(64, 128, 3, 3), b)})
    ws = weights.DeformConvWeightSet.from_file("backward_1", tmp_path / "backward_1.dcnfp16")
    packed_ickoc, _ = ws.arrays()
    p1 = cuda_op.prepack(s, torch.from_numpy(w16.astype(np.float32)).cuda())
    p2 = cuda_op.prepack(s, torch.from_numpy(w16).cuda())
    p3 = cuda_op.prepack(s, torch.from_numpy(packed_ickoc).cuda(), layout=_native.DCN_WEIGHT_IC_K_OC)
    torch.cuda.synchronize()
    assert torch.equal(p1, p2) and torch.equal(p1, p3)
    # direct-path shapes pack to an OIHW FP16 copy
    s2 = DeformConvShape(1, 16, 8, 8, 24, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 2)
    w2, _ = synthetic.weights(s2, 4)
    p4 = cuda_op.prepack(s2, torch.from_numpy(w2).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(p4.cpu().numpy().view(np.float16), w2.astype(np.float16))


def test_ragged_tiles_and_small_planes(cuda_op):
    """Planes that are not a multiple of the 128-pixel tile (fused, masked last tile), widths that
    are not a multiple of 4 (the slab pre-pass's one-column form), and planes that are not a
    multiple of 8 (direct path)."""
    for h, w_, n in ((12, 20, 3), (10, 36, 2), (8, 9, 2), (16, 6, 1), (5, 5, 2), (3, 7, 1)):
        s = DeformConvShape.jasna_propagation(n, h, w_)
        want = _native.DCN_PATH_DIRECT if (h * w_) % 8 else _native.DCN_PATH_SLAB_TC
        assert cuda_op.path(s) == want, (h, w_)
        g = synthetic.SplitMix64(h * 100 + w_)
        arrays = [synthetic.quantize_f16(a) for a in (
            g.normal(s.input_count), g.uniform(s.offset_count, -4, 4), g.uniform(s.mask_count, 0, 1),
            g.uniform(s.weight_count, -0.03, 0.03), g.uniform(s.output_channels, -0.1, 0.1))]
        ref = oracle.run(s, *arrays)
        out = cuda_op.run_float16(s, *arrays)
        assert_f16_gates(out, ref, f"{n}x{h}x{w_}")
