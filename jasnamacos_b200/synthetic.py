"""Seeded synthetic DCNv2 inputs for the benchmark configurations.

The reference draws its benchmark inputs from ``SeededGenerator`` (SplitMix64,
Sources/JasnaMetalPoC/DeformConv.swift:168-186) through Swift's
``Float.random(in:using:)``.  The latter is Swift standard-library behaviour that is not
part of the reference, so this module keeps the SplitMix64 stream and converts it with
its own documented rules:

* uniform: the top 24 bits of a SplitMix64 output, ``u = (z >> 40) * 2**-24`` in [0, 1),
  scaled to ``lo + (hi - lo) * u``;
* normal: Box-Muller on two 53-bit uniforms, ``sqrt(-2 ln u1) * cos(2 pi u2)`` with
  ``u1`` in (0, 1].

Configurations (shapes and distributions of the DCNv2 benchmark set):
  0  FP32 1x128x64x64 -> 64, 3x3, pad 1, 16 deformable groups; x ~ N(0,1); W Kaiming-uniform
     U(+-1/sqrt(1152)); bias U(-0.1, 0.1); offset ~ N(0, 2^2); mask = sigmoid(N(0,1)).
  1  config 0 quantised to FP16.
  2  N=128 tiles; offset channel 2(g*9+k) = 10*tanh(N(0,1)) + f_y[p], channel +1 = 10*tanh(N(0,1))
     + f_x[p], one flow (f_x, f_y) ~ U(-16,16) per pixel shared by all 144 (group, tap) pairs, as
     prepare_dcn_offsets_fp16 adds one flow per pixel (MetalShader.swift:828-834).
  3  1x128x270x480, flow U(-32,32).
  4  N=2048 tiles with config 2's distributions.
Tile t of a batch is generated from its own stream (seed mixed with t), so any subset of
tiles can be regenerated exactly for sampled parity checks.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .deform_conv import DeformConvShape

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)


def _mix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _C1
        z = (z ^ (z >> np.uint64(27))) * _C2
    return z ^ (z >> np.uint64(31))


class SplitMix64:
    """SeededGenerator (DeformConv.swift:168-181), vectorised: output i of the stream is
    mix(seed + (i + 1) * gamma)."""

    def __init__(self, seed: int):
        self.state = np.uint64(0x9E3779B97F4A7C15 if seed == 0 else seed & 0xFFFFFFFFFFFFFFFF)
        self.counter = 0

    def next_u64(self, count: int) -> np.ndarray:
        idx = np.arange(self.counter + 1, self.counter + 1 + count, dtype=np.uint64)
        self.counter += count
        with np.errstate(over="ignore"):
            states = self.state + idx * _GAMMA
        return _mix(states)

    def uniform(self, count: int, lo: float, hi: float) -> np.ndarray:
        u = (self.next_u64(count) >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))
        return (lo + (hi - lo) * u).astype(np.float32)

    def normal(self, count: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
        z = self.next_u64(2 * count)
        u1 = ((z[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / (1 << 53))
        u2 = (z[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
        n = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
        return (mean + std * n).astype(np.float32)


def tile_seed(seed: int, tile: int) -> int:
    """Independent stream per (config seed, tile index)."""
    return int(_mix(np.array([(seed * 0x100000001B3 + tile + 1) & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64))[0])


def sigmoid(x: np.ndarray) -> np.ndarray:
    return (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)


def quantize_f16(a: np.ndarray) -> np.ndarray:
    """FP16-quantised copy widened back to FP32: the oracle reads exactly the GPU's bits."""
    return a.astype(np.float16).astype(np.float32)


@dataclass
class DcnInputs:
    shape: DeformConvShape
    input: np.ndarray   # float32 [N*C*H*W]
    offset: np.ndarray  # float32
    mask: np.ndarray    # float32
    weight: np.ndarray  # float32 OIHW
    bias: np.ndarray    # float32

    def quantized(self) -> "DcnInputs":
        return DcnInputs(self.shape, quantize_f16(self.input), quantize_f16(self.offset),
                         quantize_f16(self.mask), quantize_f16(self.weight), quantize_f16(self.bias))

    def tensors_f16(self):
        return [a.astype(np.float16) for a in (self.input, self.offset, self.mask, self.weight, self.bias)]


def weights(shape: DeformConvShape, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Kaiming-uniform weight U(+-1/sqrt(fan_in)) (PyTorch's conv default) and bias U(-0.1, 0.1)."""
    rng = SplitMix64(seed)
    bound = 1.0 / np.sqrt((shape.input_channels // shape.groups) * shape.kernel_area)
    w = rng.uniform(shape.weight_count, -bound, bound)
    b = rng.uniform(shape.output_channels, -0.1, 0.1)
    return w, b


def gaussian_tile(shape: DeformConvShape, seed: int, offset_std: float = 2.0):
    """One image of config 0: x ~ N(0,1), offset ~ N(0, std^2), mask = sigmoid(N(0,1))."""
    one = shape.with_batch(1)
    rng = SplitMix64(seed)
    x = rng.normal(one.input_count)
    off = rng.normal(one.offset_count, 0.0, offset_std)
    msk = sigmoid(rng.normal(one.mask_count))
    return x, off, msk


def flow_tile(shape: DeformConvShape, seed: int, flow_range: float):
    """One image in BasicVSR++ second-order alignment form (configs 2-4)."""
    one = shape.with_batch(1)
    rng = SplitMix64(seed)
    plane = one.output_height * one.output_width
    pairs = one.offset_groups * one.kernel_area
    x = rng.normal(one.input_count)
    flow_x = rng.uniform(plane, -flow_range, flow_range)
    flow_y = rng.uniform(plane, -flow_range, flow_range)
    residue = 10.0 * np.tanh(rng.normal(2 * pairs * plane).astype(np.float64)).reshape(pairs, 2, plane)
    off = np.empty((pairs, 2, plane), dtype=np.float32)
    off[:, 0, :] = residue[:, 0, :] + flow_y[None, :]
    off[:, 1, :] = residue[:, 1, :] + flow_x[None, :]
    msk = sigmoid(rng.normal(pairs * plane))
    return x, off.reshape(-1), msk


CONFIG_SEED = 0x4A41534E41


def config_shape(config: int, batch: int | None = None) -> DeformConvShape:
    if config in (0, 1):
        return DeformConvShape.jasna_propagation(1)
    if config == 2:
        return DeformConvShape.jasna_propagation(128 if batch is None else batch)
    if config == 3:
        return DeformConvShape.jasna_propagation(1, 270, 480)
    if config == 4:
        return DeformConvShape.jasna_propagation(2048 if batch is None else batch)
    raise ValueError(f"unknown config {config}")


def generate(config: int, tiles=None, batch: int | None = None, seed: int = CONFIG_SEED) -> DcnInputs:
    """Inputs of `config` for the given tile indices (default: every tile of the batch).
    The returned shape's batch is len(tiles).  FP16 configs (1-4) come back FP16-quantised."""
    full = config_shape(config, batch)
    if tiles is None:
        tiles = range(full.batch)
    tiles = list(tiles)
    shape = full.with_batch(len(tiles))
    w, b = weights(shape, seed)
    xs, offs, msks = [], [], []
    for t in tiles:
        ts = tile_seed(seed + config, t)
        if config in (0, 1):
            x, off, msk = gaussian_tile(shape, ts)
        else:
            x, off, msk = flow_tile(shape, ts, 32.0 if config == 3 else 16.0)
        xs.append(x)
        offs.append(off)
        msks.append(msk)
    inputs = DcnInputs(shape, np.concatenate(xs), np.concatenate(offs), np.concatenate(msks), w, b)
    return inputs if config == 0 else inputs.quantized()


def device_gaussian_batch(shape: DeformConvShape, seed: int, device, dtype=None, weight_seed: int = CONFIG_SEED):
    """Config 0/1 distributions generated in device memory (x ~ N(0,1), offset ~ N(0, 2^2),
    mask = sigmoid(N(0,1))), FP16 unless `dtype` says otherwise; weights/bias from `weights`."""
    import torch

    dtype = torch.float16 if dtype is None else dtype
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn(shape.input_count, generator=g, device=device).to(dtype)
    off = (2.0 * torch.randn(shape.offset_count, generator=g, device=device)).to(dtype)
    msk = torch.sigmoid(torch.randn(shape.mask_count, generator=g, device=device)).to(dtype)
    w, b = weights(shape, weight_seed)
    return x, off, msk, w, b


def device_raw_batch(shape: DeformConvShape, flow_range: float, seed: int, device):
    """The offset network's raw output (2*G*9 residues ~ N(0,1), then G*9 mask logits ~ N(0,1))
    and two flows ~ U(-flow_range, flow_range) in (x, y) order, FP16, in device memory."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    plane = shape.output_height * shape.output_width
    gka = shape.offset_groups * shape.kernel_area
    raw = torch.randn(shape.batch * 3 * gka * plane, generator=g, device=device).half()
    f1 = ((torch.rand(shape.batch * 2 * plane, generator=g, device=device) * 2 - 1) * flow_range).half()
    f2 = ((torch.rand(shape.batch * 2 * plane, generator=g, device=device) * 2 - 1) * flow_range).half()
    return raw, f1, f2


def device_batch(shape: DeformConvShape, flow_range: float, seed: int, device, weight_seed: int = CONFIG_SEED):
    """Config 2/3/4 distributions generated directly in device memory with torch's seeded
    generator (for benchmark batches too large to draw on the host).  Returns FP16 tensors
    (input, offset, mask) and FP32 host (weight, bias) from `weights`."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    n = shape.batch
    plane = shape.output_height * shape.output_width
    pairs = shape.offset_groups * shape.kernel_area
    x = torch.randn(shape.input_count, generator=g, device=device, dtype=torch.float32).half()
    flow = (torch.rand(n, 2, 1, plane, generator=g, device=device) * 2 - 1) * flow_range  # (x, y)
    off = torch.empty(n, pairs, 2, plane, device=device, dtype=torch.float16)
    for i in range(n):  # one image at a time keeps the FP32 temporaries small
        res = 10.0 * torch.tanh(torch.randn(pairs, 2, plane, generator=g, device=device))
        res[:, 0, :] += flow[i, 1]
        res[:, 1, :] += flow[i, 0]
        off[i] = res.half()
    msk = torch.sigmoid(torch.randn(n * pairs * plane, generator=g, device=device)).half()
    w, b = weights(shape, weight_seed)
    return x, off.reshape(-1), msk, w, b


# Benchmark layout: which images a rank owns and how its inputs are seeded.  Tile batches
# (configs 2 and 4) are sharded over the ranks; single-image configurations (0, 1, 3) run one
# replica per rank.
BENCH_SEED = 1000
SHARDED_CONFIGS = (2, 4)
FLOW_RANGE = {0: None, 1: None, 2: 16.0, 3: 32.0, 4: 16.0}


def bench_images(config: int, rank: int, world: int, total_tiles: int | None = None) -> tuple[int, int]:
    """Images [begin, end) of the benchmark batch that `rank` of `world` processes."""
    from .sharding import shard_range

    total = config_shape(config, total_tiles if config == 4 else None).batch
    if config in SHARDED_CONFIGS:
        return shard_range(total, rank, world)
    return 0, total


def device_tiles(config: int, begin: int, end: int, device):
    """Benchmark images [begin, end) of `config` in device memory, image t generated from its
    own seed BENCH_SEED + t with torch's generator (config 0 FP32, the others FP16), so every
    image is the same whatever the rank layout: any benchmarked tile can be rebuilt on any GPU.
    Returns (x, offset, mask, weight, bias); weight and bias (host FP32) are `weights`."""
    import torch

    one = config_shape(config, batch=1)
    n = end - begin
    dtype = torch.float32 if config == 0 else torch.float16
    x = torch.empty(n * one.input_count, dtype=dtype, device=device)
    off = torch.empty(n * one.offset_count, dtype=dtype, device=device)
    msk = torch.empty(n * one.mask_count, dtype=dtype, device=device)
    for k, t in enumerate(range(begin, end)):
        if FLOW_RANGE[config] is None:
            xi, oi, mi, _, _ = device_gaussian_batch(one, seed=BENCH_SEED + t, device=device, dtype=dtype)
        else:
            xi, oi, mi, _, _ = device_batch(one, FLOW_RANGE[config], seed=BENCH_SEED + t, device=device)
        x[k * one.input_count:(k + 1) * one.input_count].copy_(xi)
        off[k * one.offset_count:(k + 1) * one.offset_count].copy_(oi)
        msk[k * one.mask_count:(k + 1) * one.mask_count].copy_(mi)
    w, b = weights(one, CONFIG_SEED)
    return x, off, msk, w, b


def bench_inputs(config: int, rank: int, world: int, device, total_tiles: int | None = None,
                 images: tuple[int, int] | None = None):
    """The device-resident inputs the benchmark times for `config` on `rank` of `world` (or for
    the explicit image range `images`): (shape of the rank's batch, first image index, x,
    offset, mask, weight, bias), generated by device_tiles."""
    b, e = images if images is not None else bench_images(config, rank, world, total_tiles)
    shape = config_shape(config, batch=1).with_batch(e - b)
    return (shape, b) + tuple(device_tiles(config, b, e, device))
