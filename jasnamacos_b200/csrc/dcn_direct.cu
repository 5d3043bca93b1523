// dcn_direct.cu -- direct (CUDA-core) DCNv2 kernels for any valid shape.
//
//  * FP32: the correctness-gate path (replaces deform_conv2d_fp32,
//    Sources/JasnaMetalPoC/MetalShader.swift:76-124).  Each output is the
//    reference sum of DeformConvCPU.run (DeformConv.swift:98-136) evaluated with
//    explicit round-to-nearest multiply/add intrinsics, so no FMA contraction
//    happens and the result is bit-identical to the CPU reference.
//  * FP16 storage / FP32 math: replaces deform_conv2d_fp16 (MetalShader.swift:126-174).
//
// Work split (not the reference's one-thread-per-output): a block owns 32
// consecutive output pixels and up to 64 output channels of one convolution
// group.  For a chunk of input channels it first evaluates every
// sampled*mask product once into shared memory (coalesced offset/mask reads,
// one bilinear sample per (ic, tap, pixel)), then 8 warps accumulate 8 output
// channels each from shared memory.  Per output the additions still run in the
// reference order (bias, then ic, ky, kx), which is all bit-exactness needs.
#include <cuda_fp16.h>

#include "dcn_common.cuh"

namespace dcn {

namespace {

constexpr int kPix = 32;        // output pixels per block (one per lane)
constexpr int kOcLanes = 8;     // warps per block; each accumulates 8 channels
constexpr int kOcPerBlock = 64; // output channels per block (8 per thread)
constexpr int kThreads = kPix * kOcLanes;

__device__ __forceinline__ float load_val(const float *p, int64_t i) { return p[i]; }
__device__ __forceinline__ float load_val(const __half *p, int64_t i) { return __half2float(p[i]); }
__device__ __forceinline__ void store_val(float *p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void store_val(__half *p, int64_t i, float v) { p[i] = __float2half_rn(v); }

// bilinear() of DeformConv.swift:146-165 with one IEEE rounding per operation.
// floor(y) is converted with saturation and NaN -> 0 (cvt.rmi.s32.f32).
template <typename T>
__device__ __forceinline__ float sample_exact(const T *plane, int H, int W, float y, float x) {
    const int64_t y0 = __float2int_rd(y);
    const int64_t x0 = __float2int_rd(x);
    const int64_t y1 = y0 + 1;
    const int64_t x1 = x0 + 1;
    const float ly = __fsub_rn(y, static_cast<float>(y0));
    const float lx = __fsub_rn(x, static_cast<float>(x0));
    const bool y0in = y0 >= 0 && y0 < H, y1in = y1 >= 0 && y1 < H;
    const bool x0in = x0 >= 0 && x0 < W, x1in = x1 >= 0 && x1 < W;
    const float v00 = (y0in && x0in) ? load_val(plane, y0 * W + x0) : 0.0f;
    const float v01 = (y0in && x1in) ? load_val(plane, y0 * W + x1) : 0.0f;
    const float v10 = (y1in && x0in) ? load_val(plane, y1 * W + x0) : 0.0f;
    const float v11 = (y1in && x1in) ? load_val(plane, y1 * W + x1) : 0.0f;
    const float hy = __fsub_rn(1.0f, ly);
    const float hx = __fsub_rn(1.0f, lx);
    const float t0 = __fmul_rn(__fmul_rn(v00, hy), hx);
    const float t1 = __fmul_rn(__fmul_rn(v01, hy), lx);
    const float t2 = __fmul_rn(__fmul_rn(v10, ly), hx);
    const float t3 = __fmul_rn(__fmul_rn(v11, ly), lx);
    return __fadd_rn(__fadd_rn(__fadd_rn(t0, t1), t2), t3);
}

// grid.x: ceil(N*out_plane / 32) pixel blocks; grid.y: G * ceil(opg / 64).
// Dynamic shared memory: chunk_ic * KA * 32 floats.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    direct_kernel(Params p, const SplitInput<T> input, const T *__restrict__ offset,
                  const T *__restrict__ mask, const T *__restrict__ weight,
                  const T *__restrict__ bias, T *__restrict__ output, int chunk_ic) {
    extern __shared__ float s_samples[];  // [chunk_ic][KA][kPix]
    const int tid = threadIdx.x;
    const int lane = tid % kPix;
    const int oc_lane = tid / kPix;
    const int oc_blocks = (p.opg + kOcPerBlock - 1) / kOcPerBlock;
    const int group = blockIdx.y / oc_blocks;
    const int oc_block = blockIdx.y % oc_blocks;
    const int64_t total_pix = static_cast<int64_t>(p.N) * p.out_plane;
    const int64_t pix0 = static_cast<int64_t>(blockIdx.x) * kPix;

    // The pixel this thread accumulates (and, in phase 1, samples for).
    const int64_t my_pix = pix0 + lane;
    const bool my_valid = my_pix < total_pix;
    const int my_n = my_valid ? static_cast<int>(my_pix / p.out_plane) : 0;
    const int my_spatial = my_valid ? static_cast<int>(my_pix % p.out_plane) : 0;

    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int oc_local = oc_block * kOcPerBlock + oc_lane + kOcLanes * j;
        acc[j] = oc_local < p.opg ? load_val(bias, group * p.opg + oc_local) : 0.0f;
    }

    const int per_ic = p.KA * kPix;
    for (int ic0 = 0; ic0 < p.cpg; ic0 += chunk_ic) {
        const int nic = min(chunk_ic, p.cpg - ic0);
        // Phase 1: sampled * mask for (ic, tap, pixel) of this chunk.
        for (int e = tid; e < nic * per_ic; e += kThreads) {
            const int lic = e / per_ic;
            const int k = (e / kPix) % p.KA;
            const int px = e % kPix;  // == lane for every e handled by this thread
            const int64_t pix = pix0 + px;
            float v = 0.0f;
            if (pix < total_pix) {
                const int n = static_cast<int>(pix / p.out_plane);
                const int spatial = static_cast<int>(pix % p.out_plane);
                const int oy = spatial / p.WO;
                const int ox = spatial % p.WO;
                const int ic = group * p.cpg + ic0 + lic;
                const int og = ic / p.cpog;
                const int ky = k / p.KW;
                const int kx = k % p.KW;
                const int offset_channel = 2 * (og * p.KA + k);
                const int64_t obase = static_cast<int64_t>(n) * 2 * p.OG * p.KA * p.out_plane;
                const float off_y = load_val(offset, obase + static_cast<int64_t>(offset_channel) * p.out_plane + spatial);
                const float off_x = load_val(offset, obase + static_cast<int64_t>(offset_channel + 1) * p.out_plane + spatial);
                const float y = __fadd_rn(static_cast<float>(oy * p.SH - p.PH + ky * p.DH), off_y);
                const float x = __fadd_rn(static_cast<float>(ox * p.SW - p.PW + kx * p.DW), off_x);
                const T *plane = input.channel(n, ic, p.in_plane);
                const float sampled = sample_exact(plane, p.H, p.W, y, x);
                const int64_t mbase = static_cast<int64_t>(n) * p.OG * p.KA * p.out_plane;
                const float m = load_val(mask, mbase + static_cast<int64_t>(og * p.KA + k) * p.out_plane + spatial);
                v = __fmul_rn(sampled, m);
            }
            s_samples[e] = v;
        }
        __syncthreads();
        // Phase 2: acc += (sampled * mask) * weight in the order ic, ky, kx.
        if (my_valid) {
            for (int lic = 0; lic < nic; ++lic) {
                for (int k = 0; k < p.KA; ++k) {
                    const float sv = s_samples[(lic * p.KA + k) * kPix + lane];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int oc_local = oc_block * kOcPerBlock + oc_lane + kOcLanes * j;
                        if (oc_local < p.opg) {
                            const int oc = group * p.opg + oc_local;
                            const float w = load_val(
                                weight, (static_cast<int64_t>(oc) * p.cpg + ic0 + lic) * p.KA + k);
                            acc[j] = __fadd_rn(acc[j], __fmul_rn(sv, w));
                        }
                    }
                }
            }
        }
        __syncthreads();
    }

    if (my_valid) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int oc_local = oc_block * kOcPerBlock + oc_lane + kOcLanes * j;
            if (oc_local < p.opg) {
                const int oc = group * p.opg + oc_local;
                store_val(output, output_index(p, my_n, oc, my_spatial), acc[j]);
            }
        }
    }
}

// Input channels per shared-memory chunk: keep chunk * KA * 32 floats <= 32 KiB
// (but at least one channel, for kernels up to 1024 taps = 128 KiB).
int chunk_channels(const Params &p) {
    int c = 256 / p.KA;
    if (c < 1) c = 1;
    if (c > p.cpg) c = p.cpg;
    return c;
}

template <typename T>
cudaError_t launch_direct(const Params &p, const SplitInput<T> &input, const T *offset, const T *mask,
                          const T *weight, const T *bias, T *output, cudaStream_t stream) {
    const int chunk = chunk_channels(p);
    const size_t smem = static_cast<size_t>(chunk) * p.KA * kPix * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(direct_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int64_t total_pix = static_cast<int64_t>(p.N) * p.out_plane;
    const int oc_blocks = (p.opg + kOcPerBlock - 1) / kOcPerBlock;
    dim3 grid(static_cast<unsigned>((total_pix + kPix - 1) / kPix), static_cast<unsigned>(p.G * oc_blocks));
    direct_kernel<T><<<grid, kThreads, smem, stream>>>(p, input, offset, mask, weight, bias, output, chunk);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_direct_f32(const Params &p, const float *input, const float *offset,
                              const float *mask, const float *weight, const float *bias,
                              float *output, cudaStream_t stream) {
    return launch_direct<float>(p, SplitInput<float>{input, nullptr, p.C, p.C}, offset, mask, weight, bias, output,
                                stream);
}

cudaError_t launch_direct_f16(const Params &p, const SplitInput<__half> &input, const __half *offset,
                              const __half *mask, const __half *weight, const __half *bias,
                              __half *output, cudaStream_t stream) {
    return launch_direct<__half>(p, input, offset, mask, weight, bias, output, stream);
}

}  // namespace dcn
