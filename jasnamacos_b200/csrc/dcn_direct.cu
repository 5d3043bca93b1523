// dcn_direct.cu -- direct (CUDA-core) DCNv2 kernels for any valid shape.
//
//  * FP32: the correctness-gate path (replaces deform_conv2d_fp32,
//    Sources/JasnaMetalPoC/MetalShader.swift:76-124).  Each output is the
//    reference sum of DeformConvCPU.run (DeformConv.swift:98-136) evaluated with
//    explicit round-to-nearest multiply/add intrinsics, so no FMA contraction
//    happens and the result is bit-identical to the CPU reference.
//  * FP16 storage / FP32 math: replaces deform_conv2d_fp16 (MetalShader.swift:126-174).
//
// Work split (not the reference's one-thread-per-output): a block owns 16
// consecutive output pixels and up to 64 output channels of one convolution group;
// thread (pixel p, channel quad g) accumulates channels 4g..4g+3 of pixel p.  The
// reduction index k = ic * KA + tap runs in chunks of 64: per chunk the block
// evaluates every sampled*mask product of its 16 pixels once into shared memory
// (four independent samples per thread, their loads in flight together) and stages
// the chunk's weights there, transposed to [k][oc].  Per output the additions still
// run in the reference order (bias, then ic, ky, kx), which is all bit-exactness
// needs.
#include <cuda_fp16.h>

#include "dcn_common.cuh"

namespace dcn {

namespace {

constexpr int kPix = 16;        // output pixels per block
constexpr int kOcPerBlock = 64; // output channels per block
constexpr int kQuads = kOcPerBlock / 4;
constexpr int kThreads = kPix * kQuads;  // 256
constexpr int kChunk = 64;      // reduction steps (ic, tap) per shared-memory chunk
constexpr int kSamplesPerThread = kChunk * kPix / kThreads;  // 4

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

// Shared-memory weight chunk [k][oc] with the 4-channel quads of row k XOR-swizzled by
// k mod 16, so the transposing stores (consecutive k from consecutive threads) spread
// over the banks while a quad stays one aligned 16-byte load.
__device__ __forceinline__ int wslot(int k, int oc) { return k * kOcPerBlock + (((oc >> 2) ^ (k & 15)) << 2) + (oc & 3); }

// grid.x: ceil(N*out_plane / 16) pixel blocks; grid.y: G * ceil(opg / 64).
template <typename T>
__global__ void __launch_bounds__(kThreads)
    direct_kernel(Params p, const SplitInput<T> input, const T *__restrict__ offset,
                  const T *__restrict__ mask, const T *__restrict__ weight,
                  const T *__restrict__ bias, T *__restrict__ output) {
    __shared__ float s_samples[kChunk][kPix];
    __shared__ __align__(16) float s_w[kChunk * kOcPerBlock];
    const int tid = threadIdx.x;
    const int px_lane = tid % kPix;
    const int quad = tid / kPix;
    const int oc_blocks = (p.opg + kOcPerBlock - 1) / kOcPerBlock;
    const int group = blockIdx.y / oc_blocks;
    const int oc_block = blockIdx.y % oc_blocks;
    const int oc_base = oc_block * kOcPerBlock;                 // first channel of the block, within the group
    const int oc_count = min(kOcPerBlock, p.opg - oc_base);
    const int64_t total_pix = static_cast<int64_t>(p.N) * p.out_plane;
    const int64_t pix0 = static_cast<int64_t>(blockIdx.x) * kPix;
    const int K = p.cpg * p.KA;                                 // reduction length per output

    // The pixel this thread accumulates -- and samples: in phase 1 thread (p, q) evaluates
    // reduction steps 4q .. 4q+3 of the chunk for pixel p.
    const int64_t my_pix = pix0 + px_lane;
    const bool my_valid = my_pix < total_pix;
    const int my_n = my_valid ? static_cast<int>(my_pix / p.out_plane) : 0;
    const int my_spatial = my_valid ? static_cast<int>(my_pix % p.out_plane) : 0;
    const int my_oy = my_spatial / p.WO;
    const int my_ox = my_spatial - my_oy * p.WO;
    const int base_y = my_oy * p.SH - p.PH;
    const int base_x = my_ox * p.SW - p.PW;
    const T *off_px = offset + static_cast<int64_t>(my_n) * 2 * p.OG * p.KA * p.out_plane + my_spatial;
    const T *msk_px = mask + static_cast<int64_t>(my_n) * p.OG * p.KA * p.out_plane + my_spatial;

    float acc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int oc_local = oc_base + quad * 4 + j;
        acc[j] = oc_local < p.opg ? load_val(bias, group * p.opg + oc_local) : 0.0f;
    }

    for (int k0 = 0; k0 < K; k0 += kChunk) {
        const int nk = min(kChunk, K - k0);
        // Phase 1: sampled * mask for this thread's four consecutive steps (ic, tap).
        float sv[kSamplesPerThread];
        {
            const int kg0 = k0 + quad * kSamplesPerThread;
            int lic = kg0 / p.KA;
            int tap = kg0 - lic * p.KA;
            int ky = tap / p.KW;
            int kx = tap - ky * p.KW;
#pragma unroll
            for (int j = 0; j < kSamplesPerThread; ++j) {
                float v = 0.0f;
                if (quad * kSamplesPerThread + j < nk && my_valid) {
                    const int ic = group * p.cpg + lic;
                    const int og = ic / p.cpog;
                    const int pair = og * p.KA + tap;
                    const float off_y = load_val(off_px, static_cast<int64_t>(2 * pair) * p.out_plane);
                    const float off_x = load_val(off_px, static_cast<int64_t>(2 * pair + 1) * p.out_plane);
                    const float y = __fadd_rn(static_cast<float>(base_y + ky * p.DH), off_y);
                    const float x = __fadd_rn(static_cast<float>(base_x + kx * p.DW), off_x);
                    const float sampled = sample_exact(input.channel(my_n, ic, p.in_plane), p.H, p.W, y, x);
                    const float m = load_val(msk_px, static_cast<int64_t>(pair) * p.out_plane);
                    v = __fmul_rn(sampled, m);
                }
                sv[j] = v;
                // next step: tap + 1, carrying into kx, ky and the channel
                if (++kx == p.KW) {
                    kx = 0;
                    ++ky;
                }
                if (++tap == p.KA) {
                    tap = 0;
                    ky = 0;
                    kx = 0;
                    ++lic;
                }
            }
        }
        // Weights of the chunk, [k][oc] (consecutive threads take consecutive k of one
        // channel, so the global reads follow OIHW).
        float wv[kChunk * kOcPerBlock / kThreads];
#pragma unroll
        for (int i = 0; i < kChunk * kOcPerBlock / kThreads; ++i) {
            const int e = tid + i * kThreads;
            const int kl = e % kChunk;
            const int ol = e / kChunk;
            wv[i] = (kl < nk && ol < oc_count)
                        ? load_val(weight, static_cast<int64_t>(group * p.opg + oc_base + ol) * K + k0 + kl)
                        : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kChunk * kOcPerBlock / kThreads; ++i) {
            const int e = tid + i * kThreads;
            s_w[wslot(e % kChunk, e / kChunk)] = wv[i];
        }
#pragma unroll
        for (int j = 0; j < kSamplesPerThread; ++j) s_samples[quad * kSamplesPerThread + j][px_lane] = sv[j];
        __syncthreads();
        // Phase 2: acc += (sampled * mask) * weight in the order ic, ky, kx.
        for (int kl = 0; kl < nk; ++kl) {
            const float v = s_samples[kl][px_lane];
            const float4 w = *reinterpret_cast<const float4 *>(&s_w[wslot(kl, quad * 4)]);
            acc[0] = __fadd_rn(acc[0], __fmul_rn(v, w.x));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(v, w.y));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(v, w.z));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(v, w.w));
        }
        __syncthreads();
    }

    if (my_valid) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int oc_local = oc_base + quad * 4 + j;
            if (oc_local < p.opg)
                store_val(output, output_index(p, my_n, group * p.opg + oc_local, my_spatial), acc[j]);
        }
    }
}

template <typename T>
cudaError_t launch_direct(const Params &p, const SplitInput<T> &input, const T *offset, const T *mask,
                          const T *weight, const T *bias, T *output, cudaStream_t stream) {
    const int64_t total_pix = static_cast<int64_t>(p.N) * p.out_plane;
    const int oc_blocks = (p.opg + kOcPerBlock - 1) / kOcPerBlock;
    dim3 grid(static_cast<unsigned>((total_pix + kPix - 1) / kPix), static_cast<unsigned>(p.G * oc_blocks));
    direct_kernel<T><<<grid, kThreads, 0, stream>>>(p, input, offset, mask, weight, bias, output);
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
