// dcn_temporal.cu -- the temporal preparation that feeds the DCN in the Jasna recurrence.
//
// Replaces MetalDeformConv.runTemporalPreparation (Sources/JasnaMetalPoC/MetalRunner.swift:510-582),
// which runs two Metal kernels (MetalShader.swift:736-813):
//   accumulate_second_order_flow_fp16: flow2 = half(flow1 + warp(previous_flow, flow1)), or 0;
//   assemble_temporal_alignment_fp16:  conditions = [warp(feat_prop, flow1), feat_current,
//                                      warp(feat_n2, flow2), flow1, flow2] (196 channels, the
//                                      offset network's input) and deform_input = [feat_prop,
//                                      feat_n2] (the DCN's input).
// Here it is one kernel over a batch of frames: every thread owns one pixel and a slice of 8 of
// the 64 feature channels, computes the pixel's second-order flow itself (two bilinear samples of
// the previous flow, rounded to FP16 as the reference stores it) and then warps its channels of
// both feature maps with the two flows, so flow2 is never read back.  deform_input is optional:
// the DCN entry points take the two feature tensors directly (dcn_io.input_second), which makes
// the concatenation copy unnecessary.  The sampling arithmetic is the reference's (`sample_fp16`,
// MetalShader.swift:52-74, and the CPU check's `sampleZero`, JasnaCLI.swift:213-225) with one
// IEEE rounding per operation, so results equal the CPU restatement bit for bit.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "dcn_b200.h"
#include "dcn_common.cuh"

namespace dcn {

namespace {

constexpr int kTpThreads = 128;   // pixels per block
constexpr int kTpSlice = 8;       // feature channels per thread
constexpr int kTpChannels = 64;   // channels of each feature map
constexpr int kTpSlices = kTpChannels / kTpSlice;

struct TemporalArgs {
    const __half *feat_prop, *feat_current, *feat_n2;  // [N][64][H][W]
    const __half *flow1, *previous;                     // [N][2][H][W], (x, y)
    __half *conditions;                                 // [N][196][H][W]
    __half *deform_input;                               // [N][128][H][W] or null
    __half *flow2;                                      // [N][2][H][W]
    int N, H, W;
    int has_second_order;
};

// One bilinear sampling position: the four corners' in-image flags, the top-left index and the
// fractions, as sample_fp16 / sampleZero compute them (floor with int32 saturation, NaN -> 0).
struct Corners {
    int64_t i00;
    bool in00, in01, in10, in11;
    float ly, lx;
};

__device__ __forceinline__ Corners corners(float y, float x, int H, int W) {
    const int64_t y0 = __float2int_rd(y), x0 = __float2int_rd(x);
    const int64_t y1 = y0 + 1, x1 = x0 + 1;
    Corners c;
    c.ly = __fsub_rn(y, static_cast<float>(y0));
    c.lx = __fsub_rn(x, static_cast<float>(x0));
    const bool r0 = y0 >= 0 && y0 < H, r1 = y1 >= 0 && y1 < H;
    const bool c0 = x0 >= 0 && x0 < W, c1 = x1 >= 0 && x1 < W;
    c.in00 = r0 && c0;
    c.in01 = r0 && c1;
    c.in10 = r1 && c0;
    c.in11 = r1 && c1;
    c.i00 = y0 * W + x0;
    return c;
}

// v00*(1-ly)*(1-lx) + v01*(1-ly)*lx + v10*ly*(1-lx) + v11*ly*lx, left to right, each
// operation rounded once.
__device__ __forceinline__ float sample(const __half *plane, const Corners &c, int W) {
    const float v00 = c.in00 ? __half2float(plane[c.i00]) : 0.0f;
    const float v01 = c.in01 ? __half2float(plane[c.i00 + 1]) : 0.0f;
    const float v10 = c.in10 ? __half2float(plane[c.i00 + W]) : 0.0f;
    const float v11 = c.in11 ? __half2float(plane[c.i00 + W + 1]) : 0.0f;
    const float hy = __fsub_rn(1.0f, c.ly), hx = __fsub_rn(1.0f, c.lx);
    const float t0 = __fmul_rn(__fmul_rn(v00, hy), hx);
    const float t1 = __fmul_rn(__fmul_rn(v01, hy), c.lx);
    const float t2 = __fmul_rn(__fmul_rn(v10, c.ly), hx);
    const float t3 = __fmul_rn(__fmul_rn(v11, c.ly), c.lx);
    return __fadd_rn(__fadd_rn(__fadd_rn(t0, t1), t2), t3);
}

__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// grid: x = pixel blocks of one frame, y = channel slice, z strides over the frames.
__global__ void __launch_bounds__(kTpThreads) temporal_prepare_kernel(const TemporalArgs a) {
    const int64_t plane = static_cast<int64_t>(a.H) * a.W;
    const int64_t p = static_cast<int64_t>(blockIdx.x) * kTpThreads + threadIdx.x;
    if (p >= plane) return;
    const int slice = blockIdx.y;
    const int y = static_cast<int>(p / a.W), x = static_cast<int>(p - static_cast<int64_t>(y) * a.W);
    const float fy = static_cast<float>(y), fx = static_cast<float>(x);
    for (int64_t n = blockIdx.z; n < a.N; n += gridDim.z) {
        const __half *f1 = a.flow1 + n * 2 * plane;
        const float f1x = __half2float(f1[p]), f1y = __half2float(f1[plane + p]);
        const Corners c1 = corners(__fadd_rn(fy, f1y), __fadd_rn(fx, f1x), a.H, a.W);
        // The second-order flow at this pixel (accumulate_second_order_flow_fp16).
        float f2x = 0.0f, f2y = 0.0f;
        if (a.has_second_order) {
            const __half *prev = a.previous + n * 2 * plane;
            f2x = round_f16(__fadd_rn(f1x, sample(prev, c1, a.W)));
            f2y = round_f16(__fadd_rn(f1y, sample(prev + plane, c1, a.W)));
        }
        __half *cond = a.conditions + n * 196 * plane;
        if (slice == 0) {
            __half *f2 = a.flow2 + n * 2 * plane;
            f2[p] = __float2half_rn(f2x);
            f2[plane + p] = __float2half_rn(f2y);
            cond[192 * plane + p] = f1[p];
            cond[193 * plane + p] = f1[plane + p];
            cond[194 * plane + p] = __float2half_rn(f2x);
            cond[195 * plane + p] = __float2half_rn(f2y);
        }
        const Corners c2 = corners(__fadd_rn(fy, f2y), __fadd_rn(fx, f2x), a.H, a.W);
        const int64_t feat = n * kTpChannels * plane;
#pragma unroll 2
        for (int k = 0; k < kTpSlice; ++k) {
            const int ch = slice * kTpSlice + k;
            const __half *prop = a.feat_prop + feat + ch * plane;
            const __half *n2 = a.feat_n2 + feat + ch * plane;
            cond[ch * plane + p] = __float2half_rn(sample(prop, c1, a.W));
            cond[(64 + ch) * plane + p] = a.feat_current[feat + ch * plane + p];
            cond[(128 + ch) * plane + p] = __float2half_rn(sample(n2, c2, a.W));
            if (a.deform_input != nullptr) {
                __half *di = a.deform_input + n * 128 * plane;
                di[ch * plane + p] = prop[p];
                di[(64 + ch) * plane + p] = n2[p];
            }
        }
    }
}

}  // namespace

cudaError_t launch_temporal_prepare(int n, int height, int width, const __half *feat_prop, const __half *feat_current,
                                    const __half *feat_n2, const __half *flow1, const __half *previous,
                                    bool has_second_order, __half *conditions, __half *deform_input, __half *flow2,
                                    cudaStream_t stream) {
    TemporalArgs a{feat_prop, feat_current, feat_n2, flow1, previous, conditions, deform_input, flow2,
                   n, height, width, has_second_order ? 1 : 0};
    const int64_t plane = static_cast<int64_t>(height) * width;
    const dim3 grid(static_cast<unsigned>((plane + kTpThreads - 1) / kTpThreads), kTpSlices,
                    static_cast<unsigned>(n < 65535 ? n : 65535));
    temporal_prepare_kernel<<<grid, kTpThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace dcn
