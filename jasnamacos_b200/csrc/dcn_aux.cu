// dcn_aux.cu -- the two small kernels around the DCNv2 operator.
//
//  * non-finite flag: flag_non_finite_fp16 (Sources/JasnaMetalPoC/MetalShader.swift:454-463).
//    The fused kernel folds this check into its epilogue; this standalone form
//    serves the direct path and callers that check other tensors.  One atomic
//    per warp that saw an Inf/NaN instead of one per element.
//  * offset/mask producer: prepare_dcn_offsets_fp16 (MetalShader.swift:817-839):
//    offset = 10*tanh(raw) + flipped flow, mask = sigmoid(raw).
#include <cuda_fp16.h>

#include "dcn_common.cuh"

namespace dcn {

namespace {

// `rows` runs of `row_len` values, `row_stride` apart (one run per image of an output
// slot inside a larger tensor; rows = 1 for a plain array).
__global__ void flag_non_finite_kernel(const __half *__restrict__ values, int64_t rows, int64_t row_len,
                                       int64_t row_stride, uint32_t *__restrict__ flag) {
    bool bad = false;
    const int64_t count = rows * row_len;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const __half h = values[(i / row_len) * row_stride + i % row_len];
        bad |= __hisinf(h) != 0 || __hisnan(h);
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x % 32) == 0) atomicOr(flag, DCN_FLAG_NONFINITE);
}

// Raw tensor [N][3*gka][plane] (gka = deformable groups x taps; 144 for Jasna: 288 offset
// residues + 144 mask logits).  Grid: x over the plane, y = raw channel, z strides over the
// images (no 64-bit division per element).  Offset channels [0, gka) take flow1, [gka, 2*gka)
// flow2.
__global__ void __launch_bounds__(256) prepare_offsets_kernel(int64_t n_images, int gka, int64_t plane,
                                                              const __half *__restrict__ raw,
                                                              const __half *__restrict__ flow1,
                                                              const __half *__restrict__ flow2,
                                                              __half *__restrict__ offset,
                                                              __half *__restrict__ mask) {
    const int64_t spatial = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (spatial >= plane) return;
    const int channel = blockIdx.y;
    const int channels = 3 * gka;
    for (int64_t n = blockIdx.z; n < n_images; n += gridDim.z) {
        const float v = __half2float(raw[(n * channels + channel) * plane + spatial]);
        if (channel < 2 * gka) {
            const int local = channel % gka;
            const __half *flow = (channel < gka ? flow1 : flow2) + n * 2 * plane;
            // The flow is stored (x, y); offsets are interleaved (dy, dx), so even channels take row 1.
            const int flow_channel = (local & 1) == 0 ? 1 : 0;
            const float residue = 10.0f * tanhf(v);
            offset[(n * 2 * gka + channel) * plane + spatial] =
                __float2half_rn(residue + __half2float(flow[flow_channel * plane + spatial]));
        } else {
            mask[(n * gka + channel - 2 * gka) * plane + spatial] = __float2half_rn(1.0f / (1.0f + expf(-v)));
        }
    }
}

// One thread waits on an mbarrier that expects an arrival nobody makes, with the bounded
// wait of the operator kernels; when the wait runs out it records the timeout the way they
// do (one bit in the device error word) and returns.
__global__ void check_wait_timeout_kernel(uint64_t limit_ns, uint32_t *err) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbarrier_init();
    if (!mbar_wait_bounded(&bar, 0, nullptr, 0, limit_ns)) atomicOr(err, kErrWaitTimeout);
}

}  // namespace

cudaError_t launch_check_wait_timeout(uint64_t limit_ns, uint32_t *err, cudaStream_t stream) {
    check_wait_timeout_kernel<<<1, 32, 0, stream>>>(limit_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_flag_non_finite_rows(const __half *values, int64_t rows, int64_t row_len, int64_t row_stride,
                                        uint32_t *flag, int sm_count, cudaStream_t stream) {
    int64_t blocks = (rows * row_len + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    flag_non_finite_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(values, rows, row_len, row_stride,
                                                                               flag);
    return cudaGetLastError();
}

cudaError_t launch_flag_non_finite(const __half *values, int64_t count, uint32_t *flag, int sm_count,
                                   cudaStream_t stream) {
    return launch_flag_non_finite_rows(values, 1, count, count, flag, sm_count, stream);
}

cudaError_t launch_prepare_offsets(int64_t n_images, int gka, int64_t plane, const __half *raw, const __half *flow1,
                                   const __half *flow2, __half *offset, __half *mask, cudaStream_t stream) {
    if (n_images <= 0 || plane <= 0) return cudaSuccess;
    const dim3 grid(static_cast<unsigned>((plane + 255) / 256), static_cast<unsigned>(3 * gka),
                    static_cast<unsigned>(n_images < 65535 ? n_images : 65535));
    prepare_offsets_kernel<<<grid, 256, 0, stream>>>(n_images, gka, plane, raw, flow1, flow2, offset, mask);
    return cudaGetLastError();
}

}  // namespace dcn
