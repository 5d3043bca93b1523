// dcn_prepack.cu -- weight prepack kernel.
//
// Replaces the reference's offline OIHW -> [ic][k][oc] FP16 transpose
// (tools/export_deform_weights.py:47-48, in-Swift at MetalRunner.swift:235-243).
// Two destination formats, chosen by the shape:
//  * fused path: the tcgen05 B operand.  For K-block b (64 K-elements), output
//    channel row n (0..63) and 16-byte chunk c (0..7) the 8 FP16 values
//    B[kk = 64b + 8c + e][n], e = 0..7, live at byte
//        b*8192 + n*128 + ((c ^ (n % 8)) * 16) + 2e
//    i.e. K-major rows of 128 bytes with the 128-byte swizzle already applied,
//    so a plain bulk copy into 1024-byte aligned shared memory yields the
//    operand a SWIZZLE_128B K-major descriptor expects.  K order: chunk
//    j = 8b + c = g*KA + k (offset group g, tap k), channel ic = 8g + e; chunks
//    past OG*KA are zero.
//  * direct path: an OIHW FP16 copy.
// Source: FP32 or FP16, OIHW ([oc][ic][kh][kw]) or IC_K_OC ([ic][kh*kw][oc]).
#include <cuda_fp16.h>

#include "dcn_common.cuh"

namespace dcn {

namespace {

template <typename T>
__device__ __forceinline__ __half to_half(T v);
template <>
__device__ __forceinline__ __half to_half<float>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __half to_half<__half>(__half v) { return v; }

// Index of W[oc][local ic][k] in the source array.
__device__ __forceinline__ int64_t src_index(int layout, int oc, int lic, int k, int cpg, int KA, int OC) {
    return layout == DCN_WEIGHT_OIHW ? (static_cast<int64_t>(oc) * cpg + lic) * KA + k
                                     : (static_cast<int64_t>(lic) * KA + k) * OC + oc;
}

template <typename T>
__global__ void prepack_fused_kernel(const T *__restrict__ src, int layout, __half *__restrict__ dst,
                                     int kb, int nchunks, int KA, int cpg, int OC) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // destination half index
    const int64_t total = static_cast<int64_t>(kb) * 64 * 64;
    if (i >= total) return;
    const int e = static_cast<int>(i % 8);
    const int phys_chunk = static_cast<int>((i / 8) % 8);
    const int n = static_cast<int>((i / 64) % 64);
    const int b = static_cast<int>(i / 4096);
    const int c = phys_chunk ^ (n % 8);
    const int j = b * 8 + c;
    __half v = __float2half_rn(0.0f);
    if (j < nchunks) {
        const int g = j / KA;
        const int k = j % KA;
        const int ic = g * 8 + e;
        v = to_half(src[src_index(layout, n, ic, k, cpg, KA, OC)]);
    }
    dst[i] = v;
}

template <typename T>
__global__ void prepack_oihw_kernel(const T *__restrict__ src, int layout, __half *__restrict__ dst, int OC,
                                    int cpg, int KA) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = static_cast<int64_t>(OC) * cpg * KA;
    if (i >= total) return;
    const int k = static_cast<int>(i % KA);
    const int lic = static_cast<int>((i / KA) % cpg);
    const int oc = static_cast<int>(i / (static_cast<int64_t>(KA) * cpg));
    dst[i] = to_half(src[src_index(layout, oc, lic, k, cpg, KA, OC)]);
}

template <typename T>
cudaError_t launch_prepack(const Params &p, bool fused, int kb, const T *src, int layout, __half *dst,
                           cudaStream_t stream) {
    if (fused) {
        const int64_t total = static_cast<int64_t>(kb) * 64 * 64;
        prepack_fused_kernel<T><<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
            src, layout, dst, kb, p.OG * p.KA, p.KA, p.cpg, p.OC);
    } else {
        const int64_t total = static_cast<int64_t>(p.OC) * p.cpg * p.KA;
        prepack_oihw_kernel<T><<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
            src, layout, dst, p.OC, p.cpg, p.KA);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prepack_weights(const Params &p, bool fused, int kb, const void *src, dcn_dtype src_dtype,
                                   int layout, void *dst, cudaStream_t stream) {
    if (src_dtype == DCN_DTYPE_F32)
        return launch_prepack<float>(p, fused, kb, static_cast<const float *>(src), layout,
                                     static_cast<__half *>(dst), stream);
    return launch_prepack<__half>(p, fused, kb, static_cast<const __half *>(src), layout,
                                  static_cast<__half *>(dst), stream);
}

}  // namespace dcn
