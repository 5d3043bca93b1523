// dcn_fused_sm100.cu -- fused FP16 DCNv2 for sm_100a: deformable gather straight
// into tensor memory + tcgen05 implicit GEMM + bias/FP16/NCHW/non-finite epilogue.
//
// Replaces the reference's two-pass FP16 path, deform_conv2d_fp16_jasna_gather
// (Sources/JasnaMetalPoC/MetalShader.swift:299-381), which materialises a
// [pixels x 1152] im2col matrix in memory, followed by
// deform_conv2d_fp16_jasna_simdgroup_gemm_fused (:387-452) and the separate
// flag_non_finite_fp16 pass (:454-463).  Here the im2col operand never leaves
// the SM: producer warps bilinearly sample, mask and round each 8-channel
// chunk to FP16 and write it into tensor memory, where tcgen05.mma consumes it
// as the A operand (M = 128 output pixels, N = 64 output channels, K = 16 per
// instruction) against weights that stay resident in shared memory for the
// whole persistent kernel.
//
// GEMM view of one output tile (128 consecutive pixels of one image):
//   out[p][oc] = bias[oc] + sum_kk A[p][kk] * B[kk][oc]
//   kk = 8*j + e, chunk j = g*KA + k (offset group g, tap k), e = channel in group
//   A[p][kk] = half( bilinear(input[n][8g+e], pos(p, g, k)) * mask[p][g][k] )
// One "stage" = 8 chunks = 64 K-elements = 4 MMAs.
//
// Warp roles (14 warps, one CTA per SM, persistent over tiles):
//   warp 0      loader   : weights once (bulk copy), then per stage the
//                          16 offset + 8 mask channel rows of the tile (TMA 3D)
//   warp 1      MMA      : TMEM allocation; one thread issues tcgen05.mma
//   warps 2-5   epilogue : TMEM -> registers, +bias, FP16, NCHW stores, Inf/NaN flag
//   warps 6-13  producers: gather + bilinear + mask -> tcgen05.st into the A stage
// Shapes this kernel takes are checked on the host (fused_supported()).
//
// Every mbarrier wait is bounded: on timeout the kernel records
// kErrWaitTimeout in the device error word, tells the other warps to stop,
// drains its own in-flight copies and MMAs, frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "dcn_common.cuh"

namespace dcn {

namespace fused {

constexpr int BM = 128;                 // output pixels per tile (TMEM lanes)
constexpr int BN = 64;                  // output channels
constexpr int kChunksPerStage = 8;      // 8 x 8 channels = 64 K-elements
constexpr int kStages = 4;              // A (TMEM) and offset/mask (smem) ring depth
constexpr int kMaxKBlocks = 18;         // resident weight K-blocks (18 x 64 = 1152)
constexpr int kBBlockBytes = BN * 128;  // one 64-wide K-block of B: 64 rows x 128 B
constexpr int kThreads = 14 * 32;
constexpr int kProducerWarps = 8;
constexpr int kEpilogueWarps = 4;
constexpr int kOffRows = 2 * kChunksPerStage;  // offset channels per stage
constexpr int kMaskRows = kChunksPerStage;     // mask channels per stage
constexpr uint32_t kStageTxBytes = (kOffRows + kMaskRows) * BM * 2;
constexpr uint32_t kTmemCols = 256;  // 2 x 64 accumulator columns + 4 x 32 A columns
constexpr uint32_t kAccCol0 = 0;
constexpr uint32_t kACol0 = 2 * BN;
constexpr uint32_t kAStageCols = kChunksPerStage * 4;  // 8 chunks x 16 B = 32 columns

struct __align__(1024) Smem {
    uint8_t b[kMaxKBlocks][kBBlockBytes];  // weights, 128B-swizzled K-major (1024-aligned)
    __half off[kStages][kOffRows][BM];     // offset rows of the stage (TMA box)
    __half msk[kStages][kMaskRows][BM];    // mask rows of the stage (TMA box)
    float bias[BN];
    uint64_t om_full[kStages];   // TMA landed offsets/masks
    uint64_t om_empty[kStages];  // producers finished reading them
    uint64_t a_full[kStages];    // producers wrote the A stage into TMEM
    uint64_t a_empty[kStages];   // MMAs reading the A stage completed
    uint64_t acc_full[2];        // accumulator buffer complete
    uint64_t acc_empty[2];       // epilogue drained the accumulator buffer
    uint64_t w_full;             // weights resident
    uint32_t tmem_base;
    int abort_flag;
};

struct Args {
    Params p;
    const uint4 *in8;          // input regrouped to [N][C/8][H][W][8] FP16 (16 B per position)
    const uint8_t *packed_w;   // kb * kBBlockBytes bytes, prepacked
    const __half *bias;        // [64]
    __half *out;               // [N][64][HO][WO]
    uint32_t *flag;            // nullable non-finite flag word
    uint32_t *err;             // sticky device error word
    int kb;                    // K-blocks (stages per tile)
    int nchunks;               // real chunks = OG * KA (the rest of the last block is zero)
    int tiles_per_image;
    int num_tiles;
};

__device__ uint32_t g_error_word;

__device__ __forceinline__ void signal_abort(Smem &s, uint32_t *err) {
    s.abort_flag = 1;
    atomicOr(err, kErrWaitTimeout);
}

__device__ __forceinline__ uint32_t pack_half2(__half2 h) {
    return *reinterpret_cast<uint32_t *>(&h);
}

__global__ void __launch_bounds__(kThreads, 1)
    fused_dcn_kernel(const __grid_constant__ CUtensorMap tmap_off,
                     const __grid_constant__ CUtensorMap tmap_msk, const Args a) {
    extern __shared__ uint8_t smem_raw[];
    Smem &s = *reinterpret_cast<Smem *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const Params &p = a.p;
    volatile int *abort_flag = &s.abort_flag;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&s.om_full[i], 1);
            mbar_init(&s.om_empty[i], kProducerWarps);
            mbar_init(&s.a_full[i], kProducerWarps);
            mbar_init(&s.a_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.acc_full[i], 1);
            mbar_init(&s.acc_empty[i], kEpilogueWarps);
        }
        mbar_init(&s.w_full, 1);
        s.abort_flag = 0;
        fence_mbarrier_init();
    }
    if (threadIdx.x < BN) s.bias[threadIdx.x] = __half2float(a.bias[threadIdx.x]);
    if (warp == 1) {
        tmem_alloc(&s.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensor_map(&tmap_off);
        prefetch_tensor_map(&tmap_msk);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ loader
        if (lane == 0) {
            mbar_arrive_expect_tx(&s.w_full, static_cast<uint32_t>(a.kb) * kBBlockBytes);
            for (int b = 0; b < a.kb; ++b)
                bulk_copy_g2s(s.b[b], a.packed_w + static_cast<size_t>(b) * kBBlockBytes, kBBlockBytes, &s.w_full);
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
                const int n = tile / a.tiles_per_image;
                const int px0 = (tile % a.tiles_per_image) * BM;
                for (int sb = 0; sb < a.kb; ++sb, ++it) {
                    const uint32_t st = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait_bounded(&s.om_empty[st], ph ^ 1u, abort_flag)) {
                        signal_abort(s, a.err);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&s.om_full[st], kStageTxBytes);
                    tma_load_3d(&s.off[st][0][0], &tmap_off, &s.om_full[st], px0, kOffRows * sb, n);
                    tma_load_3d(&s.msk[st][0][0], &tmap_msk, &s.om_full[st], px0, kMaskRows * sb, n);
                }
            }
            // Drain: wait until every copy this thread issued has landed.
            mbar_wait_bounded(&s.w_full, 0, nullptr);
            for (uint32_t k = 0; k < kStages && k < it; ++k) {
                const uint32_t last = it - 1 - k;
                mbar_wait_bounded(&s.om_full[last % kStages], (last / kStages) & 1u, nullptr);
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t idesc = make_idesc_f16_f32(BM, BN);
            const uint32_t b_base = smem_addr(&s.b[0][0]);
            bool ok = mbar_wait_bounded(&s.w_full, 0, abort_flag);
            if (!ok) signal_abort(s, a.err);
            tc_fence_after();
            uint32_t it = 0;
            uint32_t tcount = 0;
            uint64_t *last_bar = nullptr;
            uint32_t last_parity = 0;
            for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x, ++tcount) {
                const uint32_t buf = tcount & 1u;
                const uint32_t bph = (tcount >> 1) & 1u;
                if (!mbar_wait_bounded(&s.acc_empty[buf], bph ^ 1u, abort_flag)) {
                    signal_abort(s, a.err);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + kAccCol0 + buf * BN;
                for (int sb = 0; sb < a.kb; ++sb, ++it) {
                    const uint32_t st = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait_bounded(&s.a_full[st], ph, abort_flag)) {
                        signal_abort(s, a.err);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem + kACol0 + st * kAStageCols;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // K = 16 FP16 per MMA: 8 TMEM columns of A, 32 bytes along a swizzled B row.
                        const uint64_t bdesc = make_sw128_kmajor_desc(b_base + sb * kBBlockBytes + kk * 32);
                        umma_f16_ts(d_tmem, a_tmem + kk * 8, bdesc, idesc, (sb | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit(&s.a_empty[st]);
                    last_bar = &s.a_empty[st];
                    last_parity = ph;
                }
                if (!ok) break;
                umma_commit(&s.acc_full[buf]);
                last_bar = &s.acc_full[buf];
                last_parity = bph;
            }
            // Drain: the last commit arrives only after every MMA issued before it completed.
            if (last_bar != nullptr) mbar_wait_bounded(last_bar, last_parity, nullptr);
        }
    } else if (warp < 2 + kEpilogueWarps) {
        // ---------------------------------------------------------- epilogue
        const int q = warp % 4;  // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;
        bool nonfinite = false;
        uint32_t tcount = 0;
        for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x, ++tcount) {
            const uint32_t buf = tcount & 1u;
            const uint32_t bph = (tcount >> 1) & 1u;
            if (!mbar_wait_bounded(&s.acc_full[buf], bph, abort_flag)) {
                signal_abort(s, a.err);
                break;
            }
            tc_fence_after();
            uint32_t v[BN];
            const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + kAccCol0 + buf * BN;
#pragma unroll
            for (int c = 0; c < BN; c += 16) tmem_ld_32x32b_x16(taddr + c, &v[c]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.acc_empty[buf]);

            const int n = tile / a.tiles_per_image;
            const int px = (tile % a.tiles_per_image) * BM + r;
            if (px < p.out_plane) {
                __half *dst = a.out + static_cast<size_t>(n) * BN * p.out_plane + px;
#pragma unroll
                for (int oc = 0; oc < BN; ++oc) {
                    const __half h = __float2half_rn(__uint_as_float(v[oc]) + s.bias[oc]);
                    nonfinite |= __hisinf(h) != 0 || __hisnan(h);
                    dst[static_cast<size_t>(oc) * p.out_plane] = h;
                }
            }
        }
        if (a.flag != nullptr && __any_sync(0xffffffffu, nonfinite) && lane == 0)
            atomicOr(a.flag, DCN_FLAG_NONFINITE);
    } else {
        // --------------------------------------------------------- producers
        const int pw = warp - (2 + kEpilogueWarps);  // 0..7
        const int q = warp % 4;                      // TMEM lane quarter
        const int half_sel = pw / 4;                 // which 4 chunks of each stage
        const int r = q * 32 + lane;                 // tile row = pixel
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const int HW = p.in_plane;
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
            const int n = tile / a.tiles_per_image;
            const int px = (tile % a.tiles_per_image) * BM + r;
            const bool valid = px < p.out_plane;
            const int oy = valid ? px / p.WO : 0;
            const int ox = valid ? px % p.WO : 0;
            const int base_y = oy * p.SH - p.PH;
            const int base_x = ox * p.SW - p.PW;
            const uint4 *img = a.in8 + static_cast<size_t>(n) * p.OG * HW;
            for (int sb = 0; sb < a.kb; ++sb, ++it) {
                const uint32_t st = it % kStages;
                const uint32_t ph = (it / kStages) & 1u;
                if (!mbar_wait_bounded(&s.a_empty[st], ph ^ 1u, abort_flag) ||
                    !mbar_wait_bounded(&s.om_full[st], ph, abort_flag)) {
                    signal_abort(s, a.err);
                    ok = false;
                    break;
                }
                tc_fence_after();

                // Issue all 16 corner loads of the 4 chunks before using any.
                uint4 v[4][4];
                __half2 w[4][4];
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    const int c = half_sel * 4 + c4;
                    const int j = sb * kChunksPerStage + c;
#pragma unroll
                    for (int t = 0; t < 4; ++t) v[c4][t] = make_uint4(0u, 0u, 0u, 0u);
                    float w00 = 0.f, w01 = 0.f, w10 = 0.f, w11 = 0.f;
                    if (valid && j < a.nchunks) {
                        const int g = j / p.KA;
                        const int k = j - g * p.KA;
                        const int ky = k / p.KW;
                        const int kx = k - ky * p.KW;
                        const float off_y = __half2float(s.off[st][2 * c][r]);
                        const float off_x = __half2float(s.off[st][2 * c + 1][r]);
                        const float m = __half2float(s.msk[st][c][r]);
                        const float y = static_cast<float>(base_y + ky * p.DH) + off_y;
                        const float x = static_cast<float>(base_x + kx * p.DW) + off_x;
                        const int y0 = __float2int_rd(y);
                        const int x0 = __float2int_rd(x);
                        const float ly = y - static_cast<float>(y0);
                        const float lx = x - static_cast<float>(x0);
                        const float hy = 1.0f - ly;
                        const float hx = 1.0f - lx;
                        const bool y0in = static_cast<unsigned>(y0) < static_cast<unsigned>(p.H);
                        const bool y1in = static_cast<unsigned>(y0 + 1) < static_cast<unsigned>(p.H);
                        const bool x0in = static_cast<unsigned>(x0) < static_cast<unsigned>(p.W);
                        const bool x1in = static_cast<unsigned>(x0 + 1) < static_cast<unsigned>(p.W);
                        const uint4 *gplane = img + static_cast<size_t>(g) * HW;
                        const int idx = y0 * p.W + x0;
                        if (y0in && x0in) v[c4][0] = __ldg(gplane + idx);
                        if (y0in && x1in) v[c4][1] = __ldg(gplane + idx + 1);
                        if (y1in && x0in) v[c4][2] = __ldg(gplane + idx + p.W);
                        if (y1in && x1in) v[c4][3] = __ldg(gplane + idx + p.W + 1);
                        w00 = hy * hx * m;
                        w01 = hy * lx * m;
                        w10 = ly * hx * m;
                        w11 = ly * lx * m;
                    }
                    w[c4][0] = __float2half2_rn(w00);
                    w[c4][1] = __float2half2_rn(w01);
                    w[c4][2] = __float2half2_rn(w10);
                    w[c4][3] = __float2half2_rn(w11);
                }
                // The offset/mask rows of this stage are no longer needed.
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.om_empty[st]);

#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    const __half2 *h00 = reinterpret_cast<const __half2 *>(&v[c4][0]);
                    const __half2 *h01 = reinterpret_cast<const __half2 *>(&v[c4][1]);
                    const __half2 *h10 = reinterpret_cast<const __half2 *>(&v[c4][2]);
                    const __half2 *h11 = reinterpret_cast<const __half2 *>(&v[c4][3]);
                    uint32_t out[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        __half2 acc = __hmul2(w[c4][0], h00[e]);
                        acc = __hfma2(w[c4][1], h01[e], acc);
                        acc = __hfma2(w[c4][2], h10[e], acc);
                        acc = __hfma2(w[c4][3], h11[e], acc);
                        out[e] = pack_half2(acc);
                    }
                    const int c = half_sel * 4 + c4;
                    tmem_st_32x32b_x4(lane_base + kACol0 + st * kAStageCols + c * 4, out[0], out[1], out[2], out[3]);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.a_full[st]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// NCHW FP16 -> [N][C/8][H][W][8] FP16, so that one 16-byte load fetches the 8
// channels of an offset group at one position.
__global__ void __launch_bounds__(256) regroup_nchw_to_c8_kernel(const __half *__restrict__ in,
                                                                  uint4 *__restrict__ out, int C,
                                                                  int plane, int64_t total) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (n, cb, pixel)
    if (i >= total) return;
    const int pix = static_cast<int>(i % plane);
    const int64_t ncb = i / plane;
    const int cb = static_cast<int>(ncb % (C / 8));
    const int64_t n = ncb / (C / 8);
    const __half *src = in + (n * C + cb * 8) * static_cast<int64_t>(plane) + pix;
    __half h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = src[static_cast<int64_t>(e) * plane];
    uint4 o;
    o.x = pack_half2(__halves2half2(h[0], h[1]));
    o.y = pack_half2(__halves2half2(h[2], h[3]));
    o.z = pack_half2(__halves2half2(h[4], h[5]));
    o.w = pack_half2(__halves2half2(h[6], h[7]));
    out[i] = o;
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 3-D FP16 tensor map over [n][channels][plane] with a (128 pixels x rows x 1) box.
bool make_plane_map(CUtensorMap *map, const void *base, int64_t plane, int channels, int batch, int rows) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(plane), static_cast<cuuint64_t>(channels),
                          static_cast<cuuint64_t>(batch)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(plane) * 2,
                             static_cast<cuuint64_t>(plane) * channels * 2};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(BM), static_cast<cuuint32_t>(rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace fused

// Shapes the fused kernel takes: one convolution group, 64 output channels,
// 8 input channels per offset group, at most 18 K-blocks of 64, and an output
// plane that is a multiple of 8 pixels (TMA row stride rule).
bool fused_supported(const Params &p) {
    if (p.G != 1 || p.OC != fused::BN || p.cpog != 8) return false;
    const int nchunks = p.OG * p.KA;
    const int kb = (nchunks + fused::kChunksPerStage - 1) / fused::kChunksPerStage;
    if (kb > fused::kMaxKBlocks) return false;
    if (p.out_plane % 8 != 0) return false;
    if (static_cast<int64_t>(p.N) * p.OG * p.in_plane >= (int64_t{1} << 31)) return false;
    return true;
}

int fused_kblocks(const Params &p) {
    return (p.OG * p.KA + fused::kChunksPerStage - 1) / fused::kChunksPerStage;
}

size_t fused_workspace_bytes(const Params &p) {
    const size_t bytes = static_cast<size_t>(p.N) * p.C * p.in_plane * sizeof(__half);
    return (bytes + 255) & ~static_cast<size_t>(255);
}

// Once per device (with that device current): opt the kernel into its shared
// memory size and look up the device address of the sticky error word.
cudaError_t fused_prepare_device(uint32_t **err_word) {
    cudaError_t e = cudaFuncSetAttribute(fused::fused_dcn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sizeof(fused::Smem) + 1024));
    if (e != cudaSuccess) return e;
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, fused::g_error_word);
    if (e != cudaSuccess) return e;
    *err_word = static_cast<uint32_t *>(ptr);
    return cudaSuccess;
}

cudaError_t launch_fused_f16(const Params &p, const __half *input, const __half *offset, const __half *mask,
                             const uint8_t *packed_w, const __half *bias, __half *output, uint32_t *flag,
                             void *workspace, int sm_count, uint32_t *err, cudaStream_t stream) {
    using namespace fused;
    // 1) regroup the input so each offset group's 8 channels are 16 contiguous bytes.
    uint4 *in8 = static_cast<uint4 *>(workspace);
    const int64_t total = static_cast<int64_t>(p.N) * (p.C / 8) * p.in_plane;
    regroup_nchw_to_c8_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
        input, in8, p.C, p.in_plane, total);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    // 2) fused gather + tcgen05 kernel, one persistent CTA per SM.
    CUtensorMap tmap_off, tmap_msk;
    if (!make_plane_map(&tmap_off, offset, p.out_plane, 2 * p.OG * p.KA, p.N, kOffRows) ||
        !make_plane_map(&tmap_msk, mask, p.out_plane, p.OG * p.KA, p.N, kMaskRows))
        return cudaErrorInvalidValue;
    Args a;
    a.p = p;
    a.in8 = in8;
    a.packed_w = packed_w;
    a.bias = bias;
    a.out = output;
    a.flag = flag;
    a.err = err;
    a.kb = fused_kblocks(p);
    a.nchunks = p.OG * p.KA;
    a.tiles_per_image = (p.out_plane + BM - 1) / BM;
    a.num_tiles = p.N * a.tiles_per_image;
    const int grid = a.num_tiles < sm_count ? a.num_tiles : sm_count;
    fused_dcn_kernel<<<grid, kThreads, sizeof(Smem) + 1024, stream>>>(tmap_off, tmap_msk, a);
    return cudaGetLastError();
}

}  // namespace dcn
