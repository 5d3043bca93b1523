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
// instruction) against the weights, streamed from L2 one 8 KB K-block per stage.
// Keeping shared memory small matters here: the gathers read global memory through
// L1, which shares the SM's 256 KB with shared memory (holding all 144 KB of weights
// resident left about 60 KB of L1; streaming them leaves about 190 KB).
//
// GEMM view of one output tile (128 consecutive pixels of one image):
//   out[p][oc] = bias[oc] + sum_kk A[p][kk] * B[kk][oc]
//   kk = 8*j + e, chunk j = g*KA + k (offset group g, tap k), e = channel in group
//   A[p][kk] = half( bilinear(input[n][8g+e], pos(p, g, k)) * mask[p][g][k] )
// One "stage" = 8 chunks = 64 K-elements = 4 MMAs.
//
// Warp roles (14 warps, one CTA per SM, persistent over tiles):
//   warp 0      loader   : per stage the 16 offset + 8 mask channel rows of the
//                          tile (TMA 3D) and the stage's 8 KB weight K-block (bulk copy)
//   warp 1      MMA      : TMEM allocation; one thread issues tcgen05.mma
//   warps 2-5   epilogue : TMEM -> registers, +bias, FP16, NCHW stores, Inf/NaN flag
//   warps 6-13  producers: gather + bilinear + mask -> tcgen05.st into the A stage
//                          (raw-input form: offsets and masks made from the offset
//                          network's output and the flows as they are read)
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
constexpr int kMaxKBlocks = 18;         // K-blocks per tile (18 x 64 = 1152): the chunk table size
constexpr int kBBlockBytes = BN * 128;  // one 64-wide K-block of B: 64 rows x 128 B
constexpr int kThreads = 16 * 32;  // 4 warpgroups: control (loader, MMA), epilogue, 2 x producers
constexpr uint32_t kIdleBackoffNs = 200;
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
    uint8_t b[kStages][kBBlockBytes];      // the stages' weight K-blocks, 128B-swizzled K-major (1024-aligned)
    __half off[kStages][kOffRows][BM];     // offset rows of the stage (TMA box)
    __half msk[kStages][kMaskRows][BM];    // mask rows of the stage (TMA box)
    float bias[BN];
    int4 chunk[kMaxKBlocks * kChunksPerStage];  // per K-chunk: {group entry offset, ky*DH, kx*DW, real}
    uint64_t om_full[kStages];   // TMA landed offsets/masks
    uint64_t om_empty[kStages];  // producers finished reading them
    uint64_t a_full[kStages];    // producers wrote the A stage into TMEM
    uint64_t a_empty[kStages];   // MMAs reading the A stage completed
    uint64_t acc_full[2];        // accumulator buffer complete
    uint64_t acc_empty[2];       // epilogue drained the accumulator buffer
    uint32_t tmem_base;
    int abort_flag;
};

struct Args {
    Params p;
    const uint4 *pairs;        // input regrouped to corner pairs, see regroup_pairs_kernel
    const uint8_t *packed_w;   // kb * kBBlockBytes bytes, prepacked
    const __half *bias;        // [64]
    __half *out;               // [N][64][HO][WO]
    uint32_t *flag;            // nullable non-finite flag word
    uint32_t *err;             // sticky device error word
    int kb;                    // K-blocks (stages per tile)
    int nchunks;               // real chunks = OG * KA (the rest of the last block is zero)
    int tiles_per_image;
    int num_tiles;
    // Raw-input form only: the two flows [N][2][plane] ((x, y) rows; deformable groups
    // [0, OG/2) take flow1, the rest flow2) and the first mask-logit channel of the raw
    // tensor, which then stands in for both the offset and the mask tensor.
    const __half *flow1;
    const __half *flow2;
    int raw_mask_channel0;
};

__device__ uint32_t g_error_word;

__device__ __forceinline__ void signal_abort(Smem &s, uint32_t *err) {
    s.abort_flag = 1;
    atomicOr(err, kErrWaitTimeout);
}

__device__ __forceinline__ uint32_t pack_half2(__half2 h) {
    return *reinterpret_cast<uint32_t *>(&h);
}

// Per-thread state of one stage: the two 32-byte row loads of each of the
// thread's 4 chunks, and the fractional sample position + mask needed to weight
// them once they land.
struct StageRegs {
    uint32_t v[4][16];   // [chunk][row y0: 0..7 | row y0+1: 8..15], FP16 x 16 per row pair
    uint32_t frac[4];    // half2 (ly, lx)
    uint32_t msk[4];     // half mask in the low 16 bits, 0 for padding chunks
};

// FromRaw = false: offsets and masks are inputs (the reference's DCN call).
// FromRaw = true: tmap_off and tmap_msk both cover the offset network's raw output
// [N][3*OG*KA][plane] (offset residues, then mask logits), and the producers apply
// prepare_dcn_offsets_fp16 (MetalShader.swift:817-839) to each value they read, with
// the flow of the chunk's deformable group (raw_offset / raw_mask).
template <bool FromRaw>
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
        s.abort_flag = 0;
        fence_mbarrier_init();
    }
    for (int j = threadIdx.x; j < a.kb * kChunksPerStage; j += blockDim.x) {
        int4 info = make_int4(0, 0, 0, 0);
        if (j < a.nchunks) {
            const int g = j / p.KA;
            const int k = j - g * p.KA;
            const int ky = k / p.KW;
            // w: nonzero for a real chunk; 2 when the raw-input form takes flow2 for its group
            info = make_int4(g * p.H * (p.W + 1), ky * p.DH, (k - ky * p.KW) * p.DW, g < p.OG / 2 ? 1 : 2);
        }
        s.chunk[j] = info;
    }
    if (warp == 1) {
        tmem_alloc(&s.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensor_map(&tmap_off);
        prefetch_tensor_map(&tmap_msk);
    }
    // Launched as a dependent of the regroup pre-pass: no global memory before this.
    grid_dependency_wait();
    if (threadIdx.x < BN) s.bias[threadIdx.x] = __half2float(a.bias[threadIdx.x]);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;
    const int wg = warp / 4;  // warpgroup: 0 control, 1 epilogue, 2-3 producers

    if (wg == 0) {
        if (warp == 0 && lane == 0) {
            // ------------------------------------------------------------ loader
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
                const int n = tile / a.tiles_per_image;
                const int px0 = (tile % a.tiles_per_image) * BM;
                for (int sb = 0; sb < a.kb; ++sb, ++it) {
                    const uint32_t st = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    // The stage's offset/mask rows are free once the producers read them, its
                    // weight block once the MMAs of its previous use completed.
                    if (!mbar_wait_bounded(&s.om_empty[st], ph ^ 1u, abort_flag) ||
                        !mbar_wait_bounded(&s.a_empty[st], ph ^ 1u, abort_flag)) {
                        signal_abort(s, a.err);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&s.om_full[st], kStageTxBytes + kBBlockBytes);
                    tma_load_3d(&s.off[st][0][0], &tmap_off, &s.om_full[st], px0, kOffRows * sb, n);
                    tma_load_3d(&s.msk[st][0][0], &tmap_msk, &s.om_full[st], px0,
                                (FromRaw ? a.raw_mask_channel0 : 0) + kMaskRows * sb, n);
                    bulk_copy_g2s(s.b[st], a.packed_w + static_cast<size_t>(sb) * kBBlockBytes, kBBlockBytes,
                                  &s.om_full[st]);
                }
            }
            // Drain: wait until every copy this thread issued has landed.
            for (uint32_t k = 0; k < kStages && k < it; ++k) {
                const uint32_t last = it - 1 - k;
                mbar_wait_bounded(&s.om_full[last % kStages], (last / kStages) & 1u, nullptr);
            }
        } else if (warp == 1 && lane == 0) {
            // --------------------------------------------------------------- MMA
            const uint32_t idesc = make_idesc_f16_f32(BM, BN);
            bool ok = true;
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
                    // a_full: the producers stored the A stage; om_full: the stage's weight
                    // block landed (already true by then: the producers waited for it).
                    if (!mbar_wait_bounded(&s.a_full[st], ph, abort_flag) ||
                        !mbar_wait_bounded(&s.om_full[st], ph, abort_flag)) {
                        signal_abort(s, a.err);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem + kACol0 + st * kAStageCols;
                    const uint32_t b_base = smem_addr(&s.b[st][0]);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // K = 16 FP16 per MMA: 8 TMEM columns of A, 32 bytes along a swizzled B row.
                        const uint64_t bdesc = make_sw128_kmajor_desc(b_base + kk * 32);
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
    } else if (wg == 1) {
        // ---------------------------------------------------------- epilogue
        const int q = warp % 4;  // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;
        bool nonfinite = false;
        uint32_t tcount = 0;
        for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x, ++tcount) {
            const uint32_t buf = tcount & 1u;
            const uint32_t bph = (tcount >> 1) & 1u;
            if (!mbar_wait_bounded(&s.acc_full[buf], bph, abort_flag, kIdleBackoffNs)) {
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
                __half *dst = a.out + output_index(p, n, 0, px);
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
        const int q = warp % 4;                  // TMEM lane quarter
        const int half_sel = wg - 2;             // which 4 chunks of each stage
        const int r = q * 32 + lane;             // tile row = pixel
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const int row_entries = p.W + 1;
        const int local_tiles = (a.num_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                static_cast<int>(gridDim.x);
        const uint32_t total = static_cast<uint32_t>(local_tiles) * static_cast<uint32_t>(a.kb);

        // Where the prefetch pointer is: stage `pf_sb` of local tile `pf_tile`, and that
        // tile's per-pixel constants (recomputed once per tile, not per stage).
        int pf_tile = -1, pf_sb = 0;
        bool pf_valid = false;
        int pf_base_y = 0, pf_base_x = 0;
        const uint4 *pf_img = a.pairs;
        float pf_f1x = 0.0f, pf_f1y = 0.0f, pf_f2x = 0.0f, pf_f2y = 0.0f;  // raw form: this pixel's flows
        auto enter_tile = [&](int local_tile) {
            const int tile = static_cast<int>(blockIdx.x) + local_tile * static_cast<int>(gridDim.x);
            const int n = tile / a.tiles_per_image;
            const int px = (tile % a.tiles_per_image) * BM + r;
            pf_tile = local_tile;
            pf_valid = px < p.out_plane;
            const int oy = pf_valid ? px / p.WO : 0;
            const int ox = pf_valid ? px - oy * p.WO : 0;
            pf_base_y = oy * p.SH - p.PH;
            pf_base_x = ox * p.SW - p.PW;
            pf_img = a.pairs + static_cast<size_t>(n) * p.OG * p.H * row_entries * 2;
            if (FromRaw && pf_valid) {
                const int64_t f = static_cast<int64_t>(n) * 2 * p.out_plane + px;
                pf_f1x = __half2float(a.flow1[f]);
                pf_f1y = __half2float(a.flow1[f + p.out_plane]);
                pf_f2x = __half2float(a.flow2[f]);
                pf_f2y = __half2float(a.flow2[f + p.out_plane]);
            }
        };

        // Stage `itp` (the next one in order): read this pixel's offsets/masks of its 4
        // chunks and issue the 8 row loads.
        auto prefetch = [&](uint32_t itp, StageRegs &R) -> bool {
            const uint32_t st = itp % kStages;
            const uint32_t ph = (itp / kStages) & 1u;
            if (pf_tile < 0 || pf_sb == a.kb) {
                enter_tile(pf_tile + 1);
                pf_sb = 0;
            }
            const int sb = pf_sb++;
            const bool valid = pf_valid;
            const int base_y = pf_base_y, base_x = pf_base_x;
            const uint4 *img = pf_img;
            if (!mbar_wait_bounded(&s.om_full[st], ph, abort_flag)) return false;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                const int c = half_sel * 4 + c4;
                const int4 info = s.chunk[sb * kChunksPerStage + c];
#pragma unroll
                for (int t = 0; t < 16; ++t) R.v[c4][t] = 0u;
                R.frac[c4] = 0u;
                R.msk[c4] = 0u;
                if (valid && info.w) {
                    float off_y = __half2float(s.off[st][2 * c][r]);
                    float off_x = __half2float(s.off[st][2 * c + 1][r]);
                    __half mk = s.msk[st][c][r];
                    if (FromRaw) {
                        const bool second = info.w == 2;
                        off_y = raw_offset(off_y, second ? pf_f2y : pf_f1y);
                        off_x = raw_offset(off_x, second ? pf_f2x : pf_f1x);
                        mk = raw_mask(__half2float(mk));
                    }
                    const float y = static_cast<float>(base_y + info.y) + off_y;
                    const float x = static_cast<float>(base_x + info.z) + off_x;
                    const int y0 = __float2int_rd(y);
                    const int x0 = __float2int_rd(x);
                    // Entry x0+1 of a row holds the corner pair (x0, x0+1), zero-padded
                    // outside the image, so only rows need a bounds check here.
                    const bool xin = static_cast<unsigned>(x0 + 1) <= static_cast<unsigned>(p.W);
                    const bool y0in = xin && static_cast<unsigned>(y0) < static_cast<unsigned>(p.H);
                    const bool y1in = xin && static_cast<unsigned>(y0 + 1) < static_cast<unsigned>(p.H);
                    const uint4 *e0 = img + 2 * (static_cast<size_t>(info.x) + y0 * row_entries + (x0 + 1));
                    if (y0in) ldg_nc_256(e0, &R.v[c4][0]);
                    if (y1in) ldg_nc_256(e0 + 2 * row_entries, &R.v[c4][8]);
                    R.frac[c4] = pack_half2(__floats2half2_rn(y - static_cast<float>(y0), x - static_cast<float>(x0)));
                    R.msk[c4] = static_cast<uint32_t>(__half_as_ushort(mk));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.om_empty[st]);
            return true;
        };

        // Stage `itc`: bilinear-combine the landed rows and store the A stage into TMEM.
        auto commit = [&](uint32_t itc, StageRegs &R) -> bool {
            const uint32_t st = itc % kStages;
            const uint32_t ph = (itc / kStages) & 1u;
            uint32_t outw[16];  // 4 chunks x 4 columns
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&R.frac[c4]));
                const float m = __half2float(__ushort_as_half(static_cast<unsigned short>(R.msk[c4])));
                const float mhy = m * (1.0f - f.x);
                const float mly = m * f.x;
                const __half2 w00 = __float2half2_rn(mhy * (1.0f - f.y));
                const __half2 w01 = __float2half2_rn(mhy * f.y);
                const __half2 w10 = __float2half2_rn(mly * (1.0f - f.y));
                const __half2 w11 = __float2half2_rn(mly * f.y);
                const __half2 *h = reinterpret_cast<const __half2 *>(&R.v[c4][0]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    __half2 acc = __hmul2(w00, h[e]);
                    acc = __hfma2(w01, h[4 + e], acc);
                    acc = __hfma2(w10, h[8 + e], acc);
                    acc = __hfma2(w11, h[12 + e], acc);
                    outw[c4 * 4 + e] = pack_half2(acc);
                }
            }
            if (!mbar_wait_bounded(&s.a_empty[st], ph ^ 1u, abort_flag)) return false;
            tc_fence_after();
            // Chunks half_sel*4 .. half_sel*4+3 are 16 consecutive columns.
            tmem_st_32x32b_x16_wait(lane_base + kACol0 + st * kAStageCols + half_sel * 16, outw);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.a_full[st]);
            return true;
        };

        // One stage at a time: issue its 8 row loads, then combine and store.  (Keeping
        // two stages in flight per thread, with the producers given more registers by
        // setmaxnreg, was measured slower and produced rare wrong A stages.)
        StageRegs R;
        bool ok = true;
        for (uint32_t it = 0; ok && it < total; ++it) ok = prefetch(it, R) && commit(it, R);
        if (!ok) signal_abort(s, a.err);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// NCHW FP16 -> corner pairs.  Entry (n, g, y, e), e = 0..W, is 32 bytes: the 8
// channels of offset group g at (y, e-1) followed by the same channels at (y, e),
// each half zero where the column is outside the image.  A bilinear sample whose
// left corner is column x0 (-1 <= x0 <= W-1) then reads its two corners of one
// row with a single aligned 32-byte load of entry x0+1.
// Grid: x over the H (W+1) entries of one group plane, y = group g, z strides over the
// images n (so no 64-bit division per thread).
__global__ void __launch_bounds__(256) regroup_pairs_kernel(const SplitInput<__half> in,
                                                             uint4 *__restrict__ out, int N, int H, int W) {
    allow_dependent_launch();  // the fused kernel may start its set-up
    const int entries = H * (W + 1);
    const int i = blockIdx.x * blockDim.x + threadIdx.x;  // entry index within the plane
    if (i >= entries) return;
    const int g = blockIdx.y;
    const int groups = gridDim.y;
    const int y = i / (W + 1);
    const int e = i - y * (W + 1);
    const int64_t plane = static_cast<int64_t>(H) * W;
    const __half zero = __float2half_rn(0.0f);
    for (int64_t n = blockIdx.z; n < N; n += gridDim.z) {
        const __half *src = in.channel(n, g * 8, plane) + static_cast<int64_t>(y) * W;
        uint32_t w[8];
#pragma unroll
        for (int half_sel = 0; half_sel < 2; ++half_sel) {
            const int x = e - 1 + half_sel;
            const bool in_row = x >= 0 && x < W;
            __half h[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) h[c] = in_row ? src[c * plane + x] : zero;
#pragma unroll
            for (int c = 0; c < 4; ++c) w[half_sel * 4 + c] = pack_half2(__halves2half2(h[2 * c], h[2 * c + 1]));
        }
        const int64_t o = ((n * groups + g) * entries + i) * 2;
        out[o] = make_uint4(w[0], w[1], w[2], w[3]);
        out[o + 1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
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
    if (static_cast<int64_t>(p.OG) * p.H * (p.W + 1) >= (int64_t{1} << 31)) return false;
    return true;
}

int fused_kblocks(const Params &p) {
    return (p.OG * p.KA + fused::kChunksPerStage - 1) / fused::kChunksPerStage;
}

size_t fused_workspace_bytes(const Params &p) {
    // corner pairs: N * (C/8) * H * (W+1) entries of 32 bytes
    const size_t bytes = static_cast<size_t>(p.N) * (p.C / 8) * p.H * (p.W + 1) * 32;
    return (bytes + 255) & ~static_cast<size_t>(255);
}

// Once per device (with that device current): opt the kernel into its shared
// memory size and look up the device address of the sticky error word.
cudaError_t fused_prepare_device(uint32_t **err_word) {
    for (const void *fn : {reinterpret_cast<const void *>(fused::fused_dcn_kernel<false>),
                           reinterpret_cast<const void *>(fused::fused_dcn_kernel<true>)}) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(fused::Smem) + 1024));
        if (e != cudaSuccess) return e;
        cudaFuncAttributes attr;
        e = cudaFuncGetAttributes(&attr, fn);
        if (e != cudaSuccess) return e;
        if (attr.maxThreadsPerBlock < fused::kThreads) return cudaErrorInvalidConfiguration;
    }
    cudaError_t e;
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, fused::g_error_word);
    if (e != cudaSuccess) return e;
    *err_word = static_cast<uint32_t *>(ptr);
    return cudaSuccess;
}

// NCHW FP16 -> corner pairs (the layout the fused kernel gathers from).
cudaError_t launch_regroup_c8(const Params &p, const SplitInput<__half> &input, void *workspace,
                              cudaStream_t stream) {
    const int entries = p.H * (p.W + 1);
    const dim3 grid(static_cast<unsigned>((entries + 255) / 256), static_cast<unsigned>(p.C / 8),
                    static_cast<unsigned>(p.N < 65535 ? p.N : 65535));
    fused::regroup_pairs_kernel<<<grid, 256, 0, stream>>>(input, static_cast<uint4 *>(workspace), p.N, p.H, p.W);
    return cudaGetLastError();
}

namespace {

fused::Args make_fused_args(const Params &p, const void *input_c8, const uint8_t *packed_w, const __half *bias,
                            __half *output, uint32_t *flag, uint32_t *err) {
    fused::Args a{};
    a.p = p;
    a.pairs = static_cast<const uint4 *>(input_c8);
    a.packed_w = packed_w;
    a.bias = bias;
    a.out = output;
    a.flag = flag;
    a.err = err;
    a.kb = fused_kblocks(p);
    a.nchunks = p.OG * p.KA;
    a.tiles_per_image = (p.out_plane + fused::BM - 1) / fused::BM;
    a.num_tiles = p.N * a.tiles_per_image;
    return a;
}

}  // namespace

// The fused gather + tcgen05 kernel on a regrouped input, one persistent CTA per SM.
cudaError_t launch_fused_grouped(const Params &p, const void *input_c8, const __half *offset,
                                 const __half *mask, const uint8_t *packed_w, const __half *bias,
                                 __half *output, uint32_t *flag, int sm_count, uint32_t *err,
                                 cudaStream_t stream) {
    using namespace fused;
    CUtensorMap tmap_off, tmap_msk;
    if (!make_plane_map(&tmap_off, offset, p.out_plane, 2 * p.OG * p.KA, p.N, kOffRows) ||
        !make_plane_map(&tmap_msk, mask, p.out_plane, p.OG * p.KA, p.N, kMaskRows))
        return cudaErrorInvalidValue;
    const Args a = make_fused_args(p, input_c8, packed_w, bias, output, flag, err);
    const int grid = a.num_tiles < sm_count ? a.num_tiles : sm_count;
    return launch_dependent(fused_dcn_kernel<false>, dim3(grid), dim3(kThreads), sizeof(Smem) + 1024, stream, tmap_off,
                            tmap_msk, a);
}

// The same kernel fed by the offset network's raw output [N][3*OG*KA][plane] and the two
// flows [N][2][plane] (OG even): offsets and masks are made inside the producers.
cudaError_t launch_fused_grouped_raw(const Params &p, const void *input_c8, const __half *raw,
                                     const __half *flow1, const __half *flow2, const uint8_t *packed_w,
                                     const __half *bias, __half *output, uint32_t *flag, int sm_count,
                                     uint32_t *err, cudaStream_t stream) {
    using namespace fused;
    CUtensorMap tmap_off, tmap_msk;
    const int raw_channels = 3 * p.OG * p.KA;
    if (!make_plane_map(&tmap_off, raw, p.out_plane, raw_channels, p.N, kOffRows) ||
        !make_plane_map(&tmap_msk, raw, p.out_plane, raw_channels, p.N, kMaskRows))
        return cudaErrorInvalidValue;
    Args a = make_fused_args(p, input_c8, packed_w, bias, output, flag, err);
    a.flow1 = flow1;
    a.flow2 = flow2;
    a.raw_mask_channel0 = 2 * p.OG * p.KA;
    const int grid = a.num_tiles < sm_count ? a.num_tiles : sm_count;
    return launch_dependent(fused_dcn_kernel<true>, dim3(grid), dim3(kThreads), sizeof(Smem) + 1024, stream, tmap_off,
                            tmap_msk, a);
}

}  // namespace dcn
