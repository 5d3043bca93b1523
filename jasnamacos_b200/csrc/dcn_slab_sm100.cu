// dcn_slab_sm100.cu -- fused FP16 DCNv2 for small images (the 64x64 tiles of the
// Jasna restoration pipeline): every deformable group's input is staged whole in
// shared memory and gathered from there.
//
// Same operator as dcn_fused_sm100.cu (bilinear sample * mask -> FP16 A operand in
// tensor memory -> tcgen05.mma against the weights -> bias, FP16, NCHW, Inf/NaN
// flag), organised for images whose per-group input plane fits in shared memory:
//
//   work unit = up to 4 consecutive 128-pixel tiles of one image (4 accumulators,
//               64 TMEM columns each, live across all deformable groups)
//   for each deformable group g (16 for Jasna):
//       the loader bulk-copies the group's zero-bordered input slab
//       ([H+2][W+2] x 8 channels FP16, 69,696 B for 64x64) and the group's slice
//       of the weights (5 K=16 blocks, 10 KB) into one of two shared buffers
//       for each tile of the unit:
//           the loader TMA-loads the tile's 18 offset and 9 mask rows of group g
//           12 producer warps sample the 9 taps (3 each) from the slab with
//           16-byte shared loads and store 9 chunks (+1 zero chunk) of A in TMEM
//           the MMA thread issues 5 MMAs (K = 80) into the tile's accumulator
//   4 epilogue warps drain each tile's accumulator after its last group.
//
// Batches too small to give every SM a unit (one image: 32 tiles on 148 SMs) split
// the deformable groups too: a unit then covers one tile and 1/s of the groups, its
// epilogue writes the FP32 partial sum to the workspace, and slab_reduce_kernel adds
// the s partials in a fixed order (bias, FP16, NCHW, Inf/NaN flag).  s depends only on
// the shape (slab_group_splits), so the result of a shape is the same on every run.
//
// Compared with gathering from global memory this trades the random 32-byte L1
// requests (one data-pipe wavefront per lane, ~500 cycles) for random 16-byte
// shared loads (~2.5 wavefronts per 8 lanes, ~30 cycles), and reads each input
// byte from L2 once per work unit instead of once per sample.
//
// Every mbarrier wait is bounded (kWaitLimitNs); a timeout sets the device error
// word, stops the CTA's warps, drains in-flight copies and MMAs and frees TMEM.
#include <cuda.h>
#include <cstdlib>
#include <string>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "dcn_common.cuh"

namespace dcn {

namespace slab {

constexpr int BM = 128;              // pixels per tile
constexpr int BN = 64;               // output channels
constexpr int kMaxTilesPerUnit = 4;  // accumulators kept in TMEM
constexpr int kTaps = 9;             // 3x3
constexpr int kChunks = 10;          // 9 taps + 1 zero chunk -> K = 80 = 5 MMAs of K = 16
constexpr int kMmasPerStage = kChunks / 2;
constexpr int kBBlockBytes = BN * 32;                     // one K=16 block, SW32 K-major: 64 rows x 32 B
constexpr int kBGroupBytes = kMmasPerStage * kBBlockBytes;  // 10 KB per deformable group
constexpr int kStages = 6;                                // (tile, group) stages in flight
constexpr int kOffRows = 2 * kTaps;                       // 18 offset rows per (tile, group)
constexpr int kMaskRows = kTaps;                          // 9 mask rows
constexpr uint32_t kStageTxBytes = (kOffRows + kMaskRows) * BM * 2;
constexpr uint32_t kFlowTxBytes = 2 * BM * 2;
constexpr int kProducerWarps = 12;  // 3 per TMEM lane quarter, 3 taps each
constexpr int kEpilogueWarps = 4;
constexpr int kThreads = (4 + kEpilogueWarps + kProducerWarps) * 32;  // 640
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kACol0 = kMaxTilesPerUnit * BN;  // 256: A stages after the accumulators
constexpr uint32_t kAStageCols = kChunks * 4;       // 40 columns per stage
constexpr uint32_t kIdleBackoffNs = 200;
constexpr int kMaxSlabBytes = 80 * 1024;            // two slabs + ~66 KB of fixed buffers fit 227 KB
static_assert(kACol0 + kStages * kAStageCols <= kTmemCols, "accumulators and A stages exceed TMEM");

// Shared memory: fixed part; the two slabs follow it (size depends on H, W).
struct __align__(1024) Smem {
    uint8_t b[2][kBGroupBytes];           // weight slices of the two buffered groups (256-aligned)
    __half off[kStages][kOffRows][BM];    // TMA boxes: offsets (or raw offset residues)
    __half msk[kStages][kMaskRows][BM];   // masks (or raw mask logits)
    __half flow[kStages][2][BM];          // (x, y) flow rows of the stage (raw-input form only)
    float bias[BN];
    int2 tap[kTaps];                      // {ky*DH, kx*DW}
    uint64_t grp_full[2];                 // slab + weights of a group landed
    uint64_t grp_empty[2];                // producers done with the slab, MMAs done with the weights
    uint64_t om_full[kStages];
    uint64_t om_empty[kStages];
    uint64_t a_full[kStages];
    uint64_t a_empty[kStages];
    uint64_t acc_full[kMaxTilesPerUnit];
    uint64_t acc_empty[kMaxTilesPerUnit];
    uint32_t tmem_base;
    int abort_flag;
};

struct Args {
    Params p;
    const uint8_t *slabs;      // [N][OG][H+2][W+2][8] FP16 (zero border), see regroup_slabs_kernel
    const uint8_t *packed_w;   // OG * kBGroupBytes, SW32 K-major blocks
    const __half *bias;
    __half *out;
    uint32_t *flag;
    uint32_t *err;
    int raw_mask_channel0;     // raw form: first mask-logit channel (2 * OG * KA)
    int slab_bytes;            // (H+2)(W+2)*16
    int tiles_per_image;
    int tiles_per_unit;        // 1..4
    int units_per_image;
    int splits;                // group ranges per tile set (1: no split)
    int groups_per_split;      // OG / splits
    int num_units;             // N * units_per_image * splits
    float *partial;            // splits > 1: [splits][N][BN][plane] FP32 partial sums
};

// Work unit u: image n, first tile t0, tile count mt, first deformable group g0.
struct Unit {
    int n, t0, mt, g0;
};

__device__ __forceinline__ Unit decode_unit(const Args &a, int u) {
    Unit w;
    const int j = u % a.splits;
    const int rest = u / a.splits;
    w.n = rest / a.units_per_image;
    w.t0 = (rest % a.units_per_image) * a.tiles_per_unit;
    w.mt = min(a.tiles_per_unit, a.tiles_per_image - w.t0);
    w.g0 = j * a.groups_per_split;
    return w;
}

__device__ __forceinline__ uint32_t pack_half2(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

__device__ __forceinline__ void signal_abort(Smem &s, uint32_t *err) {
    s.abort_flag = 1;
    atomicOr(err, kErrWaitTimeout);
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// Shared-memory descriptor of one K=16 slice of B stored K-major with the 32-byte
// swizzle: rows of 32 bytes, 8-row (256-byte) atoms; layout code 6 = SWIZZLE_32B.
__device__ __forceinline__ uint64_t make_sw32_kmajor_desc(uint32_t smem_byte_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(256u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(6u) << 61;
    return d;
}

// FromRaw = false: offsets and masks are inputs (the reference's DCN call).
// FromRaw = true: the inputs are the offset network's raw output and the two flows,
// transformed here as prepare_dcn_offsets_fp16 does (MetalShader.swift:817-839):
// offset = half(10*tanh(residue) + flow), mask = half(sigmoid(logit)); the flow is
// stored (x, y), dy channels take its y row, and deformable groups [0, OG/2) use
// flow1, the rest flow2.  tmap_flow1/2 are unused when FromRaw is false.
template <bool FromRaw>
__global__ void __launch_bounds__(kThreads, 1)
    slab_dcn_kernel(const __grid_constant__ CUtensorMap tmap_off, const __grid_constant__ CUtensorMap tmap_msk,
                    const __grid_constant__ CUtensorMap tmap_flow1, const __grid_constant__ CUtensorMap tmap_flow2,
                    const Args a) {
    extern __shared__ uint8_t smem_raw[];
    Smem &s = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
    uint8_t *slab_base = reinterpret_cast<uint8_t *>(&s) + ((sizeof(Smem) + 127) & ~size_t{127});
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const Params &p = a.p;
    volatile int *abort_flag = &s.abort_flag;
    const int slab_stride = (a.slab_bytes + 127) & ~127;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.grp_full[i], 1);
            mbar_init(&s.grp_empty[i], kProducerWarps + 1);
        }
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&s.om_full[i], 1);
            mbar_init(&s.om_empty[i], kProducerWarps);
            mbar_init(&s.a_full[i], kProducerWarps);
            mbar_init(&s.a_empty[i], 1);
        }
        for (int i = 0; i < kMaxTilesPerUnit; ++i) {
            mbar_init(&s.acc_full[i], 1);
            mbar_init(&s.acc_empty[i], kEpilogueWarps);
        }
        s.abort_flag = 0;
        fence_mbarrier_init();
    }
    if (threadIdx.x < kTaps) {
        const int ky = threadIdx.x / p.KW;
        s.tap[threadIdx.x] = make_int2(ky * p.DH, (static_cast<int>(threadIdx.x) - ky * p.KW) * p.DW);
    }
    if (warp == 1) {
        tmem_alloc(&s.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensor_map(&tmap_off);
        prefetch_tensor_map(&tmap_msk);
        if (FromRaw) {
            prefetch_tensor_map(&tmap_flow1);
            prefetch_tensor_map(&tmap_flow2);
        }
    }
    // Launched as a dependent of the regroup pre-pass: no global memory before this.
    grid_dependency_wait();
    if (a.splits > 1) allow_dependent_launch();  // the reduction pass may start its set-up
    if (threadIdx.x < BN) s.bias[threadIdx.x] = __half2float(a.bias[threadIdx.x]);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    // The zero chunk (K columns 72..79) of every A stage is written once here and
    // never again; the producers only store chunks 0..8.
    if (warp >= 8 && warp < 12) {
        const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp % 4) * 32) << 16);
        for (int st = 0; st < kStages; ++st)
            tmem_st_32x32b_x4(lane_base + kACol0 + st * kAStageCols + kTaps * 4, 0u, 0u, 0u, 0u);
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const int OG = p.OG;
    if (warp == 0) {
        // ------------------------------------------------------------ loader
        if (lane == 0) {
            uint32_t gi = 0, si = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.num_units && ok; u += gridDim.x) {
                const Unit w = decode_unit(a, u);
                const int n = w.n, t0 = w.t0, mt = w.mt;
                for (int g = w.g0; g < w.g0 + a.groups_per_split && ok; ++g, ++gi) {
                    const uint32_t gb = gi & 1u, gph = (gi >> 1) & 1u;
                    if (!mbar_wait_bounded(&s.grp_empty[gb], gph ^ 1u, abort_flag)) {
                        signal_abort(s, a.err);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&s.grp_full[gb], static_cast<uint32_t>(a.slab_bytes + kBGroupBytes));
                    const uint8_t *src = a.slabs + (static_cast<size_t>(n) * OG + g) * a.slab_bytes;
                    uint8_t *dst = slab_base + gb * slab_stride;
                    for (int off = 0; off < a.slab_bytes; off += 32768) {
                        const int bytes = min(32768, a.slab_bytes - off);
                        bulk_copy_g2s(dst + off, src + off, static_cast<uint32_t>(bytes), &s.grp_full[gb]);
                    }
                    bulk_copy_g2s(s.b[gb], a.packed_w + static_cast<size_t>(g) * kBGroupBytes, kBGroupBytes,
                                  &s.grp_full[gb]);
                    for (int t = 0; t < mt; ++t, ++si) {
                        const uint32_t st = si % kStages, ph = (si / kStages) & 1u;
                        if (!mbar_wait_bounded(&s.om_empty[st], ph ^ 1u, abort_flag)) {
                            signal_abort(s, a.err);
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&s.om_full[st], kStageTxBytes + (FromRaw ? kFlowTxBytes : 0u));
                        const int px0 = (t0 + t) * BM;
                        tma_load_3d(&s.off[st][0][0], &tmap_off, &s.om_full[st], px0, kOffRows * g, n);
                        tma_load_3d(&s.msk[st][0][0], &tmap_msk, &s.om_full[st], px0,
                                    (FromRaw ? a.raw_mask_channel0 : 0) + kMaskRows * g, n);
                        if (FromRaw)
                            tma_load_3d(&s.flow[st][0][0], g < OG / 2 ? &tmap_flow1 : &tmap_flow2, &s.om_full[st],
                                        px0, 0, n);
                    }
                }
            }
            // Drain every copy issued before leaving.
            for (uint32_t k = 0; k < 2 && k < gi; ++k) {
                const uint32_t last = gi - 1 - k;
                mbar_wait_bounded(&s.grp_full[last & 1u], (last >> 1) & 1u, nullptr);
            }
            for (uint32_t k = 0; k < kStages && k < si; ++k) {
                const uint32_t last = si - 1 - k;
                mbar_wait_bounded(&s.om_full[last % kStages], (last / kStages) & 1u, nullptr);
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t idesc = make_idesc_f16_f32(BM, BN);
            uint32_t gi = 0, si = 0;
            uint32_t acc_par = 0;  // bit t: parity of tile t's current accumulator phase (a register, not an array)
            uint64_t *last_bar = nullptr;
            uint32_t last_parity = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.num_units && ok; u += gridDim.x) {
                const Unit w = decode_unit(a, u);
                const int mt = w.mt, g_last = w.g0 + a.groups_per_split - 1;
                for (int g = w.g0; g <= g_last && ok; ++g, ++gi) {
                    const uint32_t gb = gi & 1u, gph = (gi >> 1) & 1u;
                    if (!mbar_wait_bounded(&s.grp_full[gb], gph, abort_flag)) {
                        signal_abort(s, a.err);
                        ok = false;
                        break;
                    }
                    const uint32_t b_base = smem_addr(s.b[gb]);
                    for (int t = 0; t < mt; ++t, ++si) {
                        if (g == w.g0) {
                            if (!mbar_wait_bounded(&s.acc_empty[t], ((acc_par >> t) & 1u) ^ 1u, abort_flag)) {
                                signal_abort(s, a.err);
                                ok = false;
                                break;
                            }
                        }
                        const uint32_t st = si % kStages, ph = (si / kStages) & 1u;
                        if (!mbar_wait_bounded(&s.a_full[st], ph, abort_flag)) {
                            signal_abort(s, a.err);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d_tmem = tmem + t * BN;
                        const uint32_t a_tmem = tmem + kACol0 + st * kAStageCols;
#pragma unroll
                        for (int kk = 0; kk < kMmasPerStage; ++kk) {
                            const uint64_t bdesc = make_sw32_kmajor_desc(b_base + kk * kBBlockBytes);
                            umma_f16_ts(d_tmem, a_tmem + kk * 8, bdesc, idesc, (g != w.g0 || kk != 0) ? 1u : 0u);
                        }
                        umma_commit(&s.a_empty[st]);
                        last_bar = &s.a_empty[st];
                        last_parity = ph;
                        if (g == g_last) {
                            umma_commit(&s.acc_full[t]);
                            last_bar = &s.acc_full[t];
                            last_parity = (acc_par >> t) & 1u;
                            acc_par ^= 1u << t;
                        }
                    }
                    if (!ok) break;
                    umma_commit(&s.grp_empty[gb]);  // the weights of this group are no longer read
                }
            }
            if (last_bar != nullptr) mbar_wait_bounded(last_bar, last_parity, nullptr);
        }
    } else if (warp < 4) {
        // warps 2-3: no role
    } else if (warp < 8) {
        // ---------------------------------------------------------- epilogue
        const int q = warp % 4;
        const int r = q * 32 + lane;
        uint32_t acc_par = 0;  // bit t: parity of tile t's next acc_full phase
        bool nonfinite = false;
        bool ok = true;
        for (int u = blockIdx.x; u < a.num_units && ok; u += gridDim.x) {
            const Unit w = decode_unit(a, u);
            const int n = w.n, t0 = w.t0, mt = w.mt;
            for (int t = 0; t < mt; ++t) {
                if (!mbar_wait_bounded(&s.acc_full[t], (acc_par >> t) & 1u, abort_flag, kIdleBackoffNs)) {
                    signal_abort(s, a.err);
                    ok = false;
                    break;
                }
                acc_par ^= 1u << t;
                tc_fence_after();
                uint32_t v[BN];
                const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + t * BN;
#pragma unroll
                for (int c = 0; c < BN; c += 16) tmem_ld_32x32b_x16(taddr + c, &v[c]);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.acc_empty[t]);
                const int px = (t0 + t) * BM + r;
                if (a.partial != nullptr) {
                    // Group split: this unit's FP32 partial sum; bias, FP16 and the flag
                    // come in slab_reduce_kernel.
                    if (px < p.out_plane) {
                        const int split = w.g0 / a.groups_per_split;
                        float *dst = a.partial +
                                     ((static_cast<int64_t>(split) * p.N + n) * BN) * p.out_plane + px;
#pragma unroll
                        for (int oc = 0; oc < BN; ++oc)
                            dst[static_cast<int64_t>(oc) * p.out_plane] = __uint_as_float(v[oc]);
                    }
                } else if (px < p.out_plane) {
                    __half *dst = a.out + output_index(p, n, 0, px);
#pragma unroll
                    for (int oc = 0; oc < BN; oc += 4) {
                        const float4 bq = *reinterpret_cast<const float4 *>(&s.bias[oc]);
                        const float bb[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const __half h = __float2half_rn(__uint_as_float(v[oc + j]) + bb[j]);
                            nonfinite |= __hisinf(h) != 0 || __hisnan(h);
                            dst[static_cast<size_t>(oc + j) * p.out_plane] = h;
                        }
                    }
                }
            }
        }
        if (a.flag != nullptr && __any_sync(0xffffffffu, nonfinite) && lane == 0)
            atomicOr(a.flag, DCN_FLAG_NONFINITE);
    } else {
        // --------------------------------------------------------- producers
        const int pw = warp - 8;       // 0..11
        const int q = warp % 4;        // TMEM lane quarter
        const int tap0 = (pw / 4) * 3;  // taps tap0..tap0+2
        const int r = q * 32 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const int sw = p.W + 2;  // slab row stride in positions
        const uint32_t slab0 = smem_addr(slab_base);
        // This warp's taps as float offsets (ky*DH, kx*DW): integer-valued, so adding
        // them to the pixel's integer base in FP32 is exact, as in the reference.  The slab
        // kernel takes 3x3 kernels only, so the warp's three taps tap0..tap0+2 are one kernel
        // row: a single ky*DH and kx*DW for kx = 0, 1, 2.
        const float tyf = static_cast<float>(s.tap[tap0].x);
        float txf[3];
#pragma unroll
        for (int i = 0; i < 3; ++i) txf[i] = static_cast<float>(s.tap[tap0 + i].y);
        uint32_t gi = 0, si = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < a.num_units && ok; u += gridDim.x) {
            const Unit w = decode_unit(a, u);
            const int t0 = w.t0, mt = w.mt;
            // Per tile of the unit: this pixel's integer sampling base (oy*SH - PH,
            // ox*SW - PW) as floats, and whether the pixel exists (its samples are
            // skipped, and its A row left zero, when it is past the output plane).
            float bfy[kMaxTilesPerUnit], bfx[kMaxTilesPerUnit];
            bool tvalid[kMaxTilesPerUnit];
#pragma unroll
            for (int t = 0; t < kMaxTilesPerUnit; ++t) {
                const int px = (t0 + t) * BM + r;
                tvalid[t] = t < mt && px < p.out_plane;
                const int oy = tvalid[t] ? px / p.WO : 0;
                const int ox = tvalid[t] ? px - oy * p.WO : 0;
                bfy[t] = static_cast<float>(oy * p.SH - p.PH);
                bfx[t] = static_cast<float>(ox * p.SW - p.PW);
            }
            for (int g = 0; g < a.groups_per_split && ok; ++g, ++gi) {
                const uint32_t gb = gi & 1u, gph = (gi >> 1) & 1u;
                if (!mbar_wait_bounded(&s.grp_full[gb], gph, abort_flag)) {
                    ok = false;
                    break;
                }
                const uint32_t slab = slab0 + gb * slab_stride;
#pragma unroll
                for (int t = 0; t < kMaxTilesPerUnit; ++t) {
                    if (t >= mt) break;
                    const uint32_t st = si % kStages, ph = (si / kStages) & 1u;
                    ++si;
                    const bool valid = tvalid[t];
                    if (!mbar_wait_bounded(&s.om_full[st], ph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    float fy[3], fx[3];
                    __half m[3];
                    uint32_t base_addr[3];
                    bool in[3];
#pragma unroll
                    for (int i = 0; i < 3; ++i) {
                        const int k = tap0 + i;
                        float off_y = __half2float(s.off[st][2 * k][r]);
                        float off_x = __half2float(s.off[st][2 * k + 1][r]);
                        __half mk = s.msk[st][k][r];
                        if (FromRaw) {
                            off_y = raw_offset(off_y, __half2float(s.flow[st][1][r]));
                            off_x = raw_offset(off_x, __half2float(s.flow[st][0][r]));
                            mk = raw_mask(__half2float(mk));
                        }
                        const float y = (bfy[t] + tyf) + off_y;
                        const float x = (bfx[t] + txf[i]) + off_x;
                        m[i] = mk;
                        const int y0 = __float2int_rd(y);
                        const int x0 = __float2int_rd(x);
                        fy[i] = y - static_cast<float>(y0);
                        fx[i] = x - static_cast<float>(x0);
                        // Padded slab: rows/columns -1 and H/W are zeros, so a sample is
                        // either fully inside [-1, H-1] x [-1, W-1] or contributes zero.
                        in[i] = valid && static_cast<unsigned>(y0 + 1) <= static_cast<unsigned>(p.H) &&
                                static_cast<unsigned>(x0 + 1) <= static_cast<unsigned>(p.W);
                        base_addr[i] = slab + static_cast<uint32_t>(((y0 + 1) * sw + (x0 + 1)) * 16);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.om_empty[st]);

                    uint32_t outw[3][4];
#pragma unroll
                    for (int i = 0; i < 3; ++i) {
                        if (in[i]) {
                            const uint4 c00 = lds128(base_addr[i]);
                            const uint4 c01 = lds128(base_addr[i] + 16);
                            const uint4 c10 = lds128(base_addr[i] + sw * 16);
                            const uint4 c11 = lds128(base_addr[i] + sw * 16 + 16);
                            // The four bilinear weights, mask folded in, in packed FP16 arithmetic:
                            // (fy, fx) rounded to FP16, (1-fy, 1-fx), then (m(1-fy), m fy) and the
                            // pairs (top-left, top-right), (bottom-left, bottom-right).
                            const __half2 fyx = __floats2half2_rn(fy[i], fx[i]);
                            const __half2 hyx = __hsub2(__float2half2_rn(1.0f), fyx);
                            const __half2 my = __hmul2(__half2half2(m[i]), __lows2half2(hyx, fyx));
                            const __half2 xx = __highs2half2(hyx, fyx);
                            const __half2 wt = __hmul2(__low2half2(my), xx);
                            const __half2 wb = __hmul2(__high2half2(my), xx);
                            const __half2 w00 = __low2half2(wt), w01 = __high2half2(wt);
                            const __half2 w10 = __low2half2(wb), w11 = __high2half2(wb);
                            const __half2 *h00 = reinterpret_cast<const __half2 *>(&c00);
                            const __half2 *h01 = reinterpret_cast<const __half2 *>(&c01);
                            const __half2 *h10 = reinterpret_cast<const __half2 *>(&c10);
                            const __half2 *h11 = reinterpret_cast<const __half2 *>(&c11);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                __half2 acc = __hmul2(w00, h00[e]);
                                acc = __hfma2(w01, h01[e], acc);
                                acc = __hfma2(w10, h10[e], acc);
                                acc = __hfma2(w11, h11[e], acc);
                                outw[i][e] = pack_half2(acc);
                            }
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) outw[i][e] = 0u;
                        }
                    }
                    if (!mbar_wait_bounded(&s.a_empty[st], ph ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    tmem_st_32x32b_x12_wait(lane_base + kACol0 + st * kAStageCols + tap0 * 4, outw);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.a_full[st]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.grp_empty[gb]);  // done reading this slab
            }
        }
        if (!ok) signal_abort(s, a.err);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// NCHW FP16 -> zero-bordered slabs [N][C/8][H+2][W+2][8]: slab (n, g) holds the 8
// channels of deformable group g at every position, 16 bytes per position, with a
// one-pixel ring of zeros so bilinear corners just outside the image read zero.
// Grid: x over the (H+2)(W+2) padded positions of one slab, y = group g, z strides
// over the images n (so no 64-bit division per thread).
__global__ void __launch_bounds__(256) regroup_slabs_kernel(const SplitInput<__half> in, uint4 *__restrict__ out,
                                                             int N, int H, int W) {
    allow_dependent_launch();  // the slab kernel may start its set-up
    const int sw = W + 2;
    const int positions = (H + 2) * sw;
    const int pos = blockIdx.x * blockDim.x + threadIdx.x;
    if (pos >= positions) return;
    const int g = blockIdx.y;
    const int groups = gridDim.y;
    const int py = pos / sw;
    const int y = py - 1, x = pos - py * sw - 1;
    const bool inside = y >= 0 && y < H && x >= 0 && x < W;
    const int64_t plane = static_cast<int64_t>(H) * W;
    for (int64_t n = blockIdx.z; n < N; n += gridDim.z) {
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (inside) {
            const __half *src = in.channel(n, g * 8, plane) + static_cast<int64_t>(y) * W + x;
            __half h[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) h[c] = src[c * plane];
            o.x = pack_half2(__halves2half2(h[0], h[1]));
            o.y = pack_half2(__halves2half2(h[2], h[3]));
            o.z = pack_half2(__halves2half2(h[4], h[5]));
            o.w = pack_half2(__halves2half2(h[6], h[7]));
        }
        out[(n * groups + g) * positions + pos] = o;
    }
}

// Group split, second pass: out[n][oc][px] = FP16(bias[oc] + partial[0] + ... +
// partial[s-1]) summed in split order, four pixels per thread, with the Inf/NaN flag.
__global__ void __launch_bounds__(256) slab_reduce_kernel(Params p, const float *__restrict__ partial, int splits,
                                                           const __half *__restrict__ bias, __half *__restrict__ out,
                                                           uint32_t *__restrict__ flag) {
    grid_dependency_wait();  // the slab kernel's partial sums
    const int64_t per_split = static_cast<int64_t>(p.N) * BN * p.out_plane;
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    bool bad = false;
    if (i < per_split) {
        const int64_t row = i / p.out_plane;  // n * BN + oc
        const int px = static_cast<int>(i - row * p.out_plane);
        const int oc = static_cast<int>(row % BN);
        const int64_t n = row / BN;
        float4 acc = *reinterpret_cast<const float4 *>(partial + i);
        for (int j = 1; j < splits; ++j) {
            const float4 v = *reinterpret_cast<const float4 *>(partial + j * per_split + i);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const float b = __half2float(bias[oc]);
        const __half h[4] = {__float2half_rn(acc.x + b), __float2half_rn(acc.y + b), __float2half_rn(acc.z + b),
                             __float2half_rn(acc.w + b)};
        __half *dst = out + output_index(p, n, oc, px);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            bad |= __hisinf(h[k]) != 0 || __hisnan(h[k]);
            dst[k] = h[k];
        }
    }
    if (flag != nullptr && __any_sync(0xffffffffu, bad) && (threadIdx.x % 32) == 0) atomicOr(flag, DCN_FLAG_NONFINITE);
}

// The same transform, four source columns per thread: 8-byte loads of 4 consecutive
// pixels from each of the group's 8 channel planes, transposed in registers into four
// 16-byte slab positions.  Needs W % 4 == 0 and 8-byte aligned channel planes.  Thread
// j < W/4 of padded row py writes positions 4j+1 .. 4j+4; thread j == W/4 writes the
// two border columns 0 and W+1; the border rows 0 and H+1 are all zeros.
template <int kBlock, int kMinBlocks>
__global__ void __launch_bounds__(kBlock, kMinBlocks) regroup_slabs_x4_kernel(const SplitInput<__half> in, uint4 *__restrict__ out,
                                                                int N, int H, int W) {
    allow_dependent_launch();  // the slab kernel may start its set-up
    const int per_row = W / 4 + 1;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (H + 2) * per_row) return;
    const int g = blockIdx.y;
    const int groups = gridDim.y;
    const int py = t / per_row;
    const int j = t - py * per_row;
    const int sw = W + 2;
    const int positions = (H + 2) * sw;
    const int64_t plane = static_cast<int64_t>(H) * W;
    const bool interior_row = py >= 1 && py <= H;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int64_t n = blockIdx.z; n < N; n += gridDim.z) {
        uint4 *row = out + (n * groups + g) * positions + static_cast<int64_t>(py) * sw;
        if (j == W / 4) {
            row[0] = zero;
            row[W + 1] = zero;
            continue;
        }
        uint4 o[4] = {zero, zero, zero, zero};
        if (interior_row) {
            const __half *src = in.channel(n, g * 8, plane) + static_cast<int64_t>(py - 1) * W + 4 * j;
            uint2 v[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) v[c] = *reinterpret_cast<const uint2 *>(src + c * plane);
            // v[c] holds pixels 4j..4j+3 of channel c as half pairs (x, y); position i
            // needs channel pairs (0,1) (2,3) (4,5) (6,7) of pixel i.
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int w = i >> 1;
                const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;  // high or low halves
                uint32_t r[4];
#pragma unroll
                for (int c2 = 0; c2 < 4; ++c2) {
                    const uint32_t a = w ? v[2 * c2].y : v[2 * c2].x;
                    const uint32_t b = w ? v[2 * c2 + 1].y : v[2 * c2 + 1].x;
                    r[c2] = __byte_perm(a, b, sel);
                }
                o[i] = make_uint4(r[0], r[1], r[2], r[3]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) row[4 * j + 1 + i] = o[i];
    }
}

// The same transform for large batches, with whole-sector stores.  Item (py, j < W/4) holds
// positions py*sw + 4j + 1 .. + 4, item (py, W/4) positions py*sw + W + 1 and the next one (column
// 0 of row py + 1), and item 0 position 0 as well, so the items of a block cover one contiguous
// range of the slab.  Each block assembles its range in shared memory, then writes it with
// consecutive 16-byte stores (the transposed values of one thread are 64 bytes apart otherwise,
// and each store instruction would fill half sectors).
template <int kBlock>
__global__ void __launch_bounds__(kBlock) regroup_slabs_staged_kernel(const SplitInput<__half> in,
                                                                       uint4 *__restrict__ out, int N, int H, int W) {
    __shared__ uint4 stage[kBlock * 4 + 1];
    allow_dependent_launch();  // the slab kernel may start its set-up
    const int per_row = W / 4 + 1;
    const int items = (H + 2) * per_row;
    const int sw = W + 2;
    const int positions = (H + 2) * sw;
    const int g = blockIdx.y;
    const int groups = gridDim.y;
    const int t0 = blockIdx.x * kBlock;
    const int t = t0 + static_cast<int>(threadIdx.x);
    const auto first_position = [&](int it) {
        const int r = it / per_row, c = it - r * per_row;
        return it == 0 ? 0 : r * sw + (c < W / 4 ? 4 * c + 1 : W + 1);
    };
    const int p_begin = first_position(t0);
    const int p_end = t0 + kBlock < items ? first_position(t0 + kBlock) : positions;
    const int py = t / per_row;
    const int j = t - py * per_row;
    const int64_t plane = static_cast<int64_t>(H) * W;
    const bool interior_row = py >= 1 && py <= H;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int64_t n = blockIdx.z; n < N; n += gridDim.z) {
        if (t < items) {
            if (j == W / 4) {
                const int q = py * sw + W + 1 - p_begin;
                stage[q] = zero;
                if (py + 1 < H + 2) stage[q + 1] = zero;
            } else {
                uint4 o[4] = {zero, zero, zero, zero};
                if (interior_row) {
                    const __half *src = in.channel(n, g * 8, plane) + static_cast<int64_t>(py - 1) * W + 4 * j;
                    uint2 v[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) v[c] = *reinterpret_cast<const uint2 *>(src + c * plane);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int w = i >> 1;
                        const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;  // high or low halves
                        uint32_t r[4];
#pragma unroll
                        for (int c2 = 0; c2 < 4; ++c2) {
                            const uint32_t a = w ? v[2 * c2].y : v[2 * c2].x;
                            const uint32_t b = w ? v[2 * c2 + 1].y : v[2 * c2 + 1].x;
                            r[c2] = __byte_perm(a, b, sel);
                        }
                        o[i] = make_uint4(r[0], r[1], r[2], r[3]);
                    }
                }
                const int q = py * sw + 4 * j + 1 - p_begin;
                if (t == 0) stage[q - 1] = zero;  // position 0
#pragma unroll
                for (int i = 0; i < 4; ++i) stage[q + i] = o[i];
            }
        }
        __syncthreads();
        uint4 *dst = out + (n * groups + g) * positions;
        for (int k = p_begin + static_cast<int>(threadIdx.x); k < p_end; k += kBlock) dst[k] = stage[k - p_begin];
        __syncthreads();  // the stage is refilled for the next image
    }
}

// Weights -> per-group SW32 K-major B blocks.  Group g, block kk (K = 16: taps 2kk,
// 2kk+1 x 8 channels), output channel row n (0..63), 16-byte physical chunk pc:
// logical chunk c = pc ^ ((n >> 2) & 1), tap = 2kk + c (tap 9 is zero), channel
// ic = 8g + e.  Byte ((g*5 + kk)*64 + n)*32 + pc*16 + 2e.
template <typename T>
__global__ void prepack_slab_kernel(const T *__restrict__ src, int layout, __half *__restrict__ dst, int OG, int cpg,
                                    int KA, int OC) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // destination half
    const int64_t total = static_cast<int64_t>(OG) * kBGroupBytes / 2;
    if (i >= total) return;
    const int e = static_cast<int>(i % 8);
    const int pc = static_cast<int>((i / 8) % 2);
    const int n = static_cast<int>((i / 16) % 64);
    const int kk = static_cast<int>((i / (16 * 64)) % kMmasPerStage);
    const int g = static_cast<int>(i / (16 * 64 * kMmasPerStage));
    const int c = pc ^ ((n >> 2) & 1);
    const int tap = 2 * kk + c;
    float v = 0.0f;
    if (tap < kTaps) {
        const int ic = g * 8 + e;
        const int64_t idx = layout == DCN_WEIGHT_OIHW ? (static_cast<int64_t>(n) * cpg + ic) * KA + tap
                                                      : (static_cast<int64_t>(ic) * KA + tap) * OC + n;
        v = static_cast<float>(src[idx]);
    }
    dst[i] = __float2half_rn(v);
}

}  // namespace slab

// Shapes the slab kernel takes: the fused-kernel class (1 conv group, 64 output
// channels, 8 channels per deformable group) with a 3x3 kernel, an output plane
// that is a multiple of 8 pixels, and a per-group input slab that fits twice in
// shared memory next to the fixed buffers.
bool slab_supported(const Params &p) {
    if (p.G != 1 || p.OC != slab::BN || p.cpog != 8 || p.KH != 3 || p.KW != 3) return false;
    if (p.out_plane % 8 != 0) return false;
    const int64_t slab_bytes = static_cast<int64_t>(p.H + 2) * (p.W + 2) * 16;
    if (slab_bytes > slab::kMaxSlabBytes) return false;
    if (static_cast<int64_t>(p.N) * p.OG * slab_bytes >= (int64_t{1} << 40)) return false;
    return true;
}

namespace {

// B200 SM count: the unit count the group split aims for.  A fixed number rather than
// the device's, so that the split (and with it the summation order and the workspace
// size) depends on the shape alone.
constexpr int kSplitTargetUnits = 148;

size_t slab_slabs_bytes(const Params &p) {
    const size_t bytes = static_cast<size_t>(p.N) * p.OG * (p.H + 2) * (p.W + 2) * 16;
    return (bytes + 255) & ~size_t{255};
}

}  // namespace

// DCN_B200_GROUP_SPLIT=0 turns the split off for the process (read once), for callers
// that need an image's result to be bit-identical whatever batch it is computed in.
bool group_split_allowed() {
    static const bool allowed = [] {
        const char *v = std::getenv("DCN_B200_GROUP_SPLIT");
        return !(v != nullptr && std::string(v) == "0");
    }();
    return allowed;
}

// Deformable-group split of a shape: the largest power of two s <= OG dividing OG with
// (tiles in the batch) x s <= kSplitTargetUnits; 1 for batches that already fill the GPU.
int slab_group_splits(const Params &p) {
    if (!group_split_allowed()) return 1;
    const int64_t tiles = static_cast<int64_t>(p.N) * ((p.out_plane + slab::BM - 1) / slab::BM);
    int splits = 1;
    while (splits * 2 <= p.OG && p.OG % (splits * 2) == 0 && tiles * splits * 2 <= kSplitTargetUnits) splits *= 2;
    return splits;
}

size_t slab_workspace_bytes(const Params &p) {
    const int splits = slab_group_splits(p);
    size_t bytes = slab_slabs_bytes(p);
    if (splits > 1) bytes += static_cast<size_t>(splits) * p.N * slab::BN * p.out_plane * sizeof(float);
    return bytes;
}

size_t slab_packed_weight_bytes(const Params &p) { return static_cast<size_t>(p.OG) * slab::kBGroupBytes; }

size_t slab_smem_bytes(const Params &p) {
    const int slab_bytes = (p.H + 2) * (p.W + 2) * 16;
    return 1024 + ((sizeof(slab::Smem) + 127) & ~size_t{127}) + 2 * static_cast<size_t>((slab_bytes + 127) & ~127);
}

cudaError_t slab_prepare_device() {
    // Opt in to the largest dynamic shared memory any supported shape needs.
    const int max_slab = (slab::kMaxSlabBytes + 127) & ~127;
    const size_t smem = 1024 + ((sizeof(slab::Smem) + 127) & ~size_t{127}) + 2 * static_cast<size_t>(max_slab);
    cudaError_t e = cudaFuncSetAttribute(slab::slab_dcn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(slab::slab_dcn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem));
}

cudaError_t launch_regroup_slabs(const Params &p, const SplitInput<__half> &input, void *workspace,
                                 cudaStream_t stream) {
    const unsigned images = static_cast<unsigned>(p.N < 65535 ? p.N : 65535);
    const int64_t plane = static_cast<int64_t>(p.H) * p.W;
    const bool vec = p.W % 4 == 0 && plane % 4 == 0 && (reinterpret_cast<uintptr_t>(input.first) & 7u) == 0 &&
                     (input.second == nullptr || (reinterpret_cast<uintptr_t>(input.second) & 7u) == 0);
    if (vec) {
        const int threads = (p.H + 2) * (p.W / 4 + 1);
        if (slab_group_splits(p) > 1) {
            // Small batches: 128-thread blocks of at most 32 registers, one of which fits on an
            // SM next to a slab kernel block (640 threads x 96 registers), so the slab kernel's
            // blocks, launched as programmatic dependents, become resident and do their set-up
            // while the pre-pass still runs.
            const dim3 grid(static_cast<unsigned>((threads + 127) / 128), static_cast<unsigned>(p.C / 8), images);
            slab::regroup_slabs_x4_kernel<128, 16><<<grid, 128, 0, stream>>>(input, static_cast<uint4 *>(workspace),
                                                                             p.N, p.H, p.W);
        } else {
            const dim3 grid(static_cast<unsigned>((threads + 255) / 256), static_cast<unsigned>(p.C / 8), images);
            slab::regroup_slabs_staged_kernel<256><<<grid, 256, 0, stream>>>(input, static_cast<uint4 *>(workspace),
                                                                             p.N, p.H, p.W);
        }
    } else {
        const int positions = (p.H + 2) * (p.W + 2);
        const dim3 grid(static_cast<unsigned>((positions + 255) / 256), static_cast<unsigned>(p.C / 8), images);
        slab::regroup_slabs_kernel<<<grid, 256, 0, stream>>>(input, static_cast<uint4 *>(workspace), p.N, p.H, p.W);
    }
    return cudaGetLastError();
}

cudaError_t launch_prepack_slab(const Params &p, const void *src, dcn_dtype src_dtype, int layout, void *dst,
                                cudaStream_t stream) {
    const int64_t total = static_cast<int64_t>(p.OG) * slab::kBGroupBytes / 2;
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    if (src_dtype == DCN_DTYPE_F32)
        slab::prepack_slab_kernel<float><<<blocks, 256, 0, stream>>>(static_cast<const float *>(src), layout,
                                                                     static_cast<__half *>(dst), p.OG, p.cpg,
                                                                     p.KA, p.OC);
    else
        slab::prepack_slab_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<const __half *>(src), layout,
                                                                      static_cast<__half *>(dst), p.OG, p.cpg,
                                                                      p.KA, p.OC);
    return cudaGetLastError();
}

namespace fused {
bool make_plane_map(CUtensorMap *map, const void *base, int64_t plane, int channels, int batch, int rows);
}

namespace {

slab::Args make_slab_args(const Params &p, const void *slabs, const uint8_t *packed_w, const __half *bias,
                          __half *output, uint32_t *flag, int sm_count, uint32_t *err) {
    using namespace slab;
    Args a;
    a.p = p;
    a.slabs = static_cast<const uint8_t *>(slabs);
    a.packed_w = packed_w;
    a.bias = bias;
    a.out = output;
    a.flag = flag;
    a.err = err;
    a.raw_mask_channel0 = 2 * p.OG * p.KA;
    a.slab_bytes = (p.H + 2) * (p.W + 2) * 16;
    a.tiles_per_image = (p.out_plane + BM - 1) / BM;
    // Up to 4 tiles per work unit (each unit reads every group's slab once); fewer
    // when that would leave SMs idle.
    a.splits = slab_group_splits(p);
    a.groups_per_split = p.OG / a.splits;
    int tpu = kMaxTilesPerUnit;
    while (tpu > 1 && (a.splits > 1 ||
                       static_cast<int64_t>(p.N) * ((a.tiles_per_image + tpu - 1) / tpu) < 2 * sm_count))
        tpu /= 2;
    a.tiles_per_unit = tpu;
    a.units_per_image = (a.tiles_per_image + tpu - 1) / tpu;
    a.num_units = p.N * a.units_per_image * a.splits;
    a.partial = a.splits > 1
                    ? reinterpret_cast<float *>(const_cast<uint8_t *>(a.slabs) + slab_slabs_bytes(p))
                    : nullptr;
    return a;
}

// The second pass of a group-split launch (nothing when the shape is not split).
cudaError_t launch_split_reduce(const Params &p, const slab::Args &a, cudaStream_t stream) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || a.splits == 1) return e;
    const int64_t quads = static_cast<int64_t>(p.N) * slab::BN * p.out_plane / 4;
    return launch_dependent(slab::slab_reduce_kernel, dim3(static_cast<unsigned>((quads + 255) / 256)), dim3(256), 0,
                            stream, p, static_cast<const float *>(a.partial), a.splits, a.bias, a.out, a.flag);
}

}  // namespace

// Launch plan of the slab path (dcn_forward_f16_plan).
void slab_plan(const Params &p, int sm_count, dcn_plan *out) {
    const slab::Args a = make_slab_args(p, nullptr, nullptr, nullptr, nullptr, nullptr, sm_count, nullptr);
    out->path = DCN_PATH_SLAB_TC;
    out->group_splits = a.splits;
    out->tiles_per_unit = a.tiles_per_unit;
    out->launches = a.splits > 1 ? 3 : 2;
    out->grid = a.num_units < sm_count ? a.num_units : sm_count;
    out->prepass_images = p.N;
}

cudaError_t launch_slab_grouped(const Params &p, const void *slabs, const __half *offset, const __half *mask,
                                const uint8_t *packed_w, const __half *bias, __half *output, uint32_t *flag,
                                int sm_count, uint32_t *err, cudaStream_t stream) {
    using namespace slab;
    CUtensorMap tmap_off, tmap_msk;
    if (!fused::make_plane_map(&tmap_off, offset, p.out_plane, 2 * p.OG * p.KA, p.N, kOffRows) ||
        !fused::make_plane_map(&tmap_msk, mask, p.out_plane, p.OG * p.KA, p.N, kMaskRows))
        return cudaErrorInvalidValue;
    const Args a = make_slab_args(p, slabs, packed_w, bias, output, flag, sm_count, err);
    const int grid = a.num_units < sm_count ? a.num_units : sm_count;
    cudaError_t e = launch_dependent(slab_dcn_kernel<false>, dim3(grid), dim3(kThreads), slab_smem_bytes(p), stream,
                                     tmap_off, tmap_msk, tmap_off, tmap_msk, a);
    if (e != cudaSuccess) return e;
    return launch_split_reduce(p, a, stream);
}

// raw: [N][3*OG*KA][plane] (offset residues, then mask logits); flow1/flow2: [N][2][plane].
cudaError_t launch_slab_grouped_raw(const Params &p, const void *slabs, const __half *raw, const __half *flow1,
                                    const __half *flow2, const uint8_t *packed_w, const __half *bias,
                                    __half *output, uint32_t *flag, int sm_count, uint32_t *err,
                                    cudaStream_t stream) {
    using namespace slab;
    CUtensorMap tmap_off, tmap_msk, tmap_f1, tmap_f2;
    const int raw_channels = 3 * p.OG * p.KA;
    if (!fused::make_plane_map(&tmap_off, raw, p.out_plane, raw_channels, p.N, kOffRows) ||
        !fused::make_plane_map(&tmap_msk, raw, p.out_plane, raw_channels, p.N, kMaskRows) ||
        !fused::make_plane_map(&tmap_f1, flow1, p.out_plane, 2, p.N, 2) ||
        !fused::make_plane_map(&tmap_f2, flow2, p.out_plane, 2, p.N, 2))
        return cudaErrorInvalidValue;
    const Args a = make_slab_args(p, slabs, packed_w, bias, output, flag, sm_count, err);
    const int grid = a.num_units < sm_count ? a.num_units : sm_count;
    cudaError_t e = launch_dependent(slab_dcn_kernel<true>, dim3(grid), dim3(kThreads), slab_smem_bytes(p), stream,
                                     tmap_off, tmap_msk, tmap_f1, tmap_f2, a);
    if (e != cudaSuccess) return e;
    return launch_split_reduce(p, a, stream);
}

}  // namespace dcn
