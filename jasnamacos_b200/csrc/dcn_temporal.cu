// dcn_temporal.cu -- the temporal preparation that feeds the DCN in the Jasna recurrence.
//
// Replaces MetalDeformConv.runTemporalPreparation (Sources/JasnaMetalPoC/MetalRunner.swift:510-582),
// which runs two Metal kernels (MetalShader.swift:736-813):
//   accumulate_second_order_flow_fp16: flow2 = half(flow1 + warp(previous_flow, flow1)), or 0;
//   assemble_temporal_alignment_fp16:  conditions = [warp(feat_prop, flow1), feat_current,
//                                      warp(feat_n2, flow2), flow1, flow2] (196 channels, the
//                                      offset network's input) and deform_input = [feat_prop,
//                                      feat_n2] (the DCN's input).
// Here it is one kernel over a batch of frames: every thread owns one pixel and a slice of the
// 64 feature channels, computes the pixel's second-order flow itself (two bilinear samples of the
// previous flow, rounded to FP16 as the reference stores it) and then warps its channels of both
// feature maps with the two flows, so flow2 is never read back.  Frames whose channel slices fit
// in shared memory (Jasna's 64x64 tiles) stage them there first (temporal_prepare_staged_kernel);
// larger frames gather from global memory (temporal_prepare_kernel).  deform_input is optional:
// the DCN entry points take the two feature tensors directly (dcn_io.input_second), which makes
// the concatenation copy unnecessary.  The sampling arithmetic is the reference's (`sample_fp16`,
// MetalShader.swift:52-74, and the CPU check's `sampleZero`, JasnaCLI.swift:213-225) with one
// IEEE rounding per operation, so results equal the CPU restatement bit for bit.
#include <cooperative_groups.h>
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
    uint4 *slabs;  // the deform input as the DCN's slabs [N][16][H+2][W+2][8] (16 B per position), or null
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

// ---- frames whose channel slices fit in shared memory ------------------------------
// Two launches.  second_order_flow_kernel computes every pixel's second-order flow once per frame
// (with the global-memory sampling above) and writes it and the four flow channels of the
// conditions.  temporal_prepare_staged_kernel, its programmatic dependent, runs one block per
// (frame, map, slice of 4 channels), map 0 warping feat_prop by flow1 and map 1 feat_n2 by flow2:
// it copies its 4 planes into the deform input (and, for map 0, feat_current's into the
// conditions) with 16-byte accesses, stages its 4 channels as a channel-interleaved slab
// [(H+2)(W+2)] with a one-pixel ring of zeros (8 bytes per position), and (map 1 only) then waits
// for the second-order flow; every bilinear corner of 4 channels is then one 8-byte shared-memory
// load instead of four scattered 2-byte global loads.
// The sampling arithmetic is the same as above (out-of-slab corners read the zeros the reference
// reads), so both forms give the same bits.
constexpr int kTsThreads = 256;
constexpr int kTsSlice = 4;
constexpr int kTsSlices = kTpChannels / kTsSlice;
constexpr int kTsBytesPerPosition = 8;
constexpr int kTsStage = 4;  // staged positions per thread in flight
static_assert(kTsSlice == 4, "the staged kernel's gathers hold 4 channels per 8-byte position");

struct SlabCorners {
    int idx;  // top-left corner in the ring-padded slab, valid when in
    bool in;  // all four corners lie in the padded slab (else every corner is outside the frame)
    float ly, lx;
};

__device__ __forceinline__ SlabCorners slab_corners(float y, float x, int H, int W) {
    const int y0 = __float2int_rd(y), x0 = __float2int_rd(x);
    SlabCorners c;
    c.ly = __fsub_rn(y, static_cast<float>(y0));
    c.lx = __fsub_rn(x, static_cast<float>(x0));
    c.in = static_cast<unsigned>(y0) + 1u <= static_cast<unsigned>(H) &&
           static_cast<unsigned>(x0) + 1u <= static_cast<unsigned>(W);
    c.idx = c.in ? (y0 + 1) * (W + 2) + (x0 + 1) : 0;
    return c;
}

__device__ __forceinline__ float bilinear_terms(float v00, float v01, float v10, float v11, float ly, float lx) {
    const float hy = __fsub_rn(1.0f, ly), hx = __fsub_rn(1.0f, lx);
    const float t0 = __fmul_rn(__fmul_rn(v00, hy), hx);
    const float t1 = __fmul_rn(__fmul_rn(v01, hy), lx);
    const float t2 = __fmul_rn(__fmul_rn(v10, ly), hx);
    const float t3 = __fmul_rn(__fmul_rn(v11, ly), lx);
    return __fadd_rn(__fadd_rn(__fadd_rn(t0, t1), t2), t3);
}

__device__ __forceinline__ float2 pair_to_float2(uint32_t word) {
    __half2 h;
    memcpy(&h, &word, sizeof(h));
    return __half22float2(h);
}

// kSlabs: the deform input is written in the DCN's slab layout (zero ring included) from the staged
// slices, in place of the NCHW copy.  The kernel is then launched in clusters of two blocks, the two
// 4-channel slices of one deformable group (8 * map + ch0 / 8), which together hold whole 16-byte
// positions.
// kQuad (frames with W % 4 == 0): interior rows are staged four pixels at a time.
template <bool kSlabs, bool kQuad>
__global__ void __launch_bounds__(kTsThreads) temporal_prepare_staged_kernel(const TemporalArgs a) {
    extern __shared__ __align__(16) uint8_t ts_smem[];
    // In-frame offsets are 32-bit (a staged frame holds at most a few thousand pixels); rows and
    // columns advance incrementally with the thread stride instead of by division.
    const int W = a.W, H = a.H, sw = W + 2;
    const int positions = (H + 2) * sw;
    const int plane = H * W;
    uint2 *slab_s = reinterpret_cast<uint2 *>(ts_smem);
    // Block = (frame, map, 4-channel slice): map 0 warps feat_prop by flow1 (and copies
    // feat_current), map 1 warps feat_n2 by flow2; the two share no data.
    const int job = blockIdx.x % (2 * kTsSlices);
    const int map = job / kTsSlices;
    const int ch0 = (job % kTsSlices) * kTsSlice;
    const int step_y = kTsThreads / W, step_x = kTsThreads % W;           // pixel stride as (rows, cols)
    const int pstep_y = kTsThreads / sw, pstep_x = kTsThreads % sw;       // padded-position stride
    const int y_first = static_cast<int>(threadIdx.x) / W, x_first = static_cast<int>(threadIdx.x) % W;
    const int py_first = static_cast<int>(threadIdx.x) / sw, px_first = static_cast<int>(threadIdx.x) % sw;
    const int quads = kQuad ? W / 4 : 1;  // quad staging: first item and stride as (rows, quads)
    for (int64_t n = blockIdx.x / (2 * kTsSlices); n < a.N; n += gridDim.x / (2 * kTsSlices)) {
        const int64_t feat = (n * kTpChannels + ch0) * plane;
        const __half *src = (map ? a.feat_n2 : a.feat_prop) + feat;
        __half *cond = a.conditions + n * 196 * static_cast<int64_t>(plane);
        __half *di = a.deform_input != nullptr ? a.deform_input + n * 128 * static_cast<int64_t>(plane) : nullptr;
        // Plane copies, 16 bytes per access: feat_current's 4 planes into the conditions (map 0),
        // and the map's 4 planes into the deform input (each 4 planes are contiguous).
        const int vec = (kTsSlice * plane) / 8;  // uint4 per 4 planes (plane % 2 == 0 checked on launch)
        {
            if (map == 0) {
                const uint4 *cur4 = reinterpret_cast<const uint4 *>(a.feat_current + feat);
                uint4 *cond4 = reinterpret_cast<uint4 *>(cond + (64 + ch0) * plane);
                for (int i = threadIdx.x; i < vec; i += kTsThreads) cond4[i] = cur4[i];
            }
            if (!kSlabs && di != nullptr) {
                const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
                uint4 *d4 = reinterpret_cast<uint4 *>(di + (64 * map + ch0) * plane);
                for (int i = threadIdx.x; i < vec; i += kTsThreads) d4[i] = s4[i];
            }
        }
        // Stage the slab (zero ring).
        if constexpr (kQuad) {
            // Interior rows four pixels at a time: one 8-byte load per channel plane (pixels
            // 4j..4j+3 of one row; W % 4 == 0 keeps it 8-byte aligned), transposed in registers into
            // four 8-byte positions.  The zero ring separately.
            const int items = H * quads;
            const int qstep_y = kTsThreads / quads, qstep_x = kTsThreads % quads;
            int iy = static_cast<int>(threadIdx.x) / quads, ij = static_cast<int>(threadIdx.x) % quads;
#pragma unroll 1
            for (int t = threadIdx.x; t < items; t += kTsThreads) {
                const int e = iy * W + 4 * ij;
                uint2 v[kTsSlice];
#pragma unroll
                for (int k = 0; k < kTsSlice; ++k) v[k] = *reinterpret_cast<const uint2 *>(src + k * plane + e);
                const int pos = (iy + 1) * sw + 4 * ij + 1;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    // position i: channels (0, 1) and (2, 3) of pixel 4j + i
                    const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
                    const int w = i >> 1;
                    const uint2 o = make_uint2(__byte_perm(w ? v[0].y : v[0].x, w ? v[1].y : v[1].x, sel),
                                               __byte_perm(w ? v[2].y : v[2].x, w ? v[3].y : v[3].x, sel));
                    slab_s[pos + i] = o;
                }
                iy += qstep_y;
                ij += qstep_x;
                if (ij >= quads) {
                    ij -= quads;
                    ++iy;
                }
            }
            // The ring: rows 0 and H+1, then columns 0 and W+1 of rows 1..H.
            const int ring = 2 * sw + 2 * H;
#pragma unroll 1
            for (int r = threadIdx.x; r < ring; r += kTsThreads) {
                const int rr = r - 2 * sw;
                const int q = r < sw ? r : r < 2 * sw ? (H + 1) * sw + (r - sw) : (rr / 2 + 1) * sw + ((rr & 1) ? W + 1 : 0);
                slab_s[q] = make_uint2(0u, 0u);
            }
        } else {
            // Any width: kTsStage positions per thread in flight, one 2-byte load per channel.
            int spy = py_first, spx = px_first;  // padded row/column of this thread's next position
            for (int pos0 = threadIdx.x; pos0 < positions; pos0 += kTsThreads * kTsStage) {
                unsigned short hv[kTsStage][kTsSlice];
#pragma unroll
                for (int u = 0; u < kTsStage; ++u) {
                    const int pos = pos0 + u * kTsThreads;
                    const int y = spy - 1, x = spx - 1;
                    const bool inside = pos < positions && y >= 0 && y < H && x >= 0 && x < W;
                    const int q = inside ? y * W + x : 0;
#pragma unroll
                    for (int k = 0; k < kTsSlice; ++k) hv[u][k] = inside ? __half_as_ushort(src[k * plane + q]) : 0;
                    spy += pstep_y;
                    spx += pstep_x;
                    if (spx >= sw) {
                        spx -= sw;
                        ++spy;
                    }
                }
#pragma unroll
                for (int u = 0; u < kTsStage; ++u) {
                    const int pos = pos0 + u * kTsThreads;
                    if (pos >= positions) break;
                    const uint2 v = make_uint2(hv[u][0] | (static_cast<uint32_t>(hv[u][1]) << 16),
                                               hv[u][2] | (static_cast<uint32_t>(hv[u][3]) << 16));
                    slab_s[pos] = v;
                }
            }
        }
        if constexpr (kSlabs) {
            // The two blocks of one deformable group (slices 2s and 2s + 1, one cluster) each write
            // half of the group's positions as whole 16-byte slab positions: channels 0-3 from
            // rank 0's staged slice, 4-7 from rank 1's, read through distributed shared memory.
            namespace cg = cooperative_groups;
            cg::cluster_group cluster = cg::this_cluster();
            cluster.sync();  // both slices staged
            const uint2 *lo = cluster.map_shared_rank(slab_s, 0), *hi = cluster.map_shared_rank(slab_s, 1);
            uint4 *g = a.slabs + (n * 16 + 8 * map + ch0 / 8) * static_cast<int64_t>(positions);
            const int half = (positions + 1) / 2;
            const int end = cluster.block_rank() ? positions : half;
#pragma unroll 1
            for (int pos = (cluster.block_rank() ? half : 0) + threadIdx.x; pos < end; pos += kTsThreads) {
                const uint2 l = lo[pos], h = hi[pos];
                g[pos] = make_uint4(l.x, l.y, h.x, h.y);
            }
        } else {
            __syncthreads();
        }
        // Map 1 reads the second-order flow from second_order_flow_kernel, which this kernel
        // follows as a programmatic dependent: everything above ran while that kernel did.  Map 0
        // reads flow1, an input, and writes nothing that kernel writes.
        if (map) grid_dependency_wait();
        const __half *fl = map ? a.flow2 + n * 2 * static_cast<int64_t>(plane)
                               : a.flow1 + n * 2 * static_cast<int64_t>(plane);
        __half *out = cond + (128 * map + ch0) * plane;
        int y = y_first, x = x_first;
        // The two flow values of the next pixel are loaded one iteration ahead.
        __half nfx = __float2half_rn(0.0f), nfy = nfx;
        if (static_cast<int>(threadIdx.x) < plane) {
            nfx = fl[threadIdx.x];
            nfy = fl[plane + threadIdx.x];
        }
#pragma unroll 2
        for (int p = threadIdx.x; p < plane; p += kTsThreads) {
            const float fy = static_cast<float>(y), fx = static_cast<float>(x);
            const float vx = __half2float(nfx), vy = __half2float(nfy);
            if (p + kTsThreads < plane) {
                nfx = fl[p + kTsThreads];
                nfy = fl[plane + p + kTsThreads];
            }
            const SlabCorners c = slab_corners(__fadd_rn(fy, vy), __fadd_rn(fx, vx), H, W);
            __half *o = out + p;
            uint2 q00 = make_uint2(0u, 0u), q01 = q00, q10 = q00, q11 = q00;
            if (c.in) {
                q00 = slab_s[c.idx];
                q01 = slab_s[c.idx + 1];
                q10 = slab_s[c.idx + sw];
                q11 = slab_s[c.idx + sw + 1];
            }
            // Each 32-bit word holds two channels: one paired conversion per word.
            const float2 a00 = pair_to_float2(q00.x), b00 = pair_to_float2(q00.y);
            const float2 a01 = pair_to_float2(q01.x), b01 = pair_to_float2(q01.y);
            const float2 a10 = pair_to_float2(q10.x), b10 = pair_to_float2(q10.y);
            const float2 a11 = pair_to_float2(q11.x), b11 = pair_to_float2(q11.y);
            o[0] = __float2half_rn(bilinear_terms(a00.x, a01.x, a10.x, a11.x, c.ly, c.lx));
            o[plane] = __float2half_rn(bilinear_terms(a00.y, a01.y, a10.y, a11.y, c.ly, c.lx));
            o[2 * plane] = __float2half_rn(bilinear_terms(b00.x, b01.x, b10.x, b11.x, c.ly, c.lx));
            o[3 * plane] = __float2half_rn(bilinear_terms(b00.y, b01.y, b10.y, b11.y, c.ly, c.lx));
            y += step_y;
            x += step_x;
            if (x >= W) {
                x -= W;
                ++y;
            }
        }
        // The slab is rewritten for the next frame (in the slab form, after the partner block has
        // read it too).
        if constexpr (kSlabs)
            cooperative_groups::this_cluster().sync();
        else
            __syncthreads();
    }
}

// First pass of the staged form: per pixel the second-order flow (accumulate_second_order_flow_fp16)
// and the four flow channels of the conditions.  The staged kernel is its programmatic dependent.
__global__ void __launch_bounds__(kTsThreads) second_order_flow_kernel(const TemporalArgs a) {
    allow_dependent_launch();
    const int64_t plane = static_cast<int64_t>(a.H) * a.W;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kTsThreads + threadIdx.x;
    if (i >= plane * a.N) return;
    const int64_t n = i / plane, p = i - n * plane;
    const int y = static_cast<int>(p / a.W), x = static_cast<int>(p - static_cast<int64_t>(y) * a.W);
    const __half *f1 = a.flow1 + n * 2 * plane;
    const float f1x = __half2float(f1[p]), f1y = __half2float(f1[plane + p]);
    float f2x = 0.0f, f2y = 0.0f;
    if (a.has_second_order) {
        const Corners c1 = corners(__fadd_rn(static_cast<float>(y), f1y), __fadd_rn(static_cast<float>(x), f1x),
                                   a.H, a.W);
        const __half *prev = a.previous + n * 2 * plane;
        f2x = round_f16(__fadd_rn(f1x, sample(prev, c1, a.W)));
        f2y = round_f16(__fadd_rn(f1y, sample(prev + plane, c1, a.W)));
    }
    __half *f2 = a.flow2 + n * 2 * plane;
    __half *cond = a.conditions + n * 196 * plane;
    f2[p] = __float2half_rn(f2x);
    f2[plane + p] = __float2half_rn(f2y);
    cond[192 * plane + p] = f1[p];
    cond[193 * plane + p] = f1[plane + p];
    cond[194 * plane + p] = __float2half_rn(f2x);
    cond[195 * plane + p] = __float2half_rn(f2y);
}

}  // namespace

// Shared memory of the staged kernel for a frame (one 4-channel slab), or 0 when it exceeds 110 KB,
// which keeps at least two blocks per SM (a 64x64 frame takes 34.8 KB: five blocks, a register
// limit).
size_t temporal_staged_smem(int height, int width) {
    const size_t bytes = static_cast<size_t>(height + 2) * (width + 2) * kTsBytesPerPosition;
    return bytes <= 110 * 1024 ? bytes : 0;
}

// The staged kernel's opt-in to more than 48 KB of dynamic shared memory, a per-device (and
// per-context) function attribute.
cudaError_t temporal_prepare_device() {
    const void *kernels[] = {reinterpret_cast<const void *>(temporal_prepare_staged_kernel<false, false>),
                             reinterpret_cast<const void *>(temporal_prepare_staged_kernel<false, true>),
                             reinterpret_cast<const void *>(temporal_prepare_staged_kernel<true, false>),
                             reinterpret_cast<const void *>(temporal_prepare_staged_kernel<true, true>)};
    for (const void *k : kernels) {
        const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 110 * 1024);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_temporal_prepare(int n, int height, int width, const __half *feat_prop, const __half *feat_current,
                                    const __half *feat_n2, const __half *flow1, const __half *previous,
                                    bool has_second_order, __half *conditions, __half *deform_input, __half *flow2,
                                    void *slabs, cudaStream_t stream) {
    TemporalArgs a{feat_prop, feat_current, feat_n2, flow1, previous, conditions, deform_input, flow2,
                   static_cast<uint4 *>(slabs), n, height, width, has_second_order ? 1 : 0};
    const size_t smem = temporal_staged_smem(height, width);
    const bool vec_ok = (static_cast<int64_t>(height) * width) % 2 == 0 &&
                        ((reinterpret_cast<uintptr_t>(feat_prop) | reinterpret_cast<uintptr_t>(feat_current) |
                          reinterpret_cast<uintptr_t>(feat_n2) | reinterpret_cast<uintptr_t>(conditions) |
                          reinterpret_cast<uintptr_t>(deform_input)) & 15u) == 0;
    if (slabs != nullptr && (smem == 0 || !vec_ok || deform_input != nullptr)) return cudaErrorInvalidValue;
    if (smem > 0 && vec_ok) {
        // The shared-memory opt-in was made by temporal_prepare_device, which the C entry's device
        // set-up (current_device in dcn_api.cu) runs once per device and context.
        const int64_t pixels = static_cast<int64_t>(n) * height * width;
        second_order_flow_kernel<<<static_cast<unsigned>((pixels + kTsThreads - 1) / kTsThreads), kTsThreads, 0,
                                   stream>>>(a);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        const int64_t blocks = static_cast<int64_t>(n) * 2 * kTsSlices;
        const unsigned grid =
            static_cast<unsigned>(blocks < 65535LL * 2 * kTsSlices ? blocks : 65535LL * 2 * kTsSlices);
        const dim3 g(grid), b(kTsThreads);
        // The grid is a whole number of frames' 32 blocks, so slices 2s and 2s + 1 of a (frame, map)
        // are adjacent blocks and form one cluster of two.
        if (width % 4 == 0)
            return slabs != nullptr
                       ? launch_dependent_cluster(temporal_prepare_staged_kernel<true, true>, g, b, smem, stream, 2, a)
                       : launch_dependent(temporal_prepare_staged_kernel<false, true>, g, b, smem, stream, a);
        return slabs != nullptr
                   ? launch_dependent_cluster(temporal_prepare_staged_kernel<true, false>, g, b, smem, stream, 2, a)
                   : launch_dependent(temporal_prepare_staged_kernel<false, false>, g, b, smem, stream, a);
    }
    const int64_t plane = static_cast<int64_t>(height) * width;
    const dim3 grid(static_cast<unsigned>((plane + kTpThreads - 1) / kTpThreads), kTpSlices,
                    static_cast<unsigned>(n < 65535 ? n : 65535));
    temporal_prepare_kernel<<<grid, kTpThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace dcn
