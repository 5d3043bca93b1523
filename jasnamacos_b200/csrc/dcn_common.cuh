// dcn_common.cuh -- shape parameters and sm_100a device helpers shared by the
// DCNv2 kernels (direct FP32/FP16, fused gather + tcgen05, prepack, aux).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dcn_b200.h"

namespace dcn {

// Kernel-side copy of dcn_shape with the derived quantities the loops use
// (DeformConv.swift:22-27, :91-95).
struct Params {
    int N, C, H, W;        // input  [N][C][H][W]
    int OC, HO, WO;        // output [N][OC][HO][WO]
    int KH, KW;            // kernel
    int PH, PW, SH, SW, DH, DW;
    int G;                 // convolution groups
    int OG;                // deformable (offset) groups
    int cpg;               // input channels per conv group   (C / G)
    int opg;               // output channels per conv group  (OC / G)
    int cpog;              // input channels per offset group (C / OG)
    int KA;                // kernel area KH*KW
    int in_plane;          // H*W
    int out_plane;         // HO*WO
    int out_ct;            // channels per image of the output tensor (>= out_c0 + OC)
    int out_c0;            // first output-tensor channel this operator writes
};

inline Params make_params(const dcn_shape &s) {
    Params p;
    p.N = s.batch; p.C = s.input_channels; p.H = s.input_height; p.W = s.input_width;
    p.OC = s.output_channels; p.HO = s.output_height; p.WO = s.output_width;
    p.KH = s.kernel_height; p.KW = s.kernel_width;
    p.PH = s.pad_height; p.PW = s.pad_width; p.SH = s.stride_height; p.SW = s.stride_width;
    p.DH = s.dilation_height; p.DW = s.dilation_width;
    p.G = s.groups; p.OG = s.offset_groups;
    p.cpg = p.C / p.G; p.opg = p.OC / p.G; p.cpog = p.C / p.OG;
    p.KA = p.KH * p.KW;
    p.in_plane = p.H * p.W;
    p.out_plane = p.HO * p.WO;
    p.out_ct = p.OC;
    p.out_c0 = 0;
    return p;
}

// Element offset of output (n, oc, spatial) in the caller's output tensor, which may hold
// more channels per image than this operator writes (out_ct, starting at out_c0).
__host__ __device__ inline int64_t output_index(const Params &p, int64_t n, int oc, int64_t spatial) {
    return (n * p.out_ct + p.out_c0 + oc) * static_cast<int64_t>(p.out_plane) + spatial;
}

// NCHW input whose channels may live in two tensors: channels [0, split) in `first`
// ([N][split][H][W]) and [split, C) in `second` ([N][C - split][H][W]).  With one
// tensor, second is null and split == C.
template <typename T>
struct SplitInput {
    const T *first;
    const T *second;
    int split;
    int C;
    __host__ __device__ const T *channel(int64_t n, int c, int64_t plane) const {
        return c < split ? first + (n * split + c) * plane : second + (n * (C - split) + (c - split)) * plane;
    }
};

// Unique id of the CUDA context current on the calling thread (cuCtxGetId), or 0 when
// no context is current yet.  The per-device caches of device addresses and function
// attributes record it and are rebuilt when it changes: after cudaDeviceReset the
// runtime creates a new primary context, in which the old addresses are meaningless.
uint64_t current_context_id();

// Longest any device-side wait may spin before it gives up and reports
// DCN_ERR_DEVICE_TIMEOUT (nanoseconds of %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Bits of the sticky device error word.
constexpr uint32_t kErrWaitTimeout = 1u;

#if defined(__CUDACC__)

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// try_wait that lets the hardware suspend the thread for up to `ns` nanoseconds
// while the phase is incomplete (it resumes as soon as the phase completes).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity to complete.  Gives up (returns
// false) after kWaitLimitNs, or as soon as *abort becomes non-zero when `abort`
// is given, so a broken pipeline ends the kernel with an error status instead
// of hanging the GPU.
// `backoff_ns` > 0 sleeps between polls (for waiters off the critical path, so
// their polling does not take issue slots and shared-memory cycles).  Critical
// waiters poll with a hardware suspend hint instead, which wakes them as soon as
// the phase completes.
// `limit_ns` replaces kWaitLimitNs for callers that want a shorter bound.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  volatile int *abort, uint32_t backoff_ns = 0,
                                                  uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (backoff_ns) {
            __nanosleep(backoff_ns);
            if (mbar_try_wait(bar, parity)) return true;
        } else if (mbar_try_wait_suspend(bar, parity, 20000u)) {
            return true;
        }
        if (abort != nullptr && *abort) return false;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}


// ---- TMA / bulk copies (each CTA loads only for itself) -------------------------

__device__ __forceinline__ void bulk_copy_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                              uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *smem_dst, const void *tensor_map, uint64_t *bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(smem_dst)),
        "l"(tensor_map), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const void *tensor_map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tensor_map) : "memory");
}

// ---- programmatic dependent launch -----------------------------------------------
// The kernels after the first of an operator call are launched with programmatic stream
// serialization (launch_dependent): their CTAs may become resident while the previous
// kernel of the call is still running, do the set-up that touches no global memory
// (mbarrier init, tensor-memory allocation, tensor-map prefetch) and then block in
// grid_dependency_wait(), which returns only when every prerequisite grid has completed
// and its memory operations are visible -- so results are those of plain stream order,
// with the launch latency and the set-up hidden.  A kernel followed by one of ours calls
// allow_dependent_launch() to let that launch begin early.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

// launch_dependent with thread-block clusters of `cluster_x` blocks along x (the grid's x extent a
// multiple of it).
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, unsigned cluster_x, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

// ---- offset producer of the raw-input form ---------------------------------------
// prepare_dcn_offsets_fp16 (Sources/JasnaMetalPoC/MetalShader.swift:817-839) as the
// tensor-core kernels evaluate it inside their producers: offset = 10*tanh(residue) + flow,
// mask = sigmoid(logit), each rounded to FP16 like the reference's intermediate tensors (the
// offset returned widened to FP32, the mask as FP16, the type the producers keep it in).  Hardware tanh.approx.f32 (~2^-11 relative error), __expf and a
// fast reciprocal; both tensor-core kernels call these, so they produce the same bits.
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float raw_offset(float residue, float flow) {
    return __half2float(__float2half_rn(10.0f * tanh_approx(residue) + flow));
}

__device__ __forceinline__ __half raw_mask(float logit) {
    return __float2half_rn(__fdividef(1.0f, 1.0f + __expf(-logit)));
}

// 32-byte read-only global load (sm_100: 256-bit vector load); `p` must be
// 32-byte aligned.  volatile: the load must never be hoisted out of the bounds
// check that guards it.
__device__ __forceinline__ void ldg_nc_256(const void *p, uint32_t *r) {
    asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "l"(p));
}

// ---- tcgen05 / tensor memory ------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(smem_dst)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]; kind::f16 (FP16/BF16 inputs, FP32 accumulate).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread is complete.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_addr(bar))
        : "memory");
}

// 32 lanes x 4 consecutive 32-bit columns, one lane per thread of the warp.
__device__ __forceinline__ void tmem_st_32x32b_x4(uint32_t taddr, uint32_t r0, uint32_t r1,
                                                  uint32_t r2, uint32_t r3) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
                 "r"(r0), "r"(r1), "r"(r2), "r"(r3)
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from v[0..15], then tcgen05.wait::st, in one asm
// statement.  The source registers are operands of the statement that also waits, so the
// compiler cannot give them to other values while the store may still be reading them (a
// separate asm statement for the wait would allow that).
__device__ __forceinline__ void tmem_st_32x32b_x16_wait(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n\t"
        "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// 12 consecutive 32-bit columns (an x8 and an x4 store) from v, then tcgen05.wait::st, in one
// asm statement (same reason as above).
__device__ __forceinline__ void tmem_st_32x32b_x12_wait(uint32_t taddr, const uint32_t (&v)[3][4]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n\t"
        "tcgen05.st.sync.aligned.32x32b.x4.b32 [%9], {%10, %11, %12, %13};\n\t"
        "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
        "r"(v[0][0]), "r"(v[0][1]), "r"(v[0][2]), "r"(v[0][3]), "r"(v[1][0]), "r"(v[1][1]), "r"(v[1][2]),
        "r"(v[1][3]), "r"(taddr + 8), "r"(v[2][0]), "r"(v[2][1]), "r"(v[2][2]), "r"(v[2][3])
        : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns into v[0..15].
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t *v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms.
// Bits: [0,14) start>>4, [16,30) leading byte offset>>4 (unused for swizzled
// K-major, set to 1), [32,46) stride byte offset>>4 (1024 B between 8-row
// groups), [46,48) descriptor version 1, [61,64) layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t make_sw128_kmajor_desc(uint32_t smem_byte_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor for kind::f16: A and B FP16, D FP32, both K-major,
// M x N tile.  Bits: [4,6) D format (1 = F32), [7,10) A format (0 = F16),
// [10,13) B format (0 = F16), 15/16 A/B major (0 = K), [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t make_idesc_f16_f32(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

#endif  // __CUDACC__

}  // namespace dcn
