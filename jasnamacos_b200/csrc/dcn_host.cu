// dcn_host.cu -- dcn_forward_f16_host: the FP16 operator on host buffers.
//
// The reference operator takes host arrays and returns a host array
// (MetalDeformConv.runFloat32, Sources/JasnaMetalPoC/MetalRunner.swift:159-185, which copies
// the caller's arrays into fresh shared buffers at :584-593).  On a discrete GPU the copies
// dominate: a 64x64 Jasna tile moves 1,120 bytes per output pixel in and 128 out over PCIe,
// against ~1 ns per pixel of kernel time.  This entry point therefore cuts the batch into
// chunks of images and pipelines them: chunk k's host->device copies, its convolution
// (dcn_forward_f16: regroup pre-pass + tensor-core kernel) and its device->host copy are
// enqueued on one of the library's own per-device streams (slot k mod kSlots), so chunk k+1's
// input copy overlaps chunk k's kernels and chunk k-1's output copy runs in the other
// direction at the same time.  Each chunk tensor is one cudaMemcpyAsync.
//
// Device staging memory comes from the caller's workspace (per slot: input, offset, mask,
// output and the operator's own workspace, plus one flag word); the library allocates no
// device memory.  Its streams and events are created once per device and context and reused
// by every call; a mutex per device orders concurrent callers' enqueue sequences.
#include <cuda_runtime.h>

#include <mutex>

#include "dcn_b200.h"
#include "dcn_common.cuh"

namespace {

constexpr int kSlots = 3;  // chunks in flight
constexpr int kMaxDevices = 64;
constexpr size_t kAlign = 256;
constexpr int32_t kDefaultChunkImages = 64;

size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

struct HostStreams {
    bool ready = false;
    uint64_t ctx_id = 0;
    cudaStream_t stream[kSlots] = {};
    cudaEvent_t start = nullptr;
    cudaEvent_t done[kSlots] = {};
    std::mutex call_mutex;  // one enqueue sequence at a time on these streams
};

std::mutex g_host_mutex;
HostStreams g_host[kMaxDevices];

// The slot streams and events of the current device, created on first use (or again in a
// new context).
dcn_status host_streams(HostStreams **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return DCN_ERR_NO_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_host_mutex);
    HostStreams &h = g_host[dev];
    if (!h.ready || dcn::current_context_id() != h.ctx_id) {
        // Handles of an old context are gone with it; they are not destroyed here.
        h.ready = false;
        cudaError_t e = cudaEventCreateWithFlags(&h.start, cudaEventDisableTiming);
        for (int i = 0; i < kSlots && e == cudaSuccess; ++i) {
            e = cudaStreamCreateWithFlags(&h.stream[i], cudaStreamNonBlocking);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h.done[i], cudaEventDisableTiming);
        }
        if (e != cudaSuccess) {
            cudaGetLastError();
            return DCN_ERR_LAUNCH;
        }
        h.ctx_id = dcn::current_context_id();
        h.ready = true;
    }
    *out = &h;
    return DCN_OK;
}

// Byte layout of one slot of the staging workspace for chunks of up to `chunk` images.
struct SlotLayout {
    size_t input, offset, mask, output, ws, ws_bytes, slot_bytes;
};

SlotLayout slot_layout(const dcn_shape &shape, int32_t chunk) {
    dcn_shape one = shape;
    one.batch = 1;
    dcn_counts c;
    dcn_shape_counts(&one, &c);
    SlotLayout l;
    l.input = 0;
    l.offset = l.input + align_up(static_cast<size_t>(c.input) * chunk * 2);
    l.mask = l.offset + align_up(static_cast<size_t>(c.offset) * chunk * 2);
    l.output = l.mask + align_up(static_cast<size_t>(c.mask) * chunk * 2);
    l.ws = l.output + align_up(static_cast<size_t>(c.output) * chunk * 2);
    // The operator's workspace for the larger of the two chunk sizes a call uses: full
    // chunks and the short last one (which may take the group split, whose partial sums
    // need more per image).
    dcn_shape s = shape;
    s.batch = chunk;
    l.ws_bytes = dcn_forward_f16_workspace_bytes(&s);
    if (shape.batch % chunk != 0) {
        s.batch = shape.batch % chunk;
        const size_t tail = dcn_forward_f16_workspace_bytes(&s);
        if (tail > l.ws_bytes) l.ws_bytes = tail;
    }
    l.slot_bytes = l.ws + align_up(l.ws_bytes);
    return l;
}

int32_t effective_chunk(const dcn_shape &shape, int32_t chunk_images) {
    int32_t c = chunk_images > 0 ? chunk_images : kDefaultChunkImages;
    return c < shape.batch ? c : shape.batch;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

extern "C" size_t dcn_forward_f16_host_workspace_bytes(const dcn_shape *shape, int32_t chunk_images) {
    if (dcn_shape_validate(shape) != DCN_OK || chunk_images < 0) return 0;
    if (dcn_forward_f16_path(shape) == DCN_PATH_DIRECT) return 0;
    const int32_t chunk = effective_chunk(*shape, chunk_images);
    const int32_t slots = (shape->batch + chunk - 1) / chunk < kSlots ? (shape->batch + chunk - 1) / chunk : kSlots;
    return kAlign + static_cast<size_t>(slots) * slot_layout(*shape, chunk).slot_bytes;
}

extern "C" dcn_status dcn_forward_f16_host(const dcn_shape *shape, const void *input_host, const void *offset_host,
                                           const void *mask_host, const void *packed_weight, const void *bias,
                                           void *output_host, uint32_t *nonfinite_flag_host, int32_t chunk_images,
                                           void *workspace, size_t workspace_bytes, dcn_stream stream) {
    dcn_status st = dcn_shape_validate(shape);
    if (st != DCN_OK) return st;
    if (dcn_forward_f16_path(shape) == DCN_PATH_DIRECT) return DCN_ERR_UNSUPPORTED;
    if (!input_host || !offset_host || !mask_host || !packed_weight || !bias || !output_host || !workspace)
        return DCN_ERR_INVALID_ARGUMENT;
    if (chunk_images < 0 || !aligned(workspace, kAlign) ||
        workspace_bytes < dcn_forward_f16_host_workspace_bytes(shape, chunk_images))
        return DCN_ERR_INVALID_ARGUMENT;
    HostStreams *h = nullptr;
    if ((st = host_streams(&h)) != DCN_OK) return st;

    const int32_t chunk = effective_chunk(*shape, chunk_images);
    const int32_t chunks = (shape->batch + chunk - 1) / chunk;
    const int32_t slots = chunks < kSlots ? chunks : kSlots;
    const SlotLayout l = slot_layout(*shape, chunk);
    dcn_shape one = *shape;
    one.batch = 1;
    dcn_counts per;
    dcn_shape_counts(&one, &per);
    const size_t in_b = static_cast<size_t>(per.input) * 2, off_b = static_cast<size_t>(per.offset) * 2;
    const size_t msk_b = static_cast<size_t>(per.mask) * 2, out_b = static_cast<size_t>(per.output) * 2;
    auto *base = static_cast<uint8_t *>(workspace);
    auto *flag = reinterpret_cast<uint32_t *>(base);  // first kAlign bytes: the flag word
    const auto *hin = static_cast<const uint8_t *>(input_host);
    const auto *hoff = static_cast<const uint8_t *>(offset_host);
    const auto *hmsk = static_cast<const uint8_t *>(mask_host);
    auto *hout = static_cast<uint8_t *>(output_host);
    cudaStream_t caller = reinterpret_cast<cudaStream_t>(stream);

    std::lock_guard<std::mutex> lock(h->call_mutex);
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(uint32_t), caller);
    if (e == cudaSuccess) e = cudaEventRecord(h->start, caller);
    for (int i = 0; i < slots && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(h->stream[i], h->start, 0);
    for (int32_t k = 0; k < chunks && e == cudaSuccess; ++k) {
        const int32_t b0 = k * chunk;
        const int32_t n = shape->batch - b0 < chunk ? shape->batch - b0 : chunk;
        cudaStream_t s = h->stream[k % slots];
        uint8_t *slot = base + kAlign + static_cast<size_t>(k % slots) * l.slot_bytes;
        e = cudaMemcpyAsync(slot + l.input, hin + b0 * in_b, n * in_b, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(slot + l.offset, hoff + b0 * off_b, n * off_b, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(slot + l.mask, hmsk + b0 * msk_b, n * msk_b, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) break;
        dcn_shape cs = *shape;
        cs.batch = n;
        st = dcn_forward_f16(&cs, slot + l.input, slot + l.offset, slot + l.mask, packed_weight, bias,
                             slot + l.output, flag, slot + l.ws, l.ws_bytes, reinterpret_cast<dcn_stream>(s));
        if (st != DCN_OK) break;
        e = cudaMemcpyAsync(hout + b0 * out_b, slot + l.output, n * out_b, cudaMemcpyDeviceToHost, s);
    }
    // The caller's stream waits for every slot stream (also after an error, so that no slot
    // work is left unordered with the caller's later work).
    for (int i = 0; i < slots; ++i) {
        if (cudaEventRecord(h->done[i], h->stream[i]) == cudaSuccess) cudaStreamWaitEvent(caller, h->done[i], 0);
    }
    if (e == cudaSuccess && st == DCN_OK && nonfinite_flag_host != nullptr)
        e = cudaMemcpyAsync(nonfinite_flag_host, flag, sizeof(uint32_t), cudaMemcpyDeviceToHost, caller);
    if (st != DCN_OK) return st;
    if (e != cudaSuccess) {
        cudaGetLastError();
        return DCN_ERR_LAUNCH;
    }
    return DCN_OK;
}
