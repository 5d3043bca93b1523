// dcn_static_scratch.cu -- dcn_forward_f16_static_scratch: the fused FP16 operator
// with its scratch in a fixed array inside the library instead of a caller buffer.
//
// Who needs it: callers that cannot allocate device memory at the point where
// they run the convolution -- for example code executing inside a region that
// forbids cudaMalloc (a real-time or allocator-less runtime, a plugin host that
// owns all device allocations, or an embedding that only hands out pointers to
// tensors it created itself).  They pass inputs and outputs as usual; the
// regrouped-input scratch that dcn_forward_f16 normally takes from the caller
// lives in `g_static_scratch` below.
//
// Costs and limits:
//  * every GPU that loads this library holds kStaticScratchBytes (16 MiB) for the
//    life of the process;
//  * problems whose scratch would exceed that are rejected with
//    DCN_ERR_SCRATCH_TOO_SMALL (16 MiB holds 15 Jasna 64x64 tiles per call on the slab path, 7 on the global-gather path);
//  * all calls share the one array: two calls that overlap on the GPU (different
//    streams, no ordering between them) race on it and give wrong results;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) -- make that first call before any stream capture, for
//    example as one warm-up call at start-up.  The address is kept per device
//    together with the id of the context it belongs to; a call in a new context
//    (after cudaDeviceReset) looks it up again.
#include <cuda_runtime.h>

#include <mutex>

#include "dcn_b200.h"
#include "dcn_common.cuh"

namespace {

constexpr size_t kStaticScratchBytes = size_t{16} << 20;
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct ScratchAddress {
    void *ptr = nullptr;
    uint64_t ctx_id = 0;  // context the address belongs to
};

std::mutex g_scratch_mutex;
ScratchAddress g_scratch_address[kMaxDevices];

// Device address of g_static_scratch on the current device, looked up with that device
// current once per device and context.
dcn_status scratch_address(void **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return DCN_ERR_NO_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchAddress &a = g_scratch_address[dev];
    if (a.ptr == nullptr || dcn::current_context_id() != a.ctx_id) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess || ptr == nullptr) {
            cudaGetLastError();
            a.ptr = nullptr;
            return e == cudaErrorNoKernelImageForDevice ? DCN_ERR_UNSUPPORTED : DCN_ERR_LAUNCH;
        }
        a.ptr = ptr;
        a.ctx_id = dcn::current_context_id();
    }
    *out = a.ptr;
    return DCN_OK;
}

}  // namespace

extern "C" size_t dcn_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" dcn_status dcn_forward_f16_static_scratch(const dcn_shape *shape, const void *input,
                                                     const void *offset, const void *mask,
                                                     const void *packed_weight, const void *bias,
                                                     void *output, uint32_t *nonfinite_flag,
                                                     dcn_stream stream) {
    dcn_status st = dcn_shape_validate(shape);
    if (st != DCN_OK) return st;
    if (dcn_forward_f16_path(shape) == DCN_PATH_DIRECT) return DCN_ERR_UNSUPPORTED;
    const size_t need = dcn_forward_f16_workspace_bytes(shape);
    if (need > kStaticScratchBytes) return DCN_ERR_SCRATCH_TOO_SMALL;
    void *scratch = nullptr;
    if ((st = scratch_address(&scratch)) != DCN_OK) return st;
    // The regroup kernel overwrites every scratch byte the fused kernel reads, so
    // nothing left by an earlier call needs clearing.
    return dcn_forward_f16(shape, input, offset, mask, packed_weight, bias, output, nonfinite_flag, scratch,
                           kStaticScratchBytes, stream);
}
