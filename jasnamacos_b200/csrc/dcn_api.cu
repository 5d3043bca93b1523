// dcn_api.cu -- the extern "C" boundary declared in include/dcn_b200.h.
//
// Validation mirrors DeformConvShape.validate / DeformConvCPU.require
// (Sources/JasnaMetalPoC/DeformConv.swift:29-41, :140-144) and the Metal
// runner's shape guards (MetalRunner.swift:630-713), but unsupported shapes
// return an error instead of the reference kernels' silent early return
// (MetalShader.swift:192, :254-256).  Launches are asynchronous on the caller's
// stream; nothing here allocates device memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "dcn_b200.h"
#include "dcn_common.cuh"

namespace dcn {

cudaError_t launch_direct_f32(const Params &p, const float *input, const float *offset, const float *mask,
                              const float *weight, const float *bias, float *output, cudaStream_t stream);
cudaError_t launch_direct_f16(const Params &p, const SplitInput<__half> &input, const __half *offset,
                              const __half *mask, const __half *weight, const __half *bias, __half *output,
                              cudaStream_t stream);
cudaError_t launch_prepack_weights(const Params &p, bool fused, int kb, const void *src, dcn_dtype src_dtype,
                                   int layout, void *dst, cudaStream_t stream);
cudaError_t launch_flag_non_finite(const __half *values, int64_t count, uint32_t *flag, int sm_count,
                                   cudaStream_t stream);
cudaError_t launch_flag_non_finite_rows(const __half *values, int64_t rows, int64_t row_len, int64_t row_stride,
                                        uint32_t *flag, int sm_count, cudaStream_t stream);
cudaError_t launch_check_wait_timeout(uint64_t limit_ns, uint32_t *err, cudaStream_t stream);
cudaError_t launch_prepare_offsets(int64_t n_images, int gka, int64_t plane, const __half *raw, const __half *flow1,
                                   const __half *flow2, __half *offset, __half *mask, cudaStream_t stream);
cudaError_t launch_slab_grouped_raw(const Params &p, const void *slabs, const __half *raw, const __half *flow1,
                                    const __half *flow2, const uint8_t *packed_w, const __half *bias,
                                    __half *output, uint32_t *flag, int sm_count, uint32_t *err,
                                    cudaStream_t stream);
bool fused_supported(const Params &p);
int fused_kblocks(const Params &p);
size_t fused_workspace_bytes(const Params &p);
cudaError_t fused_prepare_device(uint32_t **err_word);
cudaError_t launch_regroup_c8(const Params &p, const SplitInput<__half> &input, void *workspace,
                              cudaStream_t stream);
cudaError_t launch_fused_grouped(const Params &p, const void *input_c8, const __half *offset, const __half *mask,
                                 const uint8_t *packed_w, const __half *bias, __half *output, uint32_t *flag,
                                 int sm_count, uint32_t *err, cudaStream_t stream);
cudaError_t launch_fused_grouped_raw(const Params &p, const void *input_c8, const __half *raw,
                                     const __half *flow1, const __half *flow2, const uint8_t *packed_w,
                                     const __half *bias, __half *output, uint32_t *flag, int sm_count,
                                     uint32_t *err, cudaStream_t stream);
bool slab_supported(const Params &p);
void slab_plan(const Params &p, int sm_count, dcn_plan *out);
size_t slab_workspace_bytes(const Params &p);
size_t slab_packed_weight_bytes(const Params &p);
cudaError_t slab_prepare_device();
cudaError_t temporal_prepare_device();
cudaError_t launch_regroup_slabs(const Params &p, const SplitInput<__half> &input, void *workspace,
                                 cudaStream_t stream);
cudaError_t launch_prepack_slab(const Params &p, const void *src, dcn_dtype src_dtype, int layout, void *dst,
                                cudaStream_t stream);
cudaError_t launch_slab_grouped(const Params &p, const void *slabs, const __half *offset, const __half *mask,
                                const uint8_t *packed_w, const __half *bias, __half *output, uint32_t *flag,
                                int sm_count, uint32_t *err, cudaStream_t stream);

cudaError_t launch_temporal_prepare(int n, int height, int width, const __half *feat_prop, const __half *feat_current,
                                    const __half *feat_n2, const __half *flow1, const __half *previous,
                                    bool has_second_order, __half *conditions, __half *deform_input, __half *flow2,
                                    void *slabs, cudaStream_t stream);
size_t temporal_staged_smem(int height, int width);
cudaError_t launch_regroup_nhwc(bool slabs, int N, int G, int H, int W, const __half *in, void *workspace,
                                cudaStream_t stream);

uint64_t current_context_id() {
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *a = nullptr, *b = nullptr;
        cudaDriverEntryPointQueryResult qa, qb;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &a, 4000, cudaEnableDefault, &qa) == cudaSuccess &&
            qa == cudaDriverEntryPointSuccess &&
            cudaGetDriverEntryPointByVersion("cuCtxGetId", &b, 12000, cudaEnableDefault, &qb) == cudaSuccess &&
            qb == cudaDriverEntryPointSuccess) {
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(a);
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(b);
        }
        cudaGetLastError();
    });
    if (get_current == nullptr || get_id == nullptr) return 0;
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

namespace {

constexpr int kMaxDevices = 64;

// Per device: the attributes every launch needs, filled with that device's context
// current and valid for that context only (ctx_id).
struct DeviceInfo {
    bool ready = false;
    bool sm100 = false;
    int sm_count = 0;
    uint32_t *err_word = nullptr;
    uint64_t ctx_id = 0;
};

std::mutex g_mutex;
DeviceInfo g_devices[kMaxDevices];

dcn_status from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return DCN_OK;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return DCN_ERR_NO_DEVICE;
    if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction) return DCN_ERR_UNSUPPORTED;
    return DCN_ERR_LAUNCH;
}

// Looks up (once per device and context, under a mutex) the attributes every launch
// needs.  A changed context id (cudaDeviceReset, then a new primary context) repeats
// the set-up, since the error word's address and the kernels' shared-memory opt-in
// belong to the old context.
dcn_status current_device(DeviceInfo **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return from_cuda(e) == DCN_ERR_LAUNCH ? DCN_ERR_NO_DEVICE : from_cuda(e);
    }
    if (dev < 0 || dev >= kMaxDevices) return DCN_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceInfo &d = g_devices[dev];
    if (!d.ready || current_context_id() != d.ctx_id) {
        d.ready = false;
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return DCN_ERR_NO_DEVICE;
        }
        d.sm100 = (major == 10 && minor == 0);
        d.sm_count = sms;
        if (d.sm100) {
            e = fused_prepare_device(&d.err_word);
            if (e == cudaSuccess) e = slab_prepare_device();
            if (e == cudaSuccess) e = temporal_prepare_device();
            if (e != cudaSuccess) {
                cudaGetLastError();
                return from_cuda(e);
            }
        }
        d.ctx_id = current_context_id();
        d.ready = true;
    }
    if (!d.sm100) return DCN_ERR_UNSUPPORTED;  // the library carries sm_100a code only
    *out = &d;
    return DCN_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Shape checks beyond DeformConvShape.validate that keep every index the
// kernels form inside 32 bits per image plane and every position inside int32.
dcn_status validate(const dcn_shape *s) {
    if (s == nullptr) return DCN_ERR_INVALID_ARGUMENT;
    if (!(s->batch > 0 && s->input_channels > 0 && s->output_channels > 0 && s->input_height > 0 &&
          s->input_width > 0 && s->output_height > 0 && s->output_width > 0 && s->kernel_height > 0 &&
          s->kernel_width > 0 && s->groups > 0 && s->offset_groups > 0 &&
          s->input_channels % s->groups == 0 && s->output_channels % s->groups == 0 &&
          s->input_channels % s->offset_groups == 0))
        return DCN_ERR_INVALID_SHAPE;
    const int64_t in_plane = static_cast<int64_t>(s->input_height) * s->input_width;
    const int64_t out_plane = static_cast<int64_t>(s->output_height) * s->output_width;
    const int64_t ka = static_cast<int64_t>(s->kernel_height) * s->kernel_width;
    if (in_plane >= (int64_t{1} << 31) || out_plane >= (int64_t{1} << 31) || ka > 1024)
        return DCN_ERR_INVALID_SHAPE;
    // Largest |integer part| of a sampling position: |o*stride| + |pad| + |k*dilation|.
    auto mag = [](int64_t v) { return v < 0 ? -v : v; };
    const int64_t ymax = mag(int64_t{s->output_height} * s->stride_height) + mag(s->pad_height) +
                         mag(int64_t{s->kernel_height} * s->dilation_height);
    const int64_t xmax = mag(int64_t{s->output_width} * s->stride_width) + mag(s->pad_width) +
                         mag(int64_t{s->kernel_width} * s->dilation_width);
    if (ymax >= (int64_t{1} << 30) || xmax >= (int64_t{1} << 30)) return DCN_ERR_INVALID_SHAPE;
    const int64_t counts[4] = {
        int64_t{s->batch} * s->input_channels * in_plane,
        int64_t{s->batch} * 2 * s->offset_groups * ka * out_plane,
        int64_t{s->batch} * s->output_channels * out_plane,
        int64_t{s->output_channels} * (s->input_channels / s->groups) * ka,
    };
    for (int64_t c : counts)
        if (c >= (int64_t{1} << 40)) return DCN_ERR_INVALID_SHAPE;
    return DCN_OK;
}

// Kernel preference for shapes both tensor-core kernels take, from the environment
// variable DCN_B200_FUSED_KERNEL (read once): "pairs" forces the global-gather
// kernel, "slab" or anything else keeps the default (slab where it applies).
bool slab_allowed() {
    static const bool allowed = [] {
        const char *v = std::getenv("DCN_B200_FUSED_KERNEL");
        return !(v != nullptr && std::string(v) == "pairs");
    }();
    return allowed;
}

// The implementation dcn_forward_f16 runs for a validated shape.
dcn_path select_path(const Params &p) {
    if (slab_allowed() && slab_supported(p)) return DCN_PATH_SLAB_TC;
    if (fused_supported(p)) return DCN_PATH_FUSED_TC;
    return DCN_PATH_DIRECT;
}

}  // namespace
}  // namespace dcn

using namespace dcn;

extern "C" {

int dcn_abi_version(void) { return DCN_B200_ABI_VERSION; }

const char *dcn_status_string(dcn_status status) {
    switch (status) {
    case DCN_OK: return "ok";
    case DCN_ERR_INVALID_SHAPE: return "Invalid deformable-convolution shape";
    case DCN_ERR_INVALID_COUNT: return "An array has the wrong number of elements for the shape";
    case DCN_ERR_NO_DEVICE: return "No CUDA device is available";
    case DCN_ERR_UNSUPPORTED: return "The shape or device is not supported by this kernel";
    case DCN_ERR_NONFINITE: return "The deformable convolution produced non-finite output";
    case DCN_ERR_LAUNCH: return "CUDA launch failed";
    case DCN_ERR_INVALID_ARGUMENT: return "Invalid argument (null or misaligned pointer, short workspace)";
    case DCN_ERR_DEVICE_TIMEOUT: return "A device-side wait timed out (pipeline error)";
    case DCN_ERR_SCRATCH_TOO_SMALL:
        return "The problem needs more scratch than the library's static scratch array holds";
    }
    return "unknown status";
}

int dcn_status_is_recoverable(dcn_status status) { return status == DCN_ERR_NONFINITE ? 1 : 0; }

dcn_status dcn_shape_validate(const dcn_shape *shape) { return validate(shape); }

dcn_status dcn_shape_counts(const dcn_shape *s, dcn_counts *out) {
    if (s == nullptr || out == nullptr) return DCN_ERR_INVALID_ARGUMENT;
    dcn_status st = validate(s);
    if (st != DCN_OK) return st;
    const int64_t out_plane = int64_t{s->output_height} * s->output_width;
    const int64_t ka = int64_t{s->kernel_height} * s->kernel_width;
    out->input = int64_t{s->batch} * s->input_channels * s->input_height * s->input_width;
    out->offset = int64_t{s->batch} * 2 * s->offset_groups * ka * out_plane;
    out->mask = int64_t{s->batch} * s->offset_groups * ka * out_plane;
    out->weight = int64_t{s->output_channels} * (s->input_channels / s->groups) * ka;
    out->bias = s->output_channels;
    out->output = int64_t{s->batch} * s->output_channels * out_plane;
    return DCN_OK;
}

dcn_status dcn_check_counts(const dcn_shape *shape, int64_t input_count, int64_t offset_count,
                            int64_t mask_count, int64_t weight_count, int64_t bias_count, int *which_out) {
    dcn_counts c;
    dcn_status st = dcn_shape_counts(shape, &c);
    if (st != DCN_OK) return st;
    const int64_t expected[5] = {c.input, c.offset, c.mask, c.weight, c.bias};
    const int64_t actual[5] = {input_count, offset_count, mask_count, weight_count, bias_count};
    for (int i = 0; i < 5; ++i) {
        if (expected[i] != actual[i]) {
            if (which_out) *which_out = i;
            return DCN_ERR_INVALID_COUNT;
        }
    }
    return DCN_OK;
}

dcn_status dcn_forward_f32(const dcn_shape *shape, const float *input, const float *offset, const float *mask,
                           const float *weight_oihw, const float *bias, float *output, dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    if (!input || !offset || !mask || !weight_oihw || !bias || !output) return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    return from_cuda(launch_direct_f32(make_params(*shape), input, offset, mask, weight_oihw, bias, output,
                                       reinterpret_cast<cudaStream_t>(stream)));
}

dcn_status dcn_forward_f16_direct(const dcn_shape *shape, const void *input, const void *offset,
                                  const void *mask, const void *weight_oihw, const void *bias, void *output,
                                  dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    if (!input || !offset || !mask || !weight_oihw || !bias || !output) return DCN_ERR_INVALID_ARGUMENT;
    if (!aligned(input, 2) || !aligned(offset, 2) || !aligned(mask, 2) || !aligned(weight_oihw, 2) ||
        !aligned(bias, 2) || !aligned(output, 2))
        return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    const Params p = make_params(*shape);
    return from_cuda(launch_direct_f16(
        p, SplitInput<__half>{static_cast<const __half *>(input), nullptr, p.C, p.C}, static_cast<const __half *>(offset),
        static_cast<const __half *>(mask), static_cast<const __half *>(weight_oihw),
        static_cast<const __half *>(bias), static_cast<__half *>(output), reinterpret_cast<cudaStream_t>(stream)));
}

dcn_path dcn_forward_f16_path(const dcn_shape *shape) {
    if (validate(shape) != DCN_OK) return DCN_PATH_DIRECT;
    return select_path(make_params(*shape));
}

dcn_status dcn_forward_f16_plan(const dcn_shape *shape, dcn_plan *out) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    if (out == nullptr) return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    const Params p = make_params(*shape);
    *out = dcn_plan{};
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_SLAB_TC) {
        slab_plan(p, dev->sm_count, out);
        return DCN_OK;
    }
    out->path = path;
    out->group_splits = 1;
    out->tiles_per_unit = 1;
    if (path == DCN_PATH_FUSED_TC) {
        const int64_t tiles = static_cast<int64_t>(p.N) * ((p.out_plane + 127) / 128);
        out->grid = tiles < dev->sm_count ? tiles : dev->sm_count;
        out->prepass_images = p.N;
        out->launches = 2;
    } else {
        out->grid = (static_cast<int64_t>(p.N) * p.out_plane + 15) / 16 * p.G * ((p.opg + 63) / 64);
        out->launches = 1;
    }
    return DCN_OK;
}

size_t dcn_packed_weight_bytes(const dcn_shape *shape) {
    if (validate(shape) != DCN_OK) return 0;
    const Params p = make_params(*shape);
    switch (select_path(p)) {
    case DCN_PATH_SLAB_TC: return slab_packed_weight_bytes(p);
    case DCN_PATH_FUSED_TC: return static_cast<size_t>(fused_kblocks(p)) * 64 * 64 * sizeof(__half);
    default: return static_cast<size_t>(p.OC) * p.cpg * p.KA * sizeof(__half);
    }
}

dcn_status dcn_prepack_weights(const dcn_shape *shape, const void *weight, dcn_dtype src_dtype,
                               dcn_weight_layout src_layout, void *packed, dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    if (!weight || !packed) return DCN_ERR_INVALID_ARGUMENT;
    if (src_dtype != DCN_DTYPE_F32 && src_dtype != DCN_DTYPE_F16) return DCN_ERR_INVALID_ARGUMENT;
    if (src_layout != DCN_WEIGHT_OIHW && src_layout != DCN_WEIGHT_IC_K_OC) return DCN_ERR_INVALID_ARGUMENT;
    if (!aligned(weight, src_dtype == DCN_DTYPE_F32 ? 4 : 2) || !aligned(packed, 16))
        return DCN_ERR_INVALID_ARGUMENT;
    const Params p = make_params(*shape);
    // The [ic][k][oc] layout only exists for one convolution group (the reference's packed kernels).
    if (src_layout == DCN_WEIGHT_IC_K_OC && p.G != 1) return DCN_ERR_UNSUPPORTED;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_SLAB_TC)
        return from_cuda(launch_prepack_slab(p, weight, src_dtype, static_cast<int>(src_layout), packed, s));
    const bool fused = path == DCN_PATH_FUSED_TC;
    return from_cuda(launch_prepack_weights(p, fused, fused ? fused_kblocks(p) : 0, weight, src_dtype,
                                            static_cast<int>(src_layout), packed, s));
}

size_t dcn_forward_f16_workspace_bytes(const dcn_shape *shape) {
    if (validate(shape) != DCN_OK) return 0;
    const Params p = make_params(*shape);
    switch (select_path(p)) {
    case DCN_PATH_SLAB_TC: return slab_workspace_bytes(p);
    case DCN_PATH_FUSED_TC: return fused_workspace_bytes(p);
    default: return 0;
    }
}

namespace {

// The tensor-core kernel of `path` on an input already in that path's grouped layout.
dcn_status launch_grouped(dcn_path path, const Params &p, const void *grouped, const void *offset,
                          const void *mask, const void *packed_weight, const void *bias, void *output,
                          uint32_t *flag, DeviceInfo *dev, cudaStream_t s) {
    const auto *off = static_cast<const __half *>(offset);
    const auto *msk = static_cast<const __half *>(mask);
    const auto *w = static_cast<const uint8_t *>(packed_weight);
    const auto *b = static_cast<const __half *>(bias);
    auto *out = static_cast<__half *>(output);
    if (path == DCN_PATH_SLAB_TC)
        return from_cuda(launch_slab_grouped(p, grouped, off, msk, w, b, out, flag, dev->sm_count, dev->err_word, s));
    return from_cuda(launch_fused_grouped(p, grouped, off, msk, w, b, out, flag, dev->sm_count, dev->err_word, s));
}

cudaError_t launch_regroup(dcn_path path, const Params &p, const SplitInput<__half> &in, void *workspace,
                           cudaStream_t s) {
    return path == DCN_PATH_SLAB_TC ? launch_regroup_slabs(p, in, workspace, s) : launch_regroup_c8(p, in, workspace, s);
}

// Applies a caller's dcn_io (null: defaults) to the kernel parameters and builds the
// input view.  The output slot goes into p (out_ct, out_c0).
dcn_status resolve_io(const dcn_io *io, dcn_path path, const void *input, Params *p, SplitInput<__half> *in) {
    *in = SplitInput<__half>{static_cast<const __half *>(input), nullptr, p->C, p->C};
    if (io == nullptr) return DCN_OK;
    if (io->input_second != nullptr) {
        const int split = io->input_split;
        if (split <= 0 || split >= p->C || !aligned(io->input_second, 2)) return DCN_ERR_INVALID_ARGUMENT;
        // The regroup pre-passes read one deformable group's 8 channels from one tensor.
        if (path != DCN_PATH_DIRECT && split % 8 != 0) return DCN_ERR_INVALID_ARGUMENT;
        in->second = static_cast<const __half *>(io->input_second);
        in->split = split;
    } else if (io->input_split != 0) {
        return DCN_ERR_INVALID_ARGUMENT;
    }
    if (io->output_image_channels == 0) {
        if (io->output_channel_offset != 0) return DCN_ERR_INVALID_ARGUMENT;
    } else {
        if (io->output_channel_offset < 0 ||
            static_cast<int64_t>(io->output_image_channels) < static_cast<int64_t>(p->OC) + io->output_channel_offset)
            return DCN_ERR_INVALID_ARGUMENT;
        p->out_ct = io->output_image_channels;
        p->out_c0 = io->output_channel_offset;
    }
    return DCN_OK;
}

}  // namespace

dcn_status dcn_forward_f16_io(const dcn_shape *shape, const dcn_io *io, const void *input, const void *offset,
                              const void *mask, const void *packed_weight, const void *bias, void *output,
                              uint32_t *nonfinite_flag, void *workspace, size_t workspace_bytes,
                              dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    if (!input || !offset || !mask || !packed_weight || !bias || !output) return DCN_ERR_INVALID_ARGUMENT;
    if (!aligned(input, 2) || !aligned(bias, 2) || !aligned(output, 2) || !aligned(packed_weight, 16) ||
        (nonfinite_flag && !aligned(nonfinite_flag, 4)))
        return DCN_ERR_INVALID_ARGUMENT;
    Params p = make_params(*shape);
    const dcn_path path = select_path(p);
    SplitInput<__half> in;
    if ((st = resolve_io(io, path, input, &p, &in)) != DCN_OK) return st;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (path == DCN_PATH_DIRECT) {
        if (!aligned(offset, 2) || !aligned(mask, 2)) return DCN_ERR_INVALID_ARGUMENT;
        cudaError_t e = launch_direct_f16(p, in, static_cast<const __half *>(offset),
                                          static_cast<const __half *>(mask),
                                          static_cast<const __half *>(packed_weight),
                                          static_cast<const __half *>(bias), static_cast<__half *>(output), s);
        if (e == cudaSuccess && nonfinite_flag)
            e = launch_flag_non_finite_rows(static_cast<const __half *>(output) + output_index(p, 0, 0, 0), p.N,
                                            static_cast<int64_t>(p.OC) * p.out_plane,
                                            static_cast<int64_t>(p.out_ct) * p.out_plane, nonfinite_flag,
                                            dev->sm_count, s);
        return from_cuda(e);
    }
    // Tensor-core paths: offsets/masks are read by TMA (16-byte aligned rows), the
    // regrouped input by 16/32-byte loads.
    if (!aligned(offset, 16) || !aligned(mask, 16)) return DCN_ERR_INVALID_ARGUMENT;
    if (!workspace || !aligned(workspace, 256) || workspace_bytes < dcn_forward_f16_workspace_bytes(shape))
        return DCN_ERR_INVALID_ARGUMENT;
    cudaError_t e = launch_regroup(path, p, in, workspace, s);
    if (e != cudaSuccess) return from_cuda(e);
    return launch_grouped(path, p, workspace, offset, mask, packed_weight, bias, output, nonfinite_flag, dev, s);
}

dcn_status dcn_forward_f16(const dcn_shape *shape, const void *input, const void *offset, const void *mask,
                           const void *packed_weight, const void *bias, void *output, uint32_t *nonfinite_flag,
                           void *workspace, size_t workspace_bytes, dcn_stream stream) {
    return dcn_forward_f16_io(shape, nullptr, input, offset, mask, packed_weight, bias, output, nonfinite_flag,
                              workspace, workspace_bytes, stream);
}

dcn_status dcn_regroup_input_f16(const dcn_shape *shape, const void *input, void *workspace,
                                 size_t workspace_bytes, dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    const Params p = make_params(*shape);
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_DIRECT) return DCN_ERR_UNSUPPORTED;
    if (!input || !workspace || !aligned(input, 2) || !aligned(workspace, 256) ||
        workspace_bytes < dcn_forward_f16_workspace_bytes(shape))
        return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    const SplitInput<__half> in{static_cast<const __half *>(input), nullptr, p.C, p.C};
    return from_cuda(launch_regroup(path, p, in, workspace, reinterpret_cast<cudaStream_t>(stream)));
}

dcn_status dcn_regroup_input_nhwc_f16(const dcn_shape *shape, const void *input_nhwc, void *workspace,
                                      size_t workspace_bytes, dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    const Params p = make_params(*shape);
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_DIRECT) return DCN_ERR_UNSUPPORTED;
    if (!input_nhwc || !workspace || !aligned(input_nhwc, 16) || !aligned(workspace, 16) ||
        workspace_bytes < dcn_forward_f16_workspace_bytes(shape))
        return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    return from_cuda(launch_regroup_nhwc(path == DCN_PATH_SLAB_TC, p.N, p.OG, p.H, p.W,
                                         static_cast<const __half *>(input_nhwc), workspace,
                                         reinterpret_cast<cudaStream_t>(stream)));
}

dcn_status dcn_forward_f16_grouped(const dcn_shape *shape, void *input_grouped, const void *offset,
                                   const void *mask, const void *packed_weight, const void *bias, void *output,
                                   uint32_t *nonfinite_flag, dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    const Params p = make_params(*shape);
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_DIRECT) return DCN_ERR_UNSUPPORTED;
    if (!input_grouped || !offset || !mask || !packed_weight || !bias || !output) return DCN_ERR_INVALID_ARGUMENT;
    if (!aligned(input_grouped, 16) || !aligned(offset, 16) || !aligned(mask, 16) || !aligned(packed_weight, 16) ||
        !aligned(bias, 2) || !aligned(output, 2) || (nonfinite_flag && !aligned(nonfinite_flag, 4)))
        return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    return launch_grouped(path, p, input_grouped, offset, mask, packed_weight, bias, output, nonfinite_flag, dev,
                          reinterpret_cast<cudaStream_t>(stream));
}

dcn_status dcn_flag_non_finite_f16(const void *values, int64_t count, uint32_t *flag, dcn_stream stream) {
    if (!values || !flag || count <= 0 || !aligned(values, 2) || !aligned(flag, 4)) return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    dcn_status st = current_device(&dev);
    if (st != DCN_OK) return st;
    return from_cuda(launch_flag_non_finite(static_cast<const __half *>(values), count, flag, dev->sm_count,
                                            reinterpret_cast<cudaStream_t>(stream)));
}

dcn_status dcn_temporal_prepare_f16(int32_t batch, int32_t width, int32_t height, const void *feat_prop,
                                    const void *feat_current, const void *feat_n2, const void *flow1,
                                    const void *previous_flow, int32_t has_second_order, void *conditions,
                                    void *deform_input, void *flow2, dcn_stream stream) {
    // runTemporalPreparation's guard (MetalRunner.swift:520-527): positive extents; the counts
    // it checks are the caller's tensor sizes here.
    if (batch <= 0 || width <= 0 || height <= 0 ||
        static_cast<int64_t>(width) * height > (int64_t{1} << 31) / 256)
        return DCN_ERR_INVALID_SHAPE;
    const void *in[] = {feat_prop, feat_current, feat_n2, flow1, previous_flow, conditions, flow2};
    for (const void *q : in)
        if (q == nullptr || !aligned(q, 2)) return DCN_ERR_INVALID_ARGUMENT;
    if (deform_input != nullptr && !aligned(deform_input, 2)) return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    dcn_status st = current_device(&dev);
    if (st != DCN_OK) return st;
    return from_cuda(launch_temporal_prepare(
        batch, height, width, static_cast<const __half *>(feat_prop), static_cast<const __half *>(feat_current),
        static_cast<const __half *>(feat_n2), static_cast<const __half *>(flow1),
        static_cast<const __half *>(previous_flow), has_second_order != 0, static_cast<__half *>(conditions),
        static_cast<__half *>(deform_input), static_cast<__half *>(flow2), nullptr,
        reinterpret_cast<cudaStream_t>(stream)));
}

size_t dcn_temporal_slabs_bytes(int32_t batch, int32_t width, int32_t height) {
    if (batch <= 0 || width <= 0 || height <= 0 || temporal_staged_smem(height, width) == 0) return 0;
    return static_cast<size_t>(batch) * 16 * (height + 2) * (width + 2) * 16;
}

dcn_status dcn_temporal_prepare_slabs_f16(int32_t batch, int32_t width, int32_t height, const void *feat_prop,
                                          const void *feat_current, const void *feat_n2, const void *flow1,
                                          const void *previous_flow, int32_t has_second_order, void *conditions,
                                          void *flow2, void *workspace, size_t workspace_bytes,
                                          dcn_stream stream) {
    if (batch <= 0 || width <= 0 || height <= 0 ||
        static_cast<int64_t>(width) * height > (int64_t{1} << 31) / 256)
        return DCN_ERR_INVALID_SHAPE;
    // The slab form is written by the shared-memory kernel only: frames whose 4-channel slab fits
    // its 110 KB, with an even pixel count (16-byte plane copies).
    if (dcn_temporal_slabs_bytes(batch, width, height) == 0 || (static_cast<int64_t>(width) * height) % 2 != 0)
        return DCN_ERR_UNSUPPORTED;
    const void *planes[] = {feat_prop, feat_current, feat_n2, conditions};
    for (const void *q : planes)
        if (q == nullptr || !aligned(q, 16)) return DCN_ERR_INVALID_ARGUMENT;
    const void *flows[] = {flow1, previous_flow, flow2};
    for (const void *q : flows)
        if (q == nullptr || !aligned(q, 2)) return DCN_ERR_INVALID_ARGUMENT;
    if (workspace == nullptr || !aligned(workspace, 16) ||
        workspace_bytes < dcn_temporal_slabs_bytes(batch, width, height))
        return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    dcn_status st = current_device(&dev);
    if (st != DCN_OK) return st;
    return from_cuda(launch_temporal_prepare(
        batch, height, width, static_cast<const __half *>(feat_prop), static_cast<const __half *>(feat_current),
        static_cast<const __half *>(feat_n2), static_cast<const __half *>(flow1),
        static_cast<const __half *>(previous_flow), has_second_order != 0, static_cast<__half *>(conditions),
        nullptr, static_cast<__half *>(flow2), workspace, reinterpret_cast<cudaStream_t>(stream)));
}

dcn_status dcn_prepare_offsets_f16(int64_t plane, const void *raw, const void *flow1, const void *flow2,
                                   void *offset, void *mask, dcn_stream stream) {
    if (plane <= 0 || plane >= (int64_t{1} << 31) / 432) return DCN_ERR_INVALID_SHAPE;
    if (!raw || !flow1 || !flow2 || !offset || !mask) return DCN_ERR_INVALID_ARGUMENT;
    if (!aligned(raw, 2) || !aligned(flow1, 2) || !aligned(flow2, 2) || !aligned(offset, 2) || !aligned(mask, 2))
        return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    dcn_status st = current_device(&dev);
    if (st != DCN_OK) return st;
    return from_cuda(launch_prepare_offsets(1, 144, plane, static_cast<const __half *>(raw),
                                            static_cast<const __half *>(flow1), static_cast<const __half *>(flow2),
                                            static_cast<__half *>(offset), static_cast<__half *>(mask),
                                            reinterpret_cast<cudaStream_t>(stream)));
}

// Both tensor-core kernels make the offsets and masks inside their producers, so the raw
// form needs the same workspace as dcn_forward_f16 (the regrouped input, plus the partial
// sums of a group-split slab batch).
size_t dcn_forward_f16_raw_workspace_bytes(const dcn_shape *shape) {
    if (validate(shape) != DCN_OK) return 0;
    const Params p = make_params(*shape);
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_DIRECT || p.OG % 2 != 0) return 0;
    return dcn_forward_f16_workspace_bytes(shape);
}

dcn_status dcn_forward_f16_raw_io(const dcn_shape *shape, const dcn_io *io, const void *input, const void *raw,
                                  const void *flow1, const void *flow2, const void *packed_weight, const void *bias,
                                  void *output, uint32_t *nonfinite_flag, void *workspace, size_t workspace_bytes,
                                  dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    Params p = make_params(*shape);
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_DIRECT || p.OG % 2 != 0) return DCN_ERR_UNSUPPORTED;
    if (!input || !raw || !flow1 || !flow2 || !packed_weight || !bias || !output) return DCN_ERR_INVALID_ARGUMENT;
    if (!aligned(input, 2) || !aligned(raw, 16) || !aligned(flow1, 16) || !aligned(flow2, 16) ||
        !aligned(packed_weight, 16) || !aligned(bias, 2) || !aligned(output, 2) ||
        (nonfinite_flag && !aligned(nonfinite_flag, 4)))
        return DCN_ERR_INVALID_ARGUMENT;
    if (!workspace || !aligned(workspace, 256) || workspace_bytes < dcn_forward_f16_raw_workspace_bytes(shape))
        return DCN_ERR_INVALID_ARGUMENT;
    SplitInput<__half> in;
    if ((st = resolve_io(io, path, input, &p, &in)) != DCN_OK) return st;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const auto *r = static_cast<const __half *>(raw);
    const auto *f1 = static_cast<const __half *>(flow1);
    const auto *f2 = static_cast<const __half *>(flow2);
    cudaError_t e = launch_regroup(path, p, in, workspace, s);
    if (e != cudaSuccess) return from_cuda(e);
    const auto *w = static_cast<const uint8_t *>(packed_weight);
    const auto *b = static_cast<const __half *>(bias);
    auto *out = static_cast<__half *>(output);
    if (path == DCN_PATH_SLAB_TC)
        return from_cuda(launch_slab_grouped_raw(p, workspace, r, f1, f2, w, b, out, nonfinite_flag, dev->sm_count,
                                                 dev->err_word, s));
    return from_cuda(launch_fused_grouped_raw(p, workspace, r, f1, f2, w, b, out, nonfinite_flag, dev->sm_count,
                                              dev->err_word, s));
}

dcn_status dcn_forward_f16_raw_grouped(const dcn_shape *shape, void *workspace, const void *raw, const void *flow1,
                                       const void *flow2, const void *packed_weight, const void *bias, void *output,
                                       uint32_t *nonfinite_flag, size_t workspace_bytes, dcn_stream stream) {
    dcn_status st = validate(shape);
    if (st != DCN_OK) return st;
    const Params p = make_params(*shape);
    const dcn_path path = select_path(p);
    if (path == DCN_PATH_DIRECT || p.OG % 2 != 0) return DCN_ERR_UNSUPPORTED;
    if (!raw || !flow1 || !flow2 || !packed_weight || !bias || !output) return DCN_ERR_INVALID_ARGUMENT;
    if (!aligned(raw, 16) || !aligned(flow1, 16) || !aligned(flow2, 16) || !aligned(packed_weight, 16) ||
        !aligned(bias, 2) || !aligned(output, 2) || (nonfinite_flag && !aligned(nonfinite_flag, 4)))
        return DCN_ERR_INVALID_ARGUMENT;
    if (!workspace || !aligned(workspace, 16) || workspace_bytes < dcn_forward_f16_raw_workspace_bytes(shape))
        return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    if ((st = current_device(&dev)) != DCN_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const auto *r = static_cast<const __half *>(raw);
    const auto *f1 = static_cast<const __half *>(flow1);
    const auto *f2 = static_cast<const __half *>(flow2);
    const auto *w = static_cast<const uint8_t *>(packed_weight);
    const auto *b = static_cast<const __half *>(bias);
    auto *out = static_cast<__half *>(output);
    if (path == DCN_PATH_SLAB_TC)
        return from_cuda(launch_slab_grouped_raw(p, workspace, r, f1, f2, w, b, out, nonfinite_flag, dev->sm_count,
                                                 dev->err_word, s));
    return from_cuda(launch_fused_grouped_raw(p, workspace, r, f1, f2, w, b, out, nonfinite_flag, dev->sm_count,
                                              dev->err_word, s));
}

dcn_status dcn_forward_f16_raw(const dcn_shape *shape, const void *input, const void *raw, const void *flow1,
                               const void *flow2, const void *packed_weight, const void *bias, void *output,
                               uint32_t *nonfinite_flag, void *workspace, size_t workspace_bytes,
                               dcn_stream stream) {
    return dcn_forward_f16_raw_io(shape, nullptr, input, raw, flow1, flow2, packed_weight, bias, output,
                                  nonfinite_flag, workspace, workspace_bytes, stream);
}

dcn_status dcn_device_error(void) {
    DeviceInfo *dev = nullptr;
    dcn_status st = current_device(&dev);
    if (st != DCN_OK) return st;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return from_cuda(e);
    uint32_t word = 0;
    e = cudaMemcpy(&word, dev->err_word, sizeof(word), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return from_cuda(e);
    if (word != 0) {
        const uint32_t zero = 0;
        cudaMemcpy(dev->err_word, &zero, sizeof(zero), cudaMemcpyHostToDevice);
        return DCN_ERR_DEVICE_TIMEOUT;
    }
    return DCN_OK;
}

dcn_status dcn_check_wait_timeout(uint32_t limit_us, dcn_stream stream) {
    if (limit_us == 0 || limit_us > 10000000u) return DCN_ERR_INVALID_ARGUMENT;
    DeviceInfo *dev = nullptr;
    dcn_status st = current_device(&dev);
    if (st != DCN_OK) return st;
    return from_cuda(launch_check_wait_timeout(static_cast<uint64_t>(limit_us) * 1000u, dev->err_word,
                                               reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
