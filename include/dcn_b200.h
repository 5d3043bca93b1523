/*
 * dcn_b200.h -- C ABI of the B200 (sm_100a) modulated deformable convolution (DCNv2).
 *
 * This is the drop-in boundary for the deformable-convolution operator of the
 * Jasna BasicVSR++ port (ken8303/jasnaMacOS).  Every entry point below replaces
 * one piece of the reference's Swift/Metal operator; the citation on each names
 * the reference file and line it stands in for (paths are relative to the
 * reference project root).
 *
 * Conventions
 *  - Plain C: pointers, sizes, one shape struct.  No CUDA, torch or C++ types.
 *  - All tensor pointers are DEVICE pointers owned by the caller, except the
 *    host buffers of dcn_forward_f16_host.  No device memory is allocated per
 *    call; kernels that need scratch take a caller-provided workspace sized by
 *    the matching *_workspace_bytes() query.
 *  - Every launch is asynchronous on the caller's stream (NULL = legacy default
 *    stream).  A status of DCN_OK means "validated and enqueued".  Errors that
 *    can only be seen on the device (non-finite output, a device-side pipeline
 *    timeout) are written to the caller's flag word and/or read back with
 *    dcn_device_error().
 *  - Layouts follow the reference (DeformConv.swift:110-132): NCHW input,
 *    offset [N][2*G*KH*KW][Ho][Wo] with (dy, dx) interleaved per (group, tap),
 *    mask [N][G*KH*KW][Ho][Wo], output NCHW.  FP32 weights are OIHW; packed
 *    weights are opaque (sized by dcn_packed_weight_bytes).
 *  - Thread safety: calls on distinct streams may run concurrently.  The only
 *    global state is a per-device attribute cache filled under a mutex (once per
 *    device and CUDA context: a new context after cudaDeviceReset refills it) and
 *    the sticky device error word.
 */
#ifndef DCN_B200_H
#define DCN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DCN_B200_ABI_VERSION 1

/* Same handle type as cudaStream_t / CUstream, without including CUDA headers. */
typedef struct CUstream_st *dcn_stream;

/* Mirrors `struct DeformConvShape` (Sources/JasnaMetalPoC/DeformConv.swift:3-20)
 * field for field and in the same order; `offset_groups` is the deformable-group
 * count.  The Metal constant block adds `hasMask` (MetalShader.swift:25); every
 * DCNv2 call in the reference passes a mask, so the mask pointer is simply
 * required here. */
typedef struct dcn_shape {
    int32_t batch;
    int32_t input_channels;
    int32_t input_height;
    int32_t input_width;
    int32_t output_channels;
    int32_t output_height;
    int32_t output_width;
    int32_t kernel_height;
    int32_t kernel_width;
    int32_t pad_height;
    int32_t pad_width;
    int32_t stride_height;
    int32_t stride_width;
    int32_t dilation_height;
    int32_t dilation_width;
    int32_t groups;
    int32_t offset_groups;
} dcn_shape;

/* Element counts derived from a shape (DeformConv.swift:22-27). */
typedef struct dcn_counts {
    int64_t input;
    int64_t offset;
    int64_t mask;
    int64_t weight;
    int64_t bias;
    int64_t output;
} dcn_counts;

/* Mirrors `enum DeformConvError` (DeformConv.swift:44-73).  The reference's
 * .metalUnavailable / .shaderResourceMissing become DCN_ERR_NO_DEVICE /
 * DCN_ERR_UNSUPPORTED; .commandFailed becomes DCN_ERR_LAUNCH (launch error) or
 * DCN_ERR_DEVICE_TIMEOUT (a bounded device-side wait gave up). */
typedef enum dcn_status {
    DCN_OK = 0,
    DCN_ERR_INVALID_SHAPE = 1,    /* .invalidShape        DeformConv.swift:29-41 */
    DCN_ERR_INVALID_COUNT = 2,    /* .invalidArrayCount   DeformConv.swift:140-144 */
    DCN_ERR_NO_DEVICE = 3,        /* .metalUnavailable    MetalRunner.swift:108-110 */
    DCN_ERR_UNSUPPORTED = 4,      /* .shaderResourceMissing / shape guards MetalRunner.swift:630-713 */
    DCN_ERR_NONFINITE = 5,        /* .nonFiniteOutput     DeformConv.swift:49,52-55 (the only recoverable one) */
    DCN_ERR_LAUNCH = 6,           /* .commandFailed       MetalRunner.swift:619-621 */
    DCN_ERR_INVALID_ARGUMENT = 7, /* NULL pointer / misaligned pointer / short workspace */
    DCN_ERR_DEVICE_TIMEOUT = 8,   /* a device-side bounded wait expired (pipeline error) */
    DCN_ERR_SCRATCH_TOO_SMALL = 9 /* the problem needs more than the library's static scratch */
} dcn_status;

typedef enum dcn_dtype {
    DCN_DTYPE_F32 = 0,
    DCN_DTYPE_F16 = 1
} dcn_dtype;

typedef enum dcn_weight_layout {
    DCN_WEIGHT_OIHW = 0,      /* [oc][ic/groups][kh][kw]: the direct kernels' layout (MetalShader.swift:118) */
    DCN_WEIGHT_IC_K_OC = 1    /* [ic][kh*kw][oc]: the reference's prepacked .dcnfp16 layout
                                 (tools/export_deform_weights.py:47, MetalShader.swift:226-229) */
} dcn_weight_layout;

/* Bits of the caller's uint32 flag word written by dcn_forward_f16 /
 * dcn_flag_non_finite_f16 (mirrors flag_non_finite_fp16, MetalShader.swift:454-463). */
#define DCN_FLAG_NONFINITE 1u

/* Implementation selected by dcn_forward_f16 for a given shape. */
typedef enum dcn_path {
    DCN_PATH_DIRECT = 0,      /* CUDA-core direct kernel (any valid shape) */
    DCN_PATH_FUSED_TC = 1,    /* sm_100a fused gather + tcgen05 implicit GEMM, gathers from
                                 global memory (any image size) */
    DCN_PATH_SLAB_TC = 2      /* the same operator with each deformable group's input staged
                                 whole in shared memory (3x3 kernels, images up to ~69x69) */
} dcn_path;

/* ---- status / shape helpers ------------------------------------------------ */

/* Human-readable text for a status (DeformConvError.description, DeformConv.swift:57-72). */
const char *dcn_status_string(dcn_status status);

/* 1 for the only recoverable numerical failure, DCN_ERR_NONFINITE
 * (DeformConvError.isRecoverableNumericalFailure, DeformConv.swift:52-55), else 0. */
int dcn_status_is_recoverable(dcn_status status);

/* DeformConvShape.validate() (DeformConv.swift:29-41), plus the limits of this
 * implementation: planes below 2^31 elements, kernel area <= 1024, sampling
 * positions whose integer part stays below 2^30 in magnitude, tensors below
 * 2^40 elements.  Strides, pads and dilations may take any value the reference
 * accepts.  Returns DCN_OK or DCN_ERR_INVALID_SHAPE. */
dcn_status dcn_shape_validate(const dcn_shape *shape);

/* Element counts of every tensor (DeformConv.swift:22-27). */
dcn_status dcn_shape_counts(const dcn_shape *shape, dcn_counts *out);

/* Array-count check of DeformConvCPU.require (DeformConv.swift:85-89,140-144).
 * On DCN_ERR_INVALID_COUNT, *which_out (if non-NULL) gets 0..4 for
 * input/offset/mask/weight/bias. */
dcn_status dcn_check_counts(const dcn_shape *shape, int64_t input_count, int64_t offset_count,
                            int64_t mask_count, int64_t weight_count, int64_t bias_count,
                            int *which_out);

/* Version of this ABI (DCN_B200_ABI_VERSION). */
int dcn_abi_version(void);

/* ---- FP32 path ----------------------------------------------------------------
 * Replaces MetalDeformConv.runFloat32 + deform_conv2d_fp32
 * (MetalRunner.swift:159-185, MetalShader.swift:76-124).  Any valid shape.
 * Every output is accumulated in the reference's order (bias, then ic, ky, kx)
 * with IEEE fp32 multiply/add and no fused multiply-add, so it is bit-identical
 * to DeformConvCPU.run (DeformConv.swift:98-136). */
dcn_status dcn_forward_f32(const dcn_shape *shape, const float *input, const float *offset,
                           const float *mask, const float *weight_oihw, const float *bias,
                           float *output, dcn_stream stream);

/* ---- FP16 direct path --------------------------------------------------------
 * Replaces deform_conv2d_fp16 (MetalShader.swift:126-174): FP16 storage, FP32
 * math in the reference order, one rounding to FP16 at the end.  OIHW FP16
 * weights, FP16 bias.  Any valid shape.  This is the cross-variant baseline the
 * reference gates its fast FP16 kernels against (MetalRunner.swift:338-354). */
dcn_status dcn_forward_f16_direct(const dcn_shape *shape, const void *input, const void *offset,
                                  const void *mask, const void *weight_oihw, const void *bias,
                                  void *output, dcn_stream stream);

/* ---- weight prepack ---------------------------------------------------------
 * Replaces the offline OIHW -> [ic][k][oc] FP16 pack (tools/export_deform_weights.py:47-48,
 * MetalRunner.swift:235-243).  Produces the opaque packed weight consumed by
 * dcn_forward_f16: for shapes that take the fused path it is the tcgen05 B
 * operand (K-major, 128-byte swizzled); otherwise an OIHW FP16 copy.
 * `weight` is FP32 or FP16 (src_dtype) in OIHW or IC_K_OC layout (src_layout). */
size_t dcn_packed_weight_bytes(const dcn_shape *shape);
dcn_status dcn_prepack_weights(const dcn_shape *shape, const void *weight, dcn_dtype src_dtype,
                               dcn_weight_layout src_layout, void *packed, dcn_stream stream);

/* Which implementation dcn_forward_f16 runs for this shape.  The choice between the
 * two tensor-core kernels can be pinned for a process with the environment
 * variable DCN_B200_FUSED_KERNEL=slab|pairs (default: slab where it applies),
 * read once; packed weights and workspaces must come from the same process. */
dcn_path dcn_forward_f16_path(const dcn_shape *shape);

/* How dcn_forward_f16 (and the raw form) launches a shape on the current device, for
 * schedulers and profilers; no counterpart in the reference, whose host dispatches one
 * Metal kernel per call.
 *   path            as dcn_forward_f16_path
 *   group_splits    slab path: deformable-group ranges per tile (> 1: a reduction pass
 *                   adds the FP32 partial sums; DCN_B200_GROUP_SPLIT=0 turns it off)
 *   tiles_per_unit  tensor-core paths: 128-pixel tiles per work unit
 *   grid            CTAs of the tensor-core (or direct) kernel
 *   prepass_images  images the regroup pre-pass converts before the kernel
 *   launches        kernel launches per call (without the direct path's non-finite
 *                   flag pass) */
typedef struct dcn_plan {
    int32_t path;
    int32_t group_splits;
    int32_t tiles_per_unit;
    int32_t launches;
    int64_t grid;
    int64_t prepass_images;
} dcn_plan;
dcn_status dcn_forward_f16_plan(const dcn_shape *shape, dcn_plan *out);

/* ---- fused FP16 path ----------------------------------------------------------
 * Replaces deform_conv2d_fp16_jasna_gather + deform_conv2d_fp16_jasna_simdgroup_gemm_fused
 * + flag_non_finite_fp16 (MetalShader.swift:299-463; host MetalRunner.swift:696-761;
 * production binding FusedFourPassRecurrenceProbe.swift:609-630).
 * input/offset/mask/bias/output FP16; packed_weight from dcn_prepack_weights.
 * `nonfinite_flag` (nullable) gets DCN_FLAG_NONFINITE OR-ed in when any output
 * is Inf/NaN; the caller zeroes it.  `workspace` must hold
 * dcn_forward_f16_workspace_bytes(shape) bytes (256-byte aligned); it is
 * scratch, overwritten by every call. */
size_t dcn_forward_f16_workspace_bytes(const dcn_shape *shape);
dcn_status dcn_forward_f16(const dcn_shape *shape, const void *input, const void *offset,
                           const void *mask, const void *packed_weight, const void *bias,
                           void *output, uint32_t *nonfinite_flag, void *workspace,
                           size_t workspace_bytes, dcn_stream stream);

/* The two launches dcn_forward_f16 makes, for callers that keep their features
 * channels-last and for timing the tensor-core kernel alone.
 * dcn_regroup_input_f16: NCHW FP16 input -> the grouped channels-last layout of the
 *   selected path at the start of `workspace` (dcn_forward_f16_workspace_bytes bytes),
 *   8 channels of one deformable group per 16 bytes:
 *     DCN_PATH_SLAB_TC  zero-bordered per-group slabs [N][C/8][H+2][W+2][8] FP16, element
 *                       (n, g, y+1, x+1, c) = input[n][8g+c][y][x], the one-pixel ring zero;
 *     DCN_PATH_FUSED_TC horizontal corner pairs [N][C/8][H][W+1] of 32 bytes: entry
 *                       (n, g, y, x) = the 8 channels at column x-1, then at column x
 *                       (zeros outside the image).
 *   A producer that writes its features in this layout itself (the reference assembles
 *   the DCN input in its own kernel, MetalShader.swift:769-813) can skip the pre-pass and
 *   call dcn_forward_f16_grouped directly.
 * dcn_forward_f16_grouped: the tensor-core kernel reading such an input from the
 *   start of a workspace (16-byte aligned, dcn_forward_f16_workspace_bytes bytes): on
 *   the slab path, batches with fewer 128-pixel tiles than the B200 has SMs split the
 *   deformable groups across SMs and keep FP32 partial sums in the workspace past the
 *   regrouped input, then add them in a fixed order in a second launch.  Results are
 *   deterministic for a shape; an image computed in a split batch can differ from the
 *   same image in a large batch by one FP16 rounding step (another FP32 summation
 *   order).  DCN_B200_GROUP_SPLIT=0 in the environment (read once per process) turns
 *   the split off, making every image's result independent of its batch.
 * Both return DCN_ERR_UNSUPPORTED for DCN_PATH_DIRECT shapes. */
dcn_status dcn_regroup_input_f16(const dcn_shape *shape, const void *input, void *workspace,
                                 size_t workspace_bytes, dcn_stream stream);
dcn_status dcn_forward_f16_grouped(const dcn_shape *shape, void *input_grouped,
                                   const void *offset, const void *mask, const void *packed_weight,
                                   const void *bias, void *output, uint32_t *nonfinite_flag,
                                   dcn_stream stream);

/* dcn_regroup_input_nhwc_f16: dcn_regroup_input_f16 for an input stored channels-last,
 *   [N][H][W][C] FP16 (16-byte aligned; the reference's tensors are NCHW,
 *   DeformConv.swift:110-132).  It writes the same bytes at the start of the workspace, so
 *   dcn_forward_f16_grouped or dcn_forward_f16_raw_grouped follows unchanged.  Tensor-core
 *   paths only (DCN_ERR_UNSUPPORTED for DCN_PATH_DIRECT shapes); workspace 16-byte aligned and
 *   at least dcn_forward_f16_workspace_bytes(shape). */
dcn_status dcn_regroup_input_nhwc_f16(const dcn_shape *shape, const void *input_nhwc, void *workspace,
                                      size_t workspace_bytes, dcn_stream stream);

/* ---- FP16 operator on host buffers ----------------------------------------------
 * Replaces the reference's host-array contract: MetalDeformConv.runFloat32 takes Swift
 * arrays and returns a new array (MetalRunner.swift:159-185), copying the inputs into fresh
 * shared buffers on every call (makeBuffer, :584-593).  Here input, offset, mask and output
 * are HOST buffers in the layouts above (FP16); packed_weight and bias are device buffers as
 * for dcn_forward_f16.  The batch is cut into chunks of `chunk_images` images (0: 64) and
 * the chunks are pipelined on the library's own per-device streams -- up to three chunks in
 * flight, each chunk's input copies (one cudaMemcpyAsync per tensor), dcn_forward_f16 and
 * output copy in order on one stream -- so host->device copies, kernels and device->host
 * copies overlap.  Host buffers should be page-locked (cudaHostAlloc / cudaHostRegister);
 * pageable memory works but the copies then do not overlap.  `workspace` is device memory
 * of dcn_forward_f16_host_workspace_bytes(shape, chunk_images) bytes (256-byte aligned):
 * the staging buffers of the chunks in flight; the call allocates no device memory (its
 * streams and events are created once per device and context).  The call is ordered after
 * earlier work on `stream` and `stream` waits for all of it: once `stream` reaches that
 * point, output_host holds the result and *nonfinite_flag_host (host memory, nullable) is
 * DCN_FLAG_NONFINITE if any output is Inf/NaN, else 0.  Tensor-core-path shapes only (else
 * DCN_ERR_UNSUPPORTED).  Concurrent calls on one device are enqueued one after another. */
size_t dcn_forward_f16_host_workspace_bytes(const dcn_shape *shape, int32_t chunk_images);
dcn_status dcn_forward_f16_host(const dcn_shape *shape, const void *input_host, const void *offset_host,
                                const void *mask_host, const void *packed_weight, const void *bias,
                                void *output_host, uint32_t *nonfinite_flag_host, int32_t chunk_images,
                                void *workspace, size_t workspace_bytes, dcn_stream stream);

/* ---- offset producer fused into the convolution ------------------------------------
 * prepare_dcn_offsets_fp16 (MetalShader.swift:817-839) followed by the DCN, as the
 * production graph chains them (FusedFourPassRecurrenceProbe.swift:609-630), in one
 * operator: `raw` is the offset network's output [N][3*G*KH*KW][Ho][Wo] FP16 (2*G*KH*KW
 * offset residues, then G*KH*KW mask logits; 432 channels for Jasna), flow1/flow2 are
 * [N][2][Ho][Wo] FP16 in (x, y) order.  offset = FP16(10*tanh(residue) + flow) with dy
 * channels taking the flow's y row and deformable groups [0, G/2) flow1, the rest flow2;
 * mask = FP16(sigmoid(logit)).  On both tensor-core paths the transform runs inside the
 * convolution's producers and the offset/mask tensors never exist in memory; the
 * workspace is the one dcn_forward_f16 takes.  Requires an even G and a tensor-core path
 * (else DCN_ERR_UNSUPPORTED); raw and flows 16-byte aligned. */
size_t dcn_forward_f16_raw_workspace_bytes(const dcn_shape *shape);
dcn_status dcn_forward_f16_raw(const dcn_shape *shape, const void *input, const void *raw,
                               const void *flow1, const void *flow2, const void *packed_weight,
                               const void *bias, void *output, uint32_t *nonfinite_flag,
                               void *workspace, size_t workspace_bytes, dcn_stream stream);
/* The raw form on an input already in its path's grouped layout at the start of
 * `workspace` (written by dcn_regroup_input_f16 or by dcn_temporal_prepare_slabs_f16):
 * dcn_forward_f16_raw without its pre-pass, as dcn_forward_f16_grouped is dcn_forward_f16
 * without it.  workspace 16-byte aligned, workspace_bytes at least
 * dcn_forward_f16_raw_workspace_bytes(shape); the grouped input is read, not changed. */
dcn_status dcn_forward_f16_raw_grouped(const dcn_shape *shape, void *workspace, const void *raw,
                                       const void *flow1, const void *flow2,
                                       const void *packed_weight, const void *bias, void *output,
                                       uint32_t *nonfinite_flag, size_t workspace_bytes,
                                       dcn_stream stream);

/* ---- tensor plumbing: split input, output slot --------------------------------
 * Where the FP16 operator reads its input channels and writes its output channels,
 * for callers whose tensors are not exactly [N][C][H][W] in / [N][OC][Ho][Wo] out:
 *  - input_second != NULL: `input` holds channels [0, input_split) as
 *    [N][input_split][H][W] and input_second holds [input_split, C) as
 *    [N][C - input_split][H][W].  This replaces the deformInput = [feat_prop, feat_n2]
 *    concatenation of assemble_temporal_alignment_fp16 (MetalShader.swift:769-813):
 *    the two 64-channel features are read in place.  On the tensor-core paths
 *    input_split must be a multiple of 8 (one deformable group never straddles the
 *    two tensors); the direct path takes any split in [1, C-1].  With
 *    input_second == NULL, input_split must be 0.
 *  - output_image_channels != 0: the output tensor has output_image_channels
 *    channels per image and the operator writes channels
 *    [output_channel_offset, output_channel_offset + OC) of it, leaving the others
 *    untouched.  This replaces the copy of the aligned feature into the backbone
 *    input of assemble_temporal_backbone_fp16 (MetalShader.swift:903-929; slot
 *    64 * (branch + 1) of a 64 * (branch + 2)-channel tensor).  With
 *    output_image_channels == 0 the output is the plain [N][OC][Ho][Wo] and
 *    output_channel_offset must be 0.
 * A NULL dcn_io means all defaults (dcn_forward_f16 and dcn_forward_f16_raw pass NULL).
 * Invalid combinations return DCN_ERR_INVALID_ARGUMENT. */
typedef struct dcn_io {
    const void *input_second;
    int32_t input_split;
    int32_t output_image_channels;
    int32_t output_channel_offset;
} dcn_io;

dcn_status dcn_forward_f16_io(const dcn_shape *shape, const dcn_io *io, const void *input,
                              const void *offset, const void *mask, const void *packed_weight,
                              const void *bias, void *output, uint32_t *nonfinite_flag,
                              void *workspace, size_t workspace_bytes, dcn_stream stream);
dcn_status dcn_forward_f16_raw_io(const dcn_shape *shape, const dcn_io *io, const void *input,
                                  const void *raw, const void *flow1, const void *flow2,
                                  const void *packed_weight, const void *bias, void *output,
                                  uint32_t *nonfinite_flag, void *workspace, size_t workspace_bytes,
                                  dcn_stream stream);

/* ---- non-finite detection -----------------------------------------------------
 * flag_non_finite_fp16 (MetalShader.swift:454-463): ORs DCN_FLAG_NONFINITE into
 * *flag if any of `count` FP16 values is Inf or NaN. */
dcn_status dcn_flag_non_finite_f16(const void *values, int64_t count, uint32_t *flag,
                                   dcn_stream stream);

/* ---- offset / mask producer ---------------------------------------------------
 * prepare_dcn_offsets_fp16 (MetalShader.swift:817-839; host MetalRunner.swift:469-508):
 * raw [432][plane] (288 offset-residue channels then 144 mask logits), flow1 and
 * flow2 [2][plane] ((x, y) order) -> offset [288][plane] = 10*tanh(raw) + the
 * flipped flow, mask [144][plane] = sigmoid(raw).  All FP16. */
dcn_status dcn_prepare_offsets_f16(int64_t plane, const void *raw, const void *flow1,
                                   const void *flow2, void *offset, void *mask, dcn_stream stream);

/* ---- temporal preparation (the producers in front of the DCN) -----------------
 * MetalDeformConv.runTemporalPreparation (MetalRunner.swift:510-582), i.e. the kernels
 * accumulate_second_order_flow_fp16 + assemble_temporal_alignment_fp16
 * (MetalShader.swift:736-813), for `batch` frames of width x height (the reference takes one
 * frame).  Per frame, all FP16: feat_prop, feat_current, feat_n2 [64][H][W]; flow1 and
 * previous_flow [2][H][W] in (x, y) order ->
 *   flow2 [2][H][W]         = flow1 + warp(previous_flow, flow1) when has_second_order, else 0;
 *   conditions [196][H][W]  = [warp(feat_prop, flow1), feat_current, warp(feat_n2, flow2),
 *                              flow1, flow2] (the offset network's input);
 *   deform_input [128][H][W] = [feat_prop, feat_n2] (the DCN's input; nullable: the DCN entry
 *                              points read the two tensors directly through dcn_io).
 * warp() is bilinear sampling with zero padding at (y + flow_y, x + flow_x) in FP32 on the FP16
 * values, rounded to FP16 (flow2 is rounded before it warps feat_n2), as the reference computes
 * it.  Frames are contiguous in every tensor. */
dcn_status dcn_temporal_prepare_f16(int32_t batch, int32_t width, int32_t height, const void *feat_prop,
                                    const void *feat_current, const void *feat_n2, const void *flow1,
                                    const void *previous_flow, int32_t has_second_order, void *conditions,
                                    void *deform_input, void *flow2, dcn_stream stream);

/* The same preparation with the deform input [feat_prop, feat_n2] written in the layout the
 * DCN's slab kernel reads (dcn_regroup_input_f16's DCN_PATH_SLAB_TC layout for the
 * 128-channel, 16-group Jasna shape: slabs [batch][16][H+2][W+2][8] FP16, zero ring
 * included) at the start of `workspace`, instead of as an NCHW tensor.  This is where
 * assemble_temporal_alignment_fp16 writes the DCN's input in the reference
 * (MetalShader.swift:769-813); writing it here in the DCN's own layout lets the DCN skip its
 * regroup pre-pass: pass the same workspace to dcn_forward_f16_grouped or
 * dcn_forward_f16_raw_grouped.  The bytes equal what dcn_regroup_input_f16 makes of the
 * NCHW deform input.  dcn_temporal_slabs_bytes gives the slab bytes (0 for frames this form
 * does not take: the form needs the shared-memory kernel, (H+2)(W+2) <= 14,080, which covers
 * every frame the slab kernel takes); it returns DCN_ERR_UNSUPPORTED for those and for an odd
 * pixel count.  feat_prop, feat_current, feat_n2, conditions and workspace 16-byte aligned;
 * workspace_bytes at least dcn_temporal_slabs_bytes (the DCN entry points want their own
 * workspace size, which is at least that). */
size_t dcn_temporal_slabs_bytes(int32_t batch, int32_t width, int32_t height);
dcn_status dcn_temporal_prepare_slabs_f16(int32_t batch, int32_t width, int32_t height,
                                          const void *feat_prop, const void *feat_current,
                                          const void *feat_n2, const void *flow1,
                                          const void *previous_flow, int32_t has_second_order,
                                          void *conditions, void *flow2, void *workspace,
                                          size_t workspace_bytes, dcn_stream stream);

/* ---- fused FP16 path without any caller allocation ----------------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory when they run the convolution (allocator-less or real-time regions,
 * plugin hosts that own every device allocation): the same operator as
 * dcn_forward_f16, but its scratch is a fixed array inside the library
 * (dcn_static_scratch_bytes() = 16 MiB, held on every GPU that loads the
 * library until the process exits), so the caller passes only inputs and outputs.
 * Tensor-core-path shapes only (else DCN_ERR_UNSUPPORTED); a problem whose
 * scratch exceeds the array returns DCN_ERR_SCRATCH_TOO_SMALL (16 MiB holds 15
 * Jasna 64x64 tiles on the slab path, 7 on the global-gather path).  All calls share the array, so calls that overlap on the GPU race
 * and must be ordered (one stream, or events).  The first call on a device looks
 * up the array's address; make it before any stream capture (one warm-up call at
 * start-up does it).  The address is kept per device and context and looked up
 * again in a new context (after cudaDeviceReset).  Allocates nothing. */
size_t dcn_static_scratch_bytes(void);
dcn_status dcn_forward_f16_static_scratch(const dcn_shape *shape, const void *input,
                                          const void *offset, const void *mask,
                                          const void *packed_weight, const void *bias,
                                          void *output, uint32_t *nonfinite_flag,
                                          dcn_stream stream);

/* ---- device error word ----------------------------------------------------------
 * Every kernel with a bounded device-side wait records a timeout in a sticky
 * per-device word instead of trapping.  Returns DCN_OK or DCN_ERR_DEVICE_TIMEOUT
 * for the current device and clears the word (synchronises the device). */
dcn_status dcn_device_error(void);

/* A check of that failure path, with no counterpart in the reference: one CTA waits, with
 * the operator kernels' bounded-wait code and a limit of `limit_us` microseconds (1 to
 * 10,000,000), on an mbarrier that nothing arrives on.  The wait must run out and record
 * the timeout in the device error word, so that the next dcn_device_error() returns
 * DCN_ERR_DEVICE_TIMEOUT while the CUDA context stays usable.  Asynchronous on `stream`. */
dcn_status dcn_check_wait_timeout(uint32_t limit_us, dcn_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* DCN_B200_H */
