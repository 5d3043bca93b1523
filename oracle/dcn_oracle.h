/*
 * dcn_oracle.h -- CPU restatement of the reference DCNv2, used ONLY as the
 * parity checker by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * arm.  Nothing in the product library links or calls this code.
 *
 * Parity pin: the reference's own known-answer test
 * (Tests/JasnaMetalPoCTests/DeformConvCPUTests.swift:4-33, output [2,3,4,5]) is
 * reproduced bit-exactly by tests/test_oracle.py.  The Swift reference itself
 * cannot be built here (no Swift toolchain), so there is no compiled `_ref`.
 */
#ifndef DCN_ORACLE_H
#define DCN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field order as DeformConvShape (Sources/JasnaMetalPoC/DeformConv.swift:3-20)
 * and as dcn_shape in include/dcn_b200.h. */
typedef struct dcn_oracle_shape {
    int32_t batch, input_channels, input_height, input_width;
    int32_t output_channels, output_height, output_width;
    int32_t kernel_height, kernel_width;
    int32_t pad_height, pad_width, stride_height, stride_width;
    int32_t dilation_height, dilation_width;
    int32_t groups, offset_groups;
} dcn_oracle_shape;

/* 0 = ok, 1 = invalid shape (DeformConvShape.validate, DeformConv.swift:29-41). */
int dcn_oracle_validate(const dcn_oracle_shape *s);

/* DeformConvCPU.run (DeformConv.swift:76-138): single-threaded scalar loop in
 * the reference's order.  Returns 0 or 1 (invalid shape). */
int dcn_oracle_run(const dcn_oracle_shape *s, const float *input, const float *offset,
                   const float *mask, const float *weight, const float *bias, float *output);

/* The same loop over batch items [n_begin, n_end) only (output indexed as for
 * the whole batch).  Used to time or check a bounded sample of a large batch. */
int dcn_oracle_run_range(const dcn_oracle_shape *s, const float *input, const float *offset,
                         const float *mask, const float *weight, const float *bias, float *output,
                         int32_t n_begin, int32_t n_end);

/* Same results as dcn_oracle_run_range, bit for bit, with sampled * mask
 * evaluated once per (image, ic, tap, pixel) instead of once per output
 * channel (a pure subexpression of DeformConv.swift:117-128). */
int dcn_oracle_run_fast_range(const dcn_oracle_shape *s, const float *input, const float *offset,
                              const float *mask, const float *weight, const float *bias,
                              float *output, int32_t n_begin, int32_t n_end);

/* The range loop split over `threads` POSIX threads, one contiguous batch slice
 * per thread, each running the single-threaded loop (the reference is
 * single-threaded per tile); `fast` selects dcn_oracle_run_fast_range.
 * threads <= 0 means 1. */
int dcn_oracle_run_threads(const dcn_oracle_shape *s, const float *input, const float *offset,
                           const float *mask, const float *weight, const float *bias,
                           float *output, int32_t n_begin, int32_t n_end, int threads, int fast);

/* Bounded sample of the literal reference loop for CPU timing: output rows
 * [oy_begin, oy_end) of every image, the batch split over `threads` POSIX
 * threads (one contiguous slice each, single-threaded per image like the
 * reference).  Outputs outside the rows are left untouched. */
int dcn_oracle_run_sample(const dcn_oracle_shape *s, const float *input, const float *offset,
                          const float *mask, const float *weight, const float *bias,
                          float *output, int32_t oy_begin, int32_t oy_end, int threads);

/* prepare_dcn_offsets_fp16 restated in FP32 (MetalShader.swift:817-839; the
 * reference's own CPU check is JasnaCLI.swift:177-211).  raw [432][plane],
 * flow1/flow2 [2][plane] in (x, y) order -> offset [288][plane], mask [144][plane]. */
void dcn_oracle_prepare_offsets(int64_t plane, const float *raw, const float *flow1,
                                const float *flow2, float *offset, float *mask);

/* MetalDeformConv.runTemporalPreparation (MetalRunner.swift:510-582) for one width x height
 * frame: accumulate_second_order_flow_fp16 then assemble_temporal_alignment_fp16
 * (MetalShader.swift:736-813), restated the way the reference's own self-check computes its
 * expectations (JasnaCLI.swift:211-290, `sampleZero`): FP32 bilinear sampling with zero padding
 * of FP16 values, every stored result rounded to FP16 (round to nearest even), flow2 rounded
 * before it is used to warp feat_n2.  Inputs hold FP16 values widened to float:
 * feat_* [64][plane], flow1 / previous_flow [2][plane] in (x, y) order.  Outputs (floats
 * holding FP16 values): conditions [196][plane] = [warp(feat_prop, flow1), feat_current,
 * warp(feat_n2, flow2), flow1, flow2], deform_input [128][plane] = [feat_prop, feat_n2]
 * (may be NULL), flow2 [2][plane] (all zeros when has_second_order is 0). */
void dcn_oracle_temporal_prepare(int32_t width, int32_t height, const float *feat_prop,
                                 const float *feat_current, const float *feat_n2,
                                 const float *flow1, const float *previous_flow,
                                 int has_second_order, float *conditions, float *deform_input,
                                 float *flow2);

/* SplitMix64 step of SeededGenerator.next (DeformConv.swift:168-181). */
uint64_t dcn_oracle_splitmix64(uint64_t *state);

#ifdef __cplusplus
}
#endif

#endif
