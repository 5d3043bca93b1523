/*
 * dcn_oracle.c -- CPU restatement of the reference DCNv2 (TEST INFRASTRUCTURE).
 *
 * Used only as the checker by tests/, __graft_entry__.smoke() and the CPU
 * baseline arm of bench.py; the product library never links it.
 *
 * Follows Sources/JasnaMetalPoC/DeformConv.swift:75-166 step for step:
 *   - loop nest n -> oc -> oy -> ox -> localIC -> ky -> kx (:98-136),
 *   - `sum = bias[oc]` first, then `sum += sampled * mask * weight` evaluated
 *     left to right as ((sampled * mask) * weight) (:103, :128),
 *   - bilinear corners zero outside the image and the left-to-right sum
 *     v00(1-ly)(1-lx) + v01(1-ly)lx + v10 ly(1-lx) + v11 ly lx (:146-165).
 * Build with -O2 -ffp-contract=off (no -ffast-math, no FMA contraction) so every
 * operation is one IEEE binary32 rounding, as in the Swift code.
 *
 * One documented divergence: Swift's Int(floor(y)) traps for NaN or positions
 * beyond the Int range.  Here floor(y) is converted with int32 saturation
 * (NaN -> 0), which is also what the CUDA kernels do (cvt.rmi.s32.f32), so the
 * oracle and the GPU path agree on inputs the reference rejects.
 */
#include "dcn_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>

/* DeformConvShape.validate (DeformConv.swift:29-41). */
int dcn_oracle_validate(const dcn_oracle_shape *s) {
    if (!(s->batch > 0 && s->input_channels > 0 && s->output_channels > 0 &&
          s->input_height > 0 && s->input_width > 0 && s->output_height > 0 &&
          s->output_width > 0 && s->kernel_height > 0 && s->kernel_width > 0 &&
          s->groups > 0 && s->offset_groups > 0 &&
          s->input_channels % s->groups == 0 && s->output_channels % s->groups == 0 &&
          s->input_channels % s->offset_groups == 0))
        return 1;
    return 0;
}

/* Int(floor(v)) with int32 saturation and NaN -> 0 (see header note). */
static int64_t floor_to_int_sat(float v) {
    float f = floorf(v);
    if (f != f) return 0;
    if (f >= 2147483648.0f) return 2147483647;
    if (f < -2147483648.0f) return -2147483648LL;
    return (int64_t)f;
}

/* DeformConvCPU.bilinear (DeformConv.swift:146-165). */
static float bilinear(const float *input, int64_t base, int64_t height, int64_t width, float y,
                      float x) {
    int64_t y0 = floor_to_int_sat(y);
    int64_t x0 = floor_to_int_sat(x);
    int64_t y1 = y0 + 1;
    int64_t x1 = x0 + 1;
    float ly = y - (float)y0;
    float lx = x - (float)x0;
#define VALUE(yy, xx)                                                                    \
    (((yy) >= 0 && (yy) < height && (xx) >= 0 && (xx) < width) ? input[base + (yy)*width + (xx)] \
                                                              : 0.0f)
    float v00 = VALUE(y0, x0);
    float v01 = VALUE(y0, x1);
    float v10 = VALUE(y1, x0);
    float v11 = VALUE(y1, x1);
#undef VALUE
    float t0 = v00 * (1.0f - ly);
    t0 = t0 * (1.0f - lx);
    float t1 = v01 * (1.0f - ly);
    t1 = t1 * lx;
    float t2 = v10 * ly;
    t2 = t2 * (1.0f - lx);
    float t3 = v11 * ly;
    t3 = t3 * lx;
    float r = t0 + t1;
    r = r + t2;
    r = r + t3;
    return r;
}

/* DeformConvCPU.run loop body (DeformConv.swift:98-136) for batch items
 * [n_begin, n_end) and output rows [oy_begin, oy_end). */
static int run_literal(const dcn_oracle_shape *s, const float *input, const float *offset,
                       const float *mask, const float *weight, const float *bias, float *output,
                       int32_t n_begin, int32_t n_end, int32_t oy_begin, int32_t oy_end) {
    if (dcn_oracle_validate(s)) return 1;
    const int64_t channels_per_group = s->input_channels / s->groups;
    const int64_t outputs_per_group = s->output_channels / s->groups;
    const int64_t channels_per_offset_group = s->input_channels / s->offset_groups;
    const int64_t output_plane = (int64_t)s->output_height * s->output_width;
    const int64_t input_plane = (int64_t)s->input_height * s->input_width;
    const int64_t kernel_area = (int64_t)s->kernel_height * s->kernel_width;
    if (n_begin < 0) n_begin = 0;
    if (n_end > s->batch) n_end = s->batch;

    for (int64_t n = n_begin; n < n_end; ++n) {
        for (int64_t oc = 0; oc < s->output_channels; ++oc) {
            const int64_t group = oc / outputs_per_group;
            for (int64_t oy = oy_begin; oy < oy_end; ++oy) {
                for (int64_t ox = 0; ox < s->output_width; ++ox) {
                    float sum = bias[oc];
                    for (int64_t local_ic = 0; local_ic < channels_per_group; ++local_ic) {
                        const int64_t ic = group * channels_per_group + local_ic;
                        const int64_t offset_group = ic / channels_per_offset_group;
                        for (int64_t ky = 0; ky < s->kernel_height; ++ky) {
                            for (int64_t kx = 0; kx < s->kernel_width; ++kx) {
                                const int64_t kernel_index = ky * s->kernel_width + kx;
                                const int64_t offset_channel =
                                    2 * (offset_group * kernel_area + kernel_index);
                                const int64_t spatial = oy * s->output_width + ox;
                                const int64_t offset_base =
                                    n * 2 * s->offset_groups * kernel_area * output_plane;
                                const float offset_y =
                                    offset[offset_base + offset_channel * output_plane + spatial];
                                const float offset_x =
                                    offset[offset_base + (offset_channel + 1) * output_plane +
                                           spatial];
                                const float y =
                                    (float)(oy * s->stride_height - s->pad_height +
                                            ky * s->dilation_height) +
                                    offset_y;
                                const float x =
                                    (float)(ox * s->stride_width - s->pad_width +
                                            kx * s->dilation_width) +
                                    offset_x;
                                const float sampled =
                                    bilinear(input, (n * s->input_channels + ic) * input_plane,
                                             s->input_height, s->input_width, y, x);
                                const int64_t mask_base =
                                    n * s->offset_groups * kernel_area * output_plane;
                                const int64_t mask_index =
                                    mask_base +
                                    (offset_group * kernel_area + kernel_index) * output_plane +
                                    spatial;
                                const int64_t weight_index =
                                    ((oc * channels_per_group + local_ic) * s->kernel_height +
                                     ky) * s->kernel_width +
                                    kx;
                                float term = sampled * mask[mask_index];
                                term = term * weight[weight_index];
                                sum = sum + term;
                            }
                        }
                    }
                    output[((n * s->output_channels + oc) * s->output_height + oy) *
                               s->output_width +
                           ox] = sum;
                }
            }
        }
    }
    return 0;
}

int dcn_oracle_run_range(const dcn_oracle_shape *s, const float *input, const float *offset,
                         const float *mask, const float *weight, const float *bias, float *output,
                         int32_t n_begin, int32_t n_end) {
    return run_literal(s, input, offset, mask, weight, bias, output, n_begin, n_end, 0,
                       s->output_height);
}

int dcn_oracle_run(const dcn_oracle_shape *s, const float *input, const float *offset,
                   const float *mask, const float *weight, const float *bias, float *output) {
    return dcn_oracle_run_range(s, input, offset, mask, weight, bias, output, 0, s->batch);
}

/* The same arithmetic as dcn_oracle_run_range, reorganised for speed: the
 * pure subexpression sampled * mask of DeformConv.swift:117-128 is evaluated
 * once per (image, ic, tap, pixel) instead of once per output channel, then
 * every output is summed in the reference order (bias, ic, ky, kx) with the
 * same roundings.  Results are bit-identical to the literal loop (checked by
 * tests/test_oracle.py); pixels are processed in blocks of `block` to bound
 * the scratch (C * KA * block floats). */
int dcn_oracle_run_fast_range(const dcn_oracle_shape *s, const float *input, const float *offset,
                              const float *mask, const float *weight, const float *bias,
                              float *output, int32_t n_begin, int32_t n_end) {
    if (dcn_oracle_validate(s)) return 1;
    const int64_t channels_per_group = s->input_channels / s->groups;
    const int64_t outputs_per_group = s->output_channels / s->groups;
    const int64_t channels_per_offset_group = s->input_channels / s->offset_groups;
    const int64_t output_plane = (int64_t)s->output_height * s->output_width;
    const int64_t input_plane = (int64_t)s->input_height * s->input_width;
    const int64_t kernel_area = (int64_t)s->kernel_height * s->kernel_width;
    const int64_t block = 1024;
    float *sm = (float *)malloc(sizeof(float) * (size_t)(s->input_channels * kernel_area * block));
    if (!sm) return 2;
    if (n_begin < 0) n_begin = 0;
    if (n_end > s->batch) n_end = s->batch;
    for (int64_t n = n_begin; n < n_end; ++n) {
        const int64_t offset_base = n * 2 * s->offset_groups * kernel_area * output_plane;
        const int64_t mask_base = n * s->offset_groups * kernel_area * output_plane;
        for (int64_t p0 = 0; p0 < output_plane; p0 += block) {
            const int64_t np = (output_plane - p0) < block ? (output_plane - p0) : block;
            for (int64_t ic = 0; ic < s->input_channels; ++ic) {
                const int64_t offset_group = ic / channels_per_offset_group;
                for (int64_t ky = 0; ky < s->kernel_height; ++ky) {
                    for (int64_t kx = 0; kx < s->kernel_width; ++kx) {
                        const int64_t kernel_index = ky * s->kernel_width + kx;
                        const int64_t offset_channel = 2 * (offset_group * kernel_area + kernel_index);
                        float *dst = sm + (ic * kernel_area + kernel_index) * block;
                        for (int64_t i = 0; i < np; ++i) {
                            const int64_t spatial = p0 + i;
                            const int64_t oy = spatial / s->output_width;
                            const int64_t ox = spatial % s->output_width;
                            const float offset_y =
                                offset[offset_base + offset_channel * output_plane + spatial];
                            const float offset_x =
                                offset[offset_base + (offset_channel + 1) * output_plane + spatial];
                            const float y = (float)(oy * s->stride_height - s->pad_height +
                                                    ky * s->dilation_height) + offset_y;
                            const float x = (float)(ox * s->stride_width - s->pad_width +
                                                    kx * s->dilation_width) + offset_x;
                            const float sampled =
                                bilinear(input, (n * s->input_channels + ic) * input_plane,
                                         s->input_height, s->input_width, y, x);
                            const int64_t mask_index =
                                mask_base + (offset_group * kernel_area + kernel_index) * output_plane +
                                spatial;
                            dst[i] = sampled * mask[mask_index];
                        }
                    }
                }
            }
            for (int64_t oc = 0; oc < s->output_channels; ++oc) {
                const int64_t group = oc / outputs_per_group;
                float *out = output + (n * s->output_channels + oc) * output_plane + p0;
                for (int64_t i = 0; i < np; ++i) out[i] = bias[oc];
                for (int64_t local_ic = 0; local_ic < channels_per_group; ++local_ic) {
                    const int64_t ic = group * channels_per_group + local_ic;
                    for (int64_t k = 0; k < kernel_area; ++k) {
                        const float w =
                            weight[(oc * channels_per_group + local_ic) * kernel_area + k];
                        const float *src = sm + (ic * kernel_area + k) * block;
                        for (int64_t i = 0; i < np; ++i) {
                            float term = src[i] * w;
                            out[i] = out[i] + term;
                        }
                    }
                }
            }
        }
    }
    free(sm);
    return 0;
}

typedef struct {
    const dcn_oracle_shape *s;
    const float *input, *offset, *mask, *weight, *bias;
    float *output;
    int32_t n_begin, n_end, oy_begin, oy_end;
    int rc;
} sample_job;

static void *sample_worker(void *arg) {
    sample_job *j = (sample_job *)arg;
    j->rc = run_literal(j->s, j->input, j->offset, j->mask, j->weight, j->bias, j->output,
                        j->n_begin, j->n_end, j->oy_begin, j->oy_end);
    return NULL;
}

int dcn_oracle_run_sample(const dcn_oracle_shape *s, const float *input, const float *offset,
                          const float *mask, const float *weight, const float *bias,
                          float *output, int32_t oy_begin, int32_t oy_end, int threads) {
    if (dcn_oracle_validate(s)) return 1;
    if (oy_begin < 0) oy_begin = 0;
    if (oy_end > s->output_height) oy_end = s->output_height;
    if (threads <= 0) threads = 1;
    if (threads > s->batch) threads = s->batch;
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    sample_job *jobs = (sample_job *)malloc(sizeof(sample_job) * (size_t)threads);
    if (!tid || !jobs) {
        free(tid);
        free(jobs);
        return 2;
    }
    int rc = 0;
    for (int t = 0; t < threads; ++t) {
        sample_job j = {s, input, offset, mask, weight, bias, output,
                        (int32_t)((int64_t)s->batch * t / threads),
                        (int32_t)((int64_t)s->batch * (t + 1) / threads), oy_begin, oy_end, 0};
        jobs[t] = j;
        if (pthread_create(&tid[t], NULL, sample_worker, &jobs[t]) != 0) {
            sample_worker(&jobs[t]);
            tid[t] = 0;
        }
    }
    for (int t = 0; t < threads; ++t) {
        if (tid[t]) pthread_join(tid[t], NULL);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    free(tid);
    free(jobs);
    return rc;
}

typedef struct {
    const dcn_oracle_shape *s;
    const float *input, *offset, *mask, *weight, *bias;
    float *output;
    int32_t n_begin, n_end;
    int fast;
    int rc;
} oracle_job;

static void *oracle_worker(void *arg) {
    oracle_job *j = (oracle_job *)arg;
    j->rc = j->fast ? dcn_oracle_run_fast_range(j->s, j->input, j->offset, j->mask, j->weight,
                                                j->bias, j->output, j->n_begin, j->n_end)
                    : dcn_oracle_run_range(j->s, j->input, j->offset, j->mask, j->weight, j->bias,
                                           j->output, j->n_begin, j->n_end);
    return NULL;
}

int dcn_oracle_run_threads(const dcn_oracle_shape *s, const float *input, const float *offset,
                           const float *mask, const float *weight, const float *bias,
                           float *output, int32_t n_begin, int32_t n_end, int threads, int fast) {
    if (dcn_oracle_validate(s)) return 1;
    if (n_begin < 0) n_begin = 0;
    if (n_end > s->batch) n_end = s->batch;
    const int32_t items = n_end > n_begin ? n_end - n_begin : 0;
    if (threads <= 0) threads = 1;
    if (threads > items) threads = items > 0 ? items : 1;
    if (threads == 1)
        return fast ? dcn_oracle_run_fast_range(s, input, offset, mask, weight, bias, output, n_begin,
                                                n_end)
                    : dcn_oracle_run_range(s, input, offset, mask, weight, bias, output, n_begin, n_end);
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    oracle_job *jobs = (oracle_job *)malloc(sizeof(oracle_job) * (size_t)threads);
    if (!tid || !jobs) {
        free(tid);
        free(jobs);
        return 2;
    }
    int rc = 0;
    for (int t = 0; t < threads; ++t) {
        jobs[t].s = s;
        jobs[t].input = input;
        jobs[t].offset = offset;
        jobs[t].mask = mask;
        jobs[t].weight = weight;
        jobs[t].bias = bias;
        jobs[t].output = output;
        jobs[t].n_begin = n_begin + (int32_t)((int64_t)items * t / threads);
        jobs[t].n_end = n_begin + (int32_t)((int64_t)items * (t + 1) / threads);
        jobs[t].fast = fast;
        jobs[t].rc = 0;
        if (pthread_create(&tid[t], NULL, oracle_worker, &jobs[t]) != 0) {
            oracle_worker(&jobs[t]);
            tid[t] = 0;
        }
    }
    for (int t = 0; t < threads; ++t) {
        if (tid[t]) pthread_join(tid[t], NULL);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    free(tid);
    free(jobs);
    return rc;
}

/* prepare_dcn_offsets_fp16 (MetalShader.swift:826-838) in FP32.  Channel c < 288
 * of `raw` is an offset residue: offset = 10*tanh(raw) + flow[1 - (c%144)%2]
 * (flow1 for c < 144, flow2 otherwise); the flow is stored (x, y), so even
 * (dy) channels take flow row 1.  Channels 288..431 are mask logits. */
void dcn_oracle_prepare_offsets(int64_t plane, const float *raw, const float *flow1,
                                const float *flow2, float *offset, float *mask) {
    for (int64_t c = 0; c < 432; ++c) {
        for (int64_t p = 0; p < plane; ++p) {
            const float v = raw[c * plane + p];
            if (c < 288) {
                const int64_t local = c % 144;
                const float *flow = c < 144 ? flow1 : flow2;
                const int64_t flow_channel = (local & 1) == 0 ? 1 : 0;
                float residue = 10.0f * tanhf(v);
                offset[c * plane + p] = residue + flow[flow_channel * plane + p];
            } else {
                mask[(c - 288) * plane + p] = 1.0f / (1.0f + expf(-v));
            }
        }
    }
}

/* FP16 rounding (round to nearest even) of a float: the reference stores every Metal
 * result as `half`. */
static float round_f16(float v) { return (float)(_Float16)v; }

/* runTemporalPreparation (MetalRunner.swift:510-582): accumulate_second_order_flow_fp16
 * (MetalShader.swift:739-762) and assemble_temporal_alignment_fp16 (:768-813), in the order of
 * the reference's self-check (JasnaCLI.swift:248-290); `bilinear` is its `sampleZero`
 * (:213-225), the same arithmetic as DeformConvCPU.bilinear. */
void dcn_oracle_temporal_prepare(int32_t width, int32_t height, const float *feat_prop,
                                 const float *feat_current, const float *feat_n2,
                                 const float *flow1, const float *previous_flow,
                                 int has_second_order, float *conditions, float *deform_input,
                                 float *flow2) {
    const int64_t w = width, h = height, plane = w * h;
    for (int64_t c = 0; c < 2; ++c) {
        for (int64_t p = 0; p < plane; ++p) {
            if (!has_second_order) {
                flow2[c * plane + p] = 0.0f;
                continue;
            }
            const float y = (float)(p / w), x = (float)(p % w);
            const float warped = bilinear(previous_flow, c * plane, h, w, y + flow1[plane + p], x + flow1[p]);
            flow2[c * plane + p] = round_f16(flow1[c * plane + p] + warped);
        }
    }
    for (int64_t c = 0; c < 196; ++c) {
        for (int64_t p = 0; p < plane; ++p) {
            const float y = (float)(p / w), x = (float)(p % w);
            float v;
            if (c < 64)
                v = round_f16(bilinear(feat_prop, c * plane, h, w, y + flow1[plane + p], x + flow1[p]));
            else if (c < 128)
                v = feat_current[(c - 64) * plane + p];
            else if (c < 192)
                v = round_f16(bilinear(feat_n2, (c - 128) * plane, h, w, y + flow2[plane + p], x + flow2[p]));
            else if (c < 194)
                v = flow1[(c - 192) * plane + p];
            else
                v = flow2[(c - 194) * plane + p];
            conditions[c * plane + p] = v;
        }
    }
    if (deform_input != NULL) {
        for (int64_t i = 0; i < 64 * plane; ++i) {
            deform_input[i] = feat_prop[i];
            deform_input[64 * plane + i] = feat_n2[i];
        }
    }
}

/* SeededGenerator.next (DeformConv.swift:175-181). */
uint64_t dcn_oracle_splitmix64(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
