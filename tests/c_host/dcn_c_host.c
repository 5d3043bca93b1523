/*
 * dcn_c_host.c -- a plain C11 host of the DCNv2 library: the calls a Swift (or any C-ABI)
 * host makes in place of MetalDeformConv, with device memory from the CUDA runtime and
 * nothing else (no Python, no torch).  Checked against the C oracle (test
 * infrastructure) on the same values:
 *   - dcn_prepack_weights + dcn_forward_f16 on a slab-path batch (2 x 128 x 16 x 24, the
 *     group split with its reduction pass) and a global-gather image (1 x 128 x 64 x 96):
 *     FP16 gates max abs <= 2e-2, mean abs <= 2e-3;
 *   - dcn_forward_f16_host on page-locked host buffers (5 images in chunks of 2, 2 and 1,
 *     the chunks pipelined on the library's streams): FP16 gates against the oracle, and
 *     the non-finite flag delivered to host memory;
 *   - dcn_forward_f32: bit-identical to the oracle;
 *   - the non-finite flag and the error codes of invalid shapes and misaligned pointers.
 * Inputs are multiples of powers of two small enough to be exact in FP16, so the FP16 and
 * FP32 runs see the same values and no rounding code is needed here.
 * Build: gcc -std=c11 -I include -I oracle -I $CUDA/include dcn_c_host.c
 *        -L jasnamacos_b200/lib -ldcn_b200 -L oracle/_build -ldcn_oracle -L $CUDA/lib64 -lcudart
 * Exit status 0 and a last line "PASS" when every check holds.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "dcn_b200.h"
#include "dcn_oracle.h"

static int failures = 0;

#define CHECK(cond, ...)                                  \
    do {                                                  \
        if (!(cond)) {                                    \
            fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
            fprintf(stderr, __VA_ARGS__);                 \
            fprintf(stderr, "\n");                        \
            ++failures;                                   \
        }                                                 \
    } while (0)

#define CUDA_OK(call)                                                             \
    do {                                                                          \
        cudaError_t e_ = (call);                                                  \
        if (e_ != cudaSuccess) {                                                  \
            fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            exit(2);                                                              \
        }                                                                         \
    } while (0)

/* FP16 bits of a float that FP16 represents exactly (zero or a normal FP16 number). */
static uint16_t half_bits_exact(float v) {
    uint32_t u;
    memcpy(&u, &v, sizeof u);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    if ((u & 0x7fffffffu) == 0) return sign;
    const int exp = (int)((u >> 23) & 0xffu) - 127 + 15;
    return (uint16_t)(sign | (uint16_t)(exp << 10) | (uint16_t)((u >> 13) & 0x3ffu));
}

static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        const float v = ldexpf((float)man, -24);
        return (h & 0x8000u) ? -v : v;
    }
    if (exp == 31) u = sign | 0x7f800000u | (man << 13);
    else u = sign | ((exp - 15 + 127) << 23) | (man << 13);
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* Uniform integer in [lo, hi) from the reference's SplitMix64 stream. */
static int64_t draw(uint64_t *state, int64_t lo, int64_t hi) {
    return lo + (int64_t)(dcn_oracle_splitmix64(state) % (uint64_t)(hi - lo));
}

static dcn_shape jasna_shape(int n, int h, int w) {
    dcn_shape s;
    memset(&s, 0, sizeof s);
    s.batch = n;
    s.input_channels = 128;
    s.input_height = h;
    s.input_width = w;
    s.output_channels = 64;
    s.output_height = h;
    s.output_width = w;
    s.kernel_height = 3;
    s.kernel_width = 3;
    s.pad_height = 1;
    s.pad_width = 1;
    s.stride_height = 1;
    s.stride_width = 1;
    s.dilation_height = 1;
    s.dilation_width = 1;
    s.groups = 1;
    s.offset_groups = 16;
    return s;
}

typedef struct {
    float *x, *off, *msk, *w, *b; /* host values, exact in FP16 */
    dcn_counts c;
} case_data;

static case_data make_case(const dcn_shape *s, uint64_t seed) {
    case_data d;
    CHECK(dcn_shape_counts(s, &d.c) == DCN_OK, "dcn_shape_counts");
    d.x = malloc(sizeof(float) * (size_t)d.c.input);
    d.off = malloc(sizeof(float) * (size_t)d.c.offset);
    d.msk = malloc(sizeof(float) * (size_t)d.c.mask);
    d.w = malloc(sizeof(float) * (size_t)d.c.weight);
    d.b = malloc(sizeof(float) * (size_t)d.c.bias);
    uint64_t st = seed;
    for (int64_t i = 0; i < d.c.input; ++i) d.x[i] = (float)draw(&st, -1024, 1024) / 256.0f;   /* [-4, 4) */
    for (int64_t i = 0; i < d.c.offset; ++i) d.off[i] = (float)draw(&st, -384, 384) / 64.0f; /* [-6, 6) */
    for (int64_t i = 0; i < d.c.mask; ++i) d.msk[i] = (float)draw(&st, 0, 1024) / 1024.0f;   /* [0, 1) */
    for (int64_t i = 0; i < d.c.weight; ++i) d.w[i] = (float)draw(&st, -240, 240) / 8192.0f; /* |w| < 0.03 */
    for (int64_t i = 0; i < d.c.bias; ++i) d.b[i] = (float)draw(&st, -100, 100) / 1024.0f;
    return d;
}

static void free_case(case_data *d) {
    free(d->x);
    free(d->off);
    free(d->msk);
    free(d->w);
    free(d->b);
}

static void *to_device_f16(const float *v, int64_t n) {
    uint16_t *h = malloc(sizeof(uint16_t) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) h[i] = half_bits_exact(v[i]);
    void *d = NULL;
    CUDA_OK(cudaMalloc(&d, sizeof(uint16_t) * (size_t)n));
    CUDA_OK(cudaMemcpy(d, h, sizeof(uint16_t) * (size_t)n, cudaMemcpyHostToDevice));
    free(h);
    return d;
}

static void *to_device_f32(const float *v, int64_t n) {
    void *d = NULL;
    CUDA_OK(cudaMalloc(&d, sizeof(float) * (size_t)n));
    CUDA_OK(cudaMemcpy(d, v, sizeof(float) * (size_t)n, cudaMemcpyHostToDevice));
    return d;
}

static float *oracle_run(const dcn_shape *s, const case_data *d) {
    dcn_oracle_shape os;
    memcpy(&os, s, sizeof os);
    float *ref = malloc(sizeof(float) * (size_t)d->c.output);
    CHECK(dcn_oracle_run_threads(&os, d->x, d->off, d->msk, d->w, d->b, ref, 0, s->batch, 8, 1) == 0, "oracle");
    return ref;
}

/* The FP16 operator through the C ABI, against the oracle; returns the path taken. */
static int check_f16(const dcn_shape *s, uint64_t seed, const char *name) {
    case_data d = make_case(s, seed);
    const dcn_path path = dcn_forward_f16_path(s);
    void *x = to_device_f16(d.x, d.c.input), *off = to_device_f16(d.off, d.c.offset);
    void *msk = to_device_f16(d.msk, d.c.mask), *w = to_device_f16(d.w, d.c.weight);
    void *b = to_device_f16(d.b, d.c.bias);
    void *packed = NULL, *ws = NULL, *out = NULL;
    uint32_t *flag = NULL;
    const size_t pw = dcn_packed_weight_bytes(s), wsb = dcn_forward_f16_workspace_bytes(s);
    CUDA_OK(cudaMalloc(&packed, pw));
    CUDA_OK(cudaMalloc(&ws, wsb > 0 ? wsb : 256));
    CUDA_OK(cudaMalloc(&out, sizeof(uint16_t) * (size_t)d.c.output));
    CUDA_OK(cudaMalloc((void **)&flag, sizeof(uint32_t)));
    CUDA_OK(cudaMemset(flag, 0, sizeof(uint32_t)));
    CHECK(dcn_prepack_weights(s, w, DCN_DTYPE_F16, DCN_WEIGHT_OIHW, packed, NULL) == DCN_OK, "%s: prepack", name);
    const dcn_status st = dcn_forward_f16(s, x, off, msk, packed, b, out, flag, ws, wsb, NULL);
    CHECK(st == DCN_OK, "%s: dcn_forward_f16 -> %s", name, dcn_status_string(st));
    CUDA_OK(cudaDeviceSynchronize());
    CHECK(dcn_device_error() == DCN_OK, "%s: device error word", name);
    uint32_t hflag = 1;
    CUDA_OK(cudaMemcpy(&hflag, flag, sizeof hflag, cudaMemcpyDeviceToHost));
    CHECK(hflag == 0, "%s: non-finite flag set on finite output", name);
    uint16_t *h = malloc(sizeof(uint16_t) * (size_t)d.c.output);
    CUDA_OK(cudaMemcpy(h, out, sizeof(uint16_t) * (size_t)d.c.output, cudaMemcpyDeviceToHost));
    float *ref = oracle_run(s, &d);
    double max_abs = 0.0, sum_abs = 0.0;
    for (int64_t i = 0; i < d.c.output; ++i) {
        const double e = fabs((double)half_to_float(h[i]) - (double)ref[i]);
        if (e > max_abs) max_abs = e;
        sum_abs += e;
    }
    const double mean_abs = sum_abs / (double)d.c.output;
    printf("%s: path %d, FP16 max abs %.3g, mean abs %.3g\n", name, (int)path, max_abs, mean_abs);
    CHECK(max_abs <= 2e-2 && mean_abs <= 2e-3, "%s: FP16 gates (max %.3g, mean %.3g)", name, max_abs, mean_abs);

    /* An infinite bias makes every output non-finite: the flag must be raised. */
    const uint16_t big = 0x7c00u;
    uint16_t *hb = malloc(sizeof(uint16_t) * (size_t)d.c.bias);
    for (int64_t i = 0; i < d.c.bias; ++i) hb[i] = big;
    CUDA_OK(cudaMemcpy(b, hb, sizeof(uint16_t) * (size_t)d.c.bias, cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemset(flag, 0, sizeof(uint32_t)));
    CHECK(dcn_forward_f16(s, x, off, msk, packed, b, out, flag, ws, wsb, NULL) == DCN_OK, "%s: overflow call", name);
    CUDA_OK(cudaMemcpy(&hflag, flag, sizeof hflag, cudaMemcpyDeviceToHost));
    CHECK(hflag & DCN_FLAG_NONFINITE, "%s: non-finite flag not raised", name);

    free(hb);
    free(h);
    free(ref);
    cudaFree(x);
    cudaFree(off);
    cudaFree(msk);
    cudaFree(w);
    cudaFree(b);
    cudaFree(packed);
    cudaFree(ws);
    cudaFree(out);
    cudaFree(flag);
    free_case(&d);
    return (int)path;
}

/* The host-buffer entry point: inputs and output in page-locked host memory, chunks of
 * `chunk` images pipelined by the library; FP16 gates against the oracle. */
static void check_f16_host(const dcn_shape *s, uint64_t seed, int32_t chunk) {
    case_data d = make_case(s, seed);
    uint16_t *hx = NULL, *hoff = NULL, *hmsk = NULL, *hout = NULL;
    uint32_t *hflag = NULL;
    CUDA_OK(cudaHostAlloc((void **)&hx, sizeof(uint16_t) * (size_t)d.c.input, cudaHostAllocDefault));
    CUDA_OK(cudaHostAlloc((void **)&hoff, sizeof(uint16_t) * (size_t)d.c.offset, cudaHostAllocDefault));
    CUDA_OK(cudaHostAlloc((void **)&hmsk, sizeof(uint16_t) * (size_t)d.c.mask, cudaHostAllocDefault));
    CUDA_OK(cudaHostAlloc((void **)&hout, sizeof(uint16_t) * (size_t)d.c.output, cudaHostAllocDefault));
    CUDA_OK(cudaHostAlloc((void **)&hflag, sizeof(uint32_t), cudaHostAllocDefault));
    for (int64_t i = 0; i < d.c.input; ++i) hx[i] = half_bits_exact(d.x[i]);
    for (int64_t i = 0; i < d.c.offset; ++i) hoff[i] = half_bits_exact(d.off[i]);
    for (int64_t i = 0; i < d.c.mask; ++i) hmsk[i] = half_bits_exact(d.msk[i]);
    void *w = to_device_f16(d.w, d.c.weight), *b = to_device_f16(d.b, d.c.bias);
    void *packed = NULL, *ws = NULL;
    const size_t wsb = dcn_forward_f16_host_workspace_bytes(s, chunk);
    CHECK(wsb > 0, "host workspace size");
    CUDA_OK(cudaMalloc(&packed, dcn_packed_weight_bytes(s)));
    CUDA_OK(cudaMalloc(&ws, wsb));
    CHECK(dcn_prepack_weights(s, w, DCN_DTYPE_F16, DCN_WEIGHT_OIHW, packed, NULL) == DCN_OK, "host: prepack");
    cudaStream_t stream;
    CUDA_OK(cudaStreamCreate(&stream));
    *hflag = 0xffffffffu;
    dcn_status st = dcn_forward_f16_host(s, hx, hoff, hmsk, packed, b, hout, hflag, chunk, ws, wsb,
                                         (dcn_stream)stream);
    CHECK(st == DCN_OK, "dcn_forward_f16_host -> %s", dcn_status_string(st));
    CUDA_OK(cudaStreamSynchronize(stream));
    CHECK(*hflag == 0, "host: flag %u on finite output", *hflag);
    CHECK(dcn_device_error() == DCN_OK, "host: device error word");
    float *ref = oracle_run(s, &d);
    double max_abs = 0.0, sum_abs = 0.0;
    for (int64_t i = 0; i < d.c.output; ++i) {
        const double e = fabs((double)half_to_float(hout[i]) - (double)ref[i]);
        if (e > max_abs) max_abs = e;
        sum_abs += e;
    }
    const double mean_abs = sum_abs / (double)d.c.output;
    printf("host buffers, %d images in chunks of %d: FP16 max abs %.3g, mean abs %.3g\n", s->batch, chunk,
           max_abs, mean_abs);
    CHECK(max_abs <= 2e-2 && mean_abs <= 2e-3, "host: FP16 gates (max %.3g, mean %.3g)", max_abs, mean_abs);
    CHECK(dcn_forward_f16_host(s, hx, hoff, hmsk, packed, b, hout, hflag, chunk, ws, wsb - 1, (dcn_stream)stream) ==
              DCN_ERR_INVALID_ARGUMENT,
          "host: short workspace accepted");

    /* Infinite bias: every output non-finite, the flag must reach host memory. */
    const uint16_t inf = 0x7c00u;
    for (int64_t i = 0; i < d.c.bias; ++i) CUDA_OK(cudaMemcpy((uint16_t *)b + i, &inf, 2, cudaMemcpyHostToDevice));
    *hflag = 0;
    CHECK(dcn_forward_f16_host(s, hx, hoff, hmsk, packed, b, hout, hflag, chunk, ws, wsb, (dcn_stream)stream) ==
              DCN_OK,
          "host: overflow call");
    CUDA_OK(cudaStreamSynchronize(stream));
    CHECK(*hflag & DCN_FLAG_NONFINITE, "host: non-finite flag not delivered");

    CUDA_OK(cudaStreamDestroy(stream));
    free(ref);
    cudaFreeHost(hx);
    cudaFreeHost(hoff);
    cudaFreeHost(hmsk);
    cudaFreeHost(hout);
    cudaFreeHost(hflag);
    cudaFree(w);
    cudaFree(b);
    cudaFree(packed);
    cudaFree(ws);
    free_case(&d);
}

static void check_f32(const dcn_shape *s, uint64_t seed) {
    case_data d = make_case(s, seed);
    float *x = to_device_f32(d.x, d.c.input), *off = to_device_f32(d.off, d.c.offset);
    float *msk = to_device_f32(d.msk, d.c.mask), *w = to_device_f32(d.w, d.c.weight);
    float *b = to_device_f32(d.b, d.c.bias), *out = NULL;
    CUDA_OK(cudaMalloc((void **)&out, sizeof(float) * (size_t)d.c.output));
    const dcn_status st = dcn_forward_f32(s, x, off, msk, w, b, out, NULL);
    CHECK(st == DCN_OK, "dcn_forward_f32 -> %s", dcn_status_string(st));
    float *h = malloc(sizeof(float) * (size_t)d.c.output);
    CUDA_OK(cudaMemcpy(h, out, sizeof(float) * (size_t)d.c.output, cudaMemcpyDeviceToHost));
    float *ref = oracle_run(s, &d);
    int64_t differ = 0;
    for (int64_t i = 0; i < d.c.output; ++i) differ += memcmp(&h[i], &ref[i], sizeof(float)) != 0;
    printf("FP32: %lld of %lld outputs differ from the oracle\n", (long long)differ, (long long)d.c.output);
    CHECK(differ == 0, "FP32 path is not bit-identical to the oracle");
    free(h);
    free(ref);
    cudaFree(x);
    cudaFree(off);
    cudaFree(msk);
    cudaFree(w);
    cudaFree(b);
    cudaFree(out);
    free_case(&d);
}

static void check_errors(void) {
    dcn_shape bad = jasna_shape(1, 16, 24);
    bad.offset_groups = 3; /* 128 channels do not split into 3 deformable groups */
    CHECK(dcn_shape_validate(&bad) == DCN_ERR_INVALID_SHAPE, "invalid shape accepted");
    CHECK(dcn_forward_f16(&bad, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 0, NULL) == DCN_ERR_INVALID_SHAPE,
          "forward with an invalid shape");
    dcn_shape s = jasna_shape(1, 16, 24);
    void *buf = NULL;
    CUDA_OK(cudaMalloc(&buf, 1 << 20));
    char *p = (char *)buf;
    const dcn_status st = dcn_forward_f16(&s, p + 1, p, p, p, p, p, NULL, p, 1 << 20, NULL);
    CHECK(st == DCN_ERR_INVALID_ARGUMENT, "misaligned input accepted (%s)", dcn_status_string(st));
    CHECK(dcn_status_is_recoverable(DCN_ERR_NONFINITE) == 1 && dcn_status_is_recoverable(DCN_ERR_LAUNCH) == 0,
          "recoverability");
    CHECK(dcn_status_string(DCN_ERR_UNSUPPORTED) != NULL, "status string");
    cudaFree(buf);
}

/* FP16 bits of a float, rounded to nearest even. */
static uint16_t half_bits_rne(float v) {
    _Float16 h = (_Float16)v;
    uint16_t b;
    memcpy(&b, &h, sizeof b);
    return b;
}

/* dcn_temporal_prepare_f16 (runTemporalPreparation's two kernels) on `frames` frames of w x h with
 * seeded FP16 features and flows, against dcn_oracle_temporal_prepare frame by frame, bit for bit. */
static void check_temporal(int frames, int w, int h, uint64_t seed) {
    const int64_t plane = (int64_t)w * h;
    const int64_t nf = frames * 64 * plane, nflow = frames * 2 * plane;
    float *in[5];
    uint16_t *bits[5];
    const int64_t counts[5] = {nf, nf, nf, nflow, nflow};
    uint64_t st = seed;
    for (int t = 0; t < 5; ++t) {
        in[t] = (float *)malloc(sizeof(float) * (size_t)counts[t]);
        bits[t] = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)counts[t]);
        for (int64_t i = 0; i < counts[t]; ++i) {
            /* features in [-2, 2), flows in [-12, 12) px, 1/256 steps, then FP16 */
            const float v = t < 3 ? (float)draw(&st, -512, 512) / 256.0f : (float)draw(&st, -3072, 3072) / 256.0f;
            bits[t][i] = half_bits_rne(v);
            in[t][i] = half_to_float(bits[t][i]);
        }
    }
    void *d_in[5], *d_cond, *d_di, *d_flow2;
    for (int t = 0; t < 5; ++t) {
        CUDA_OK(cudaMalloc(&d_in[t], sizeof(uint16_t) * (size_t)counts[t]));
        CUDA_OK(cudaMemcpy(d_in[t], bits[t], sizeof(uint16_t) * (size_t)counts[t], cudaMemcpyHostToDevice));
    }
    const int64_t ncond = frames * 196 * plane, ndi = frames * 128 * plane;
    CUDA_OK(cudaMalloc(&d_cond, sizeof(uint16_t) * (size_t)ncond));
    CUDA_OK(cudaMalloc(&d_di, sizeof(uint16_t) * (size_t)ndi));
    CUDA_OK(cudaMalloc(&d_flow2, sizeof(uint16_t) * (size_t)nflow));
    const dcn_status rc = dcn_temporal_prepare_f16(frames, w, h, d_in[0], d_in[1], d_in[2], d_in[3], d_in[4], 1,
                                                   d_cond, d_di, d_flow2, NULL);
    CHECK(rc == DCN_OK, "temporal %dx%d: %s", w, h, dcn_status_string(rc));
    CUDA_OK(cudaDeviceSynchronize());
    uint16_t *cond = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)ncond);
    uint16_t *di = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)ndi);
    uint16_t *flow2 = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)nflow);
    CUDA_OK(cudaMemcpy(cond, d_cond, sizeof(uint16_t) * (size_t)ncond, cudaMemcpyDeviceToHost));
    CUDA_OK(cudaMemcpy(di, d_di, sizeof(uint16_t) * (size_t)ndi, cudaMemcpyDeviceToHost));
    CUDA_OK(cudaMemcpy(flow2, d_flow2, sizeof(uint16_t) * (size_t)nflow, cudaMemcpyDeviceToHost));
    float *rc_cond = (float *)malloc(sizeof(float) * (size_t)(196 * plane));
    float *rc_di = (float *)malloc(sizeof(float) * (size_t)(128 * plane));
    float *rc_flow2 = (float *)malloc(sizeof(float) * (size_t)(2 * plane));
    int64_t mismatches = 0;
    for (int f = 0; f < frames; ++f) {
        dcn_oracle_temporal_prepare(w, h, in[0] + f * 64 * plane, in[1] + f * 64 * plane, in[2] + f * 64 * plane,
                                    in[3] + f * 2 * plane, in[4] + f * 2 * plane, 1, rc_cond, rc_di, rc_flow2);
        for (int64_t i = 0; i < 196 * plane; ++i) mismatches += cond[f * 196 * plane + i] != half_bits_rne(rc_cond[i]);
        for (int64_t i = 0; i < 128 * plane; ++i) mismatches += di[f * 128 * plane + i] != half_bits_rne(rc_di[i]);
        for (int64_t i = 0; i < 2 * plane; ++i) mismatches += flow2[f * 2 * plane + i] != half_bits_rne(rc_flow2[i]);
    }
    CHECK(mismatches == 0, "temporal %dx%d x%d: %lld values differ from the oracle", w, h, frames,
          (long long)mismatches);
    printf("temporal preparation %dx%d x%d: bit-exact against the oracle\n", w, h, frames);
    /* The slab form: the deform input as the DCN's slabs [frames][16][H+2][W+2][8] (zero ring),
     * written into a buffer filled with 0xA5 first; conditions and flow2 as above. */
    const size_t slab_bytes = dcn_temporal_slabs_bytes(frames, w, h);
    if (slab_bytes > 0 && plane % 2 == 0) {
        void *d_ws = NULL;
        CUDA_OK(cudaMalloc(&d_ws, slab_bytes));
        CUDA_OK(cudaMemset(d_ws, 0xA5, slab_bytes));
        CUDA_OK(cudaMemset(d_cond, 0, sizeof(uint16_t) * (size_t)ncond));
        const dcn_status rs = dcn_temporal_prepare_slabs_f16(frames, w, h, d_in[0], d_in[1], d_in[2], d_in[3],
                                                             d_in[4], 1, d_cond, d_flow2, d_ws, slab_bytes, NULL);
        CHECK(rs == DCN_OK, "temporal slabs %dx%d: %s", w, h, dcn_status_string(rs));
        CUDA_OK(cudaDeviceSynchronize());
        uint16_t *slabs = (uint16_t *)malloc(slab_bytes);
        uint16_t *cond2 = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)ncond);
        CUDA_OK(cudaMemcpy(slabs, d_ws, slab_bytes, cudaMemcpyDeviceToHost));
        CUDA_OK(cudaMemcpy(cond2, d_cond, sizeof(uint16_t) * (size_t)ncond, cudaMemcpyDeviceToHost));
        int64_t bad = memcmp(cond2, cond, sizeof(uint16_t) * (size_t)ncond) != 0;
        const int sw = w + 2, sh = h + 2;
        for (int f = 0; f < frames; ++f)
            for (int g = 0; g < 16; ++g)
                for (int py = 0; py < sh; ++py)
                    for (int px = 0; px < sw; ++px)
                        for (int c = 0; c < 8; ++c) {
                            const int y = py - 1, x = px - 1;
                            const int inside = y >= 0 && y < h && x >= 0 && x < w;
                            /* di was checked against the oracle above */
                            const uint16_t want = inside ? di[f * 128 * plane + (8 * g + c) * plane + y * w + x] : 0;
                            bad += slabs[((((int64_t)f * 16 + g) * sh + py) * sw + px) * 8 + c] != want;
                        }
        CHECK(bad == 0, "temporal slabs %dx%d x%d: %lld values differ", w, h, frames, (long long)bad);
        printf("temporal preparation %dx%d x%d, slab form: the DCN's slab layout of the oracle's deform input\n", w,
               h, frames);
        free(slabs);
        free(cond2);
        cudaFree(d_ws);
    }
    for (int t = 0; t < 5; ++t) {
        free(in[t]);
        free(bits[t]);
        cudaFree(d_in[t]);
    }
    cudaFree(d_cond);
    cudaFree(d_di);
    cudaFree(d_flow2);
    free(cond);
    free(di);
    free(flow2);
    free(rc_cond);
    free(rc_di);
    free(rc_flow2);
}

int main(void) {
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) {
        fprintf(stderr, "no CUDA device\n");
        return 2;
    }
    printf("ABI version %d\n", dcn_abi_version());
    const dcn_shape slab = jasna_shape(2, 16, 24);
    const dcn_shape frame = jasna_shape(1, 64, 96);
    CHECK(check_f16(&slab, 11, "slab 2x16x24") == DCN_PATH_SLAB_TC, "slab shape took another path");
    CHECK(check_f16(&frame, 12, "global-gather 1x64x96") == DCN_PATH_FUSED_TC, "frame took another path");
    const dcn_shape five = jasna_shape(5, 16, 24);
    check_f16_host(&five, 14, 2);
    check_f32(&slab, 13);
    check_temporal(2, 64, 64, 15);  /* the shared-memory form */
    check_temporal(1, 17, 13, 16);  /* an odd pixel count: the global-memory form */
    check_errors();
    if (failures) {
        printf("FAILED (%d)\n", failures);
        return 1;
    }
    printf("PASS\n");
    return 0;
}
