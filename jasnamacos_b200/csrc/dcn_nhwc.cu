// dcn_nhwc.cu -- channels-last input for the tensor-core paths.
//
// The reference takes NCHW tensors (DeformConv.swift:110-132).  A host that keeps its features
// channels-last ([N][H][W][C]) would otherwise transpose them first; this pre-pass reads them in
// place and writes the same grouped layouts the NCHW pre-passes write, so dcn_forward_f16_grouped
// and dcn_forward_f16_raw_grouped follow unchanged:
//   slabs (slab kernel):           [N][G][H+2][W+2] x 16 bytes, the 8 channels of deformable group
//                                  g at each position, a one-pixel ring of zeros;
//   corner pairs (global gather):  [N][G][H][W+1] x 32 bytes, entry (y, e) = the group's 8 channels
//                                  at column e-1, then at column e (zeros outside the image).
// In channels-last memory a group's 8 channels at one pixel are one aligned 16-byte chunk, so each
// destination chunk is one 16-byte load.  Threads take the group index fastest: a warp reads whole
// pixels (G x 16 contiguous bytes each) and writes two adjacent positions of each group's plane,
// i.e. whole 32-byte sectors on both sides.
#include <cuda_fp16.h>

#include "dcn_common.cuh"

namespace dcn {

namespace {

template <bool kSlabs>
__global__ void __launch_bounds__(256) regroup_nhwc_kernel(const uint4 *__restrict__ in, uint4 *__restrict__ out,
                                                           int N, int G, int H, int W) {
    allow_dependent_launch();  // the tensor-core kernel may start its set-up
    // Destination units of one image: slab positions, or corner-pair entries.
    const int64_t units = kSlabs ? static_cast<int64_t>(H + 2) * (W + 2) : static_cast<int64_t>(H) * (W + 1);
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= units * G) return;
    const int g = static_cast<int>(t % G);
    const int64_t u = t / G;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    int y, x0;  // source row, and the column of the (first) chunk
    if (kSlabs) {
        const int py = static_cast<int>(u / (W + 2));
        y = py - 1;
        x0 = static_cast<int>(u - static_cast<int64_t>(py) * (W + 2)) - 1;
    } else {
        y = static_cast<int>(u / (W + 1));
        x0 = static_cast<int>(u - static_cast<int64_t>(y) * (W + 1)) - 1;
    }
    const bool row_in = y >= 0 && y < H;
    for (int64_t n = blockIdx.y; n < N; n += gridDim.y) {
        // Chunk (n, y, x, g) of the channels-last input: 16 bytes at ((n*H + y)*W + x)*G + g.
        const uint4 *src = in + ((n * H + (row_in ? y : 0)) * W) * G + g;
        const uint4 a = row_in && x0 >= 0 && x0 < W ? src[static_cast<int64_t>(x0) * G] : zero;
        if (kSlabs) {
            out[(n * G + g) * units + u] = a;
        } else {
            const int x1 = x0 + 1;
            const uint4 b = row_in && x1 < W ? src[static_cast<int64_t>(x1) * G] : zero;
            uint4 *dst = out + ((n * G + g) * units + u) * 2;
            dst[0] = a;
            dst[1] = b;
        }
    }
}

}  // namespace

// `slabs` selects the slab layout (else corner pairs).  `in` is 16-byte aligned with C = 8 * G.
cudaError_t launch_regroup_nhwc(bool slabs, int N, int G, int H, int W, const __half *in, void *workspace,
                                cudaStream_t stream) {
    const int64_t units = slabs ? static_cast<int64_t>(H + 2) * (W + 2) : static_cast<int64_t>(H) * (W + 1);
    const int64_t threads = units * G;
    const dim3 grid(static_cast<unsigned>((threads + 255) / 256), static_cast<unsigned>(N < 65535 ? N : 65535));
    const auto *src = reinterpret_cast<const uint4 *>(in);
    auto *dst = static_cast<uint4 *>(workspace);
    if (slabs)
        regroup_nhwc_kernel<true><<<grid, 256, 0, stream>>>(src, dst, N, G, H, W);
    else
        regroup_nhwc_kernel<false><<<grid, 256, 0, stream>>>(src, dst, N, G, H, W);
    return cudaGetLastError();
}

}  // namespace dcn
