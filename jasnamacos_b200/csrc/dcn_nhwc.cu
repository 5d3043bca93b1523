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
// i.e. whole 32-byte sectors on both sides.  Each thread handles four such chunks, their loads
// issued before any store, so that enough bytes are in flight to keep HBM busy.
#include <cuda_fp16.h>

#include "dcn_common.cuh"

namespace dcn {

namespace {

constexpr int kItems = 4;  // destination chunks per thread, loads issued before any store

template <bool kSlabs>
__global__ void __launch_bounds__(256) regroup_nhwc_kernel(const uint4 *__restrict__ in, uint4 *__restrict__ out,
                                                           int N, int G, int H, int W) {
    allow_dependent_launch();  // the tensor-core kernel may start its set-up
    // Destination units of one image: slab positions, or corner-pair entries; thread t takes items
    // t, t + S, t + 2S, t + 3S of the image's units x groups (S = the grid's thread count).
    // Per-image indices fit 32 bits (checked on launch).
    const int units = kSlabs ? (H + 2) * (W + 2) : H * (W + 1);
    const int total = units * G;
    const int stride = static_cast<int>(gridDim.x * blockDim.x);
    const int t0 = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int64_t n = blockIdx.y; n < N; n += gridDim.y) {
        uint4 a[kItems], b[kItems];
        int64_t dst[kItems];
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            const int t = t0 + j * stride;
            dst[j] = -1;
            a[j] = b[j] = zero;
            if (t >= total) continue;
            const int u = t / G, g = t - u * G;
            int y, x0;  // source row, and the column of the (first) chunk
            if (kSlabs) {
                const int py = u / (W + 2);
                y = py - 1;
                x0 = u - py * (W + 2) - 1;
            } else {
                y = u / (W + 1);
                x0 = u - y * (W + 1) - 1;
            }
            const bool row_in = y >= 0 && y < H;
            // Chunk (n, y, x, g) of the channels-last input: 16 bytes at ((n*H + y)*W + x)*G + g.
            const uint4 *src = in + ((n * H + (row_in ? y : 0)) * W) * G + g;
            if (row_in && x0 >= 0 && x0 < W) a[j] = src[static_cast<int64_t>(x0) * G];
            if (!kSlabs && row_in && x0 + 1 < W) b[j] = src[static_cast<int64_t>(x0 + 1) * G];
            dst[j] = (n * G + g) * static_cast<int64_t>(units) + u;
        }
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
            if (dst[j] < 0) continue;
            if (kSlabs) {
                out[dst[j]] = a[j];
            } else {
                out[2 * dst[j]] = a[j];
                out[2 * dst[j] + 1] = b[j];
            }
        }
    }
}

}  // namespace

// `slabs` selects the slab layout (else corner pairs).  `in` is 16-byte aligned with C = 8 * G.
cudaError_t launch_regroup_nhwc(bool slabs, int N, int G, int H, int W, const __half *in, void *workspace,
                                cudaStream_t stream) {
    const int64_t units = slabs ? static_cast<int64_t>(H + 2) * (W + 2) : static_cast<int64_t>(H) * (W + 1);
    if (units * G + static_cast<int64_t>(kItems) * 256 * 65535 >= (int64_t{1} << 31)) return cudaErrorInvalidValue;
    const int64_t threads = (units * G + kItems - 1) / kItems;
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
