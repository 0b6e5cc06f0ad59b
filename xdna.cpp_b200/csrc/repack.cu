// GPU repack between GGUF rows and the stripe-tile layout (formats.cuh), and
// its inverse.  One thread per (row, block); each tile is written in full by
// the threads of its rows, so the kernels run out of place (raw -> packed).
// This replaces the reference's host-side Q4_0 column prepack
// (src/xdna-q4-prepack.cpp:39-114) and, unlike it, keeps scales bit-exact.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "formats.cuh"
#include "gemv.cuh"

namespace xb {
namespace {

template <bool kPack>
__global__ void repack_kernel(int type, const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t N,
                              int64_t K, int64_t row0, int64_t nrows) {
    const Geometry g = make_geometry(type, N, K);
    const int64_t total = nrows * g.nb;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = row0 + i / g.nb;
        const int64_t b = i % g.nb;
        const int64_t t = row / TILE_ROWS;
        const int r = static_cast<int>(row % TILE_ROWS);
        const int tr = static_cast<int>(N - t * TILE_ROWS < TILE_ROWS ? N - t * TILE_ROWS : TILE_ROWS);
        const int64_t base = (t * TILE_ROWS - row0) * g.row_bytes;  // src/dst point at row row0
        if (kPack)
            repack_one(g, tr, r, b, src + base, dst + base);
        else
            unrepack_one(g, tr, r, b, src + base, dst + base);
    }
}

__global__ void bf16_kernel(const uint16_t* __restrict__ s, float* __restrict__ d, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        d[i] = __uint_as_float(uint32_t(s[i]) << 16);
}

cudaError_t check_args(int type, int64_t N, int64_t K, int64_t row0, int64_t nrows) {
    const FormatInfo f = format_info(type);
    if (!f.block_vals || K < 0 || K % f.block_vals || N < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N)
        return cudaErrorInvalidValue;
    const int tr = layout_kind(type, N, K) == 1 ? MMA_TILE_ROWS : TILE_ROWS;
    if (row0 % tr || (nrows % tr && row0 + nrows != N)) return cudaErrorInvalidValue;
    return cudaSuccess;
}

}  // namespace

cudaError_t repack_launch(int type, const void* raw, void* packed, int64_t N, int64_t K, int64_t row0,
                          int64_t nrows, cudaStream_t stream) {
    cudaError_t e = check_args(type, N, K, row0, nrows);
    if (e != cudaSuccess || nrows == 0 || K == 0) return e;
    if (layout_kind(type, N, K) == 1) return mma_repack_launch(type, raw, packed, nrows, K, true, stream);
    const int64_t total = nrows * (K / format_info(type).block_vals);
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads < 65536 ? (total + threads - 1) / threads : 65536;
    repack_kernel<true><<<unsigned(blocks), threads, 0, stream>>>(type, static_cast<const uint8_t*>(raw),
                                                                 static_cast<uint8_t*>(packed), N, K, row0, nrows);
    return cudaGetLastError();
}

cudaError_t unpack_launch(int type, const void* packed, void* raw, int64_t N, int64_t K, int64_t row0,
                          int64_t nrows, cudaStream_t stream) {
    cudaError_t e = check_args(type, N, K, row0, nrows);
    if (e != cudaSuccess || nrows == 0 || K == 0) return e;
    if (layout_kind(type, N, K) == 1) return mma_repack_launch(type, packed, raw, nrows, K, false, stream);
    const int64_t total = nrows * (K / format_info(type).block_vals);
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads < 65536 ? (total + threads - 1) / threads : 65536;
    repack_kernel<false><<<unsigned(blocks), threads, 0, stream>>>(type, static_cast<const uint8_t*>(packed),
                                                                  static_cast<uint8_t*>(raw), N, K, row0, nrows);
    return cudaGetLastError();
}

cudaError_t bf16_to_f32_launch(const uint16_t* src, float* dst, int64_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads < 4096 ? (n + threads - 1) / threads : 4096;
    bf16_kernel<<<unsigned(blocks), threads, 0, stream>>>(src, dst, n);
    return cudaGetLastError();
}

}  // namespace xb
