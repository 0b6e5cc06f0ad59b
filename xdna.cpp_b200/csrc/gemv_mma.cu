// Integer tensor-core GEMV for 4-bit linear formats (Q4_0, Q4_K) on sm_100a.
//
// Why tensor cores for an M = 1 GEMV: the contraction is bandwidth bound, but
// unpacking and multiplying 4-bit weights on the FP32 pipes costs ~4
// instructions per weight value, more than the SM can issue at HBM speed.
// Here each value costs about one instruction:
//
//   * x (F32) is first rewritten, per 32-value block b, as a 24-bit fixed-point
//     integer X_j = rint(x_j / 2^e_b) (|X| <= 2^22) split into three signed
//     base-256 digits: X = D2 * 65536 + D1 * 256 + D0 (xprep_kernel).  The
//     representation error is <= 2^(e_b - 1), about 2^-23 of the block's
//     largest |x| -- the precision of F32 itself.
//   * mma.sync.m16n8k32.s32.u8.s8 multiplies 16 weight rows by the digit
//     planes.  The B operand is block diagonal: in one 32-wide k-chunk, k rows
//     4b..4b+3 hold four values of block b and only column b is non-zero there,
//     so C[row][b] accumulates the exact integer dot product of block b.  The
//     C fragment puts blocks 2t, 2t+1 of rows g, g+8 in lane (g, t), so the
//     per-block scales (Q4_0 d, Q4_K d * sc and dmin * m) are applied with no
//     idle lanes.
//   * weights arrive pre-swizzled (formats.cuh, MMA layout) so one 16-byte
//     streaming load per lane yields two chunks' A fragments after a mask and
//     a shift; there is no x reuse problem because B comes from L1/L2.
//
// Accumulation: exact int32 inside a block, F32 across blocks (the products
// never round, so the result is at least as accurate as the reference's
// sequential F32 dot).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "formats.cuh"
#include "gemv.cuh"

namespace xb {
namespace {


__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// x preparation: one warp per 32-value block.
//   frags[(group * 8 + chunk) * 8 + block_in_group] = {D0, D1, D2, 0} words
//   holding the digits of values 4*chunk .. 4*chunk + 3 (byte j = value 4c+j);
//   scale[b] = 2^e_b; xsum[b] = sum of the block's x (F32).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(64) xprep_kernel(const float* __restrict__ x, int64_t K, uint8_t* __restrict__ frags,
                                                    float* __restrict__ scale, float* __restrict__ xsum,
                                                    int* __restrict__ queue) {
    pdl_release();
    pdl_wait();
    if (blockIdx.x == 0 && threadIdx.x == 0) *queue = 0;  // tile queue of the GEMV that follows
    const int lane = threadIdx.x & 31;
    const int64_t nblk = K / 32;
    for (int64_t b = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; b < nblk;
         b += (int64_t(gridDim.x) * blockDim.x) >> 5) {
        const float v = x[b * 32 + lane];
        float m = fabsf(v), s = v;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            s += __shfl_xor_sync(0xffffffffu, s, o);
        }
        int E = 0;
        if (m > 0.f) frexpf(m, &E);  // m < 2^E
        int e = m > 0.f ? E - 22 : 0;
        e = e < -120 ? -120 : (e > 120 ? 120 : e);
        const int X = __float2int_rn(v * ldexpf(1.0f, -e));  // |X| <= 2^22
        const int d0 = ((X + 128) & 255) - 128;
        const int X1 = (X - d0) >> 8;
        const int d1 = ((X1 + 128) & 255) - 128;
        const int d2 = (X1 - d1) >> 8;
        const int64_t gi = b >> 3;
        const int blk = static_cast<int>(b & 7), c = lane >> 2, j = lane & 3;
        uint8_t* w = frags + ((gi * 8 + c) * 8 + blk) * 16;
        w[j] = static_cast<uint8_t>(d0);
        w[4 + j] = static_cast<uint8_t>(d1);
        w[8 + j] = static_cast<uint8_t>(d2);
        w[12 + j] = 0;
        if (lane == 0) {
            scale[b] = ldexpf(1.0f, e);
            xsum[b] = s;
        }
    }
}

// ---------------------------------------------------------------------------
// GEMV.  A CTA of 8 warps works on one 16-row tile at a time; warp w takes
// groups w, w + 8, ... of the tile and the warps combine their partial rows
// through shared memory.  Tiles come from a queue (first one static, then an
// atomic counter that xprep_kernel zeroes), so CTAs that finish early take
// more work instead of idling at the tail.  Each warp keeps DRAM busy ahead
// of its loads with one bulk L2 prefetch per group (cp.async.bulk.prefetch:
// no registers, no completion to track) for the groups it will read next.
// ---------------------------------------------------------------------------
constexpr int kWarps = 8;
constexpr int kGemvThreads = kWarps * 32;
constexpr int kPrefetch = 3;  // groups ahead per warp

struct GemvArgs {
    const uint8_t* W;
    const uint4* frags;   // x digits, 64 x 16 B per group
    const float* scale;   // per 32-value block
    const float* xsum;
    float* y;
    int* queue;           // tile counter, zeroed by xprep
    int64_t N, K;
    int64_t ntiles, ngroups;
};

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// One group of 16 rows x 256 values: accumulate rows g and g+8 of this lane.
// bA / bB are this lane's B registers; only their owning lanes ever load them,
// so elsewhere they stay zero without being cleared per chunk.
template <int TYPE>
__device__ __forceinline__ void group_dot(const uint8_t* gb, const uint4* __restrict__ fg, const float* __restrict__ sc_,
                                          const float* __restrict__ xs_, int lane, int g, int t, bool ldA, bool ldB,
                                          uint4& bA, uint4& bB, float& y0, float& y8) {
    uint4 A[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] = ld_stream(gb + (i * 32 + lane) * 16);
    uint4 h0, h8;
    uint2 d4;
    if (TYPE == T_Q4_K) {
        h0 = ld_stream(gb + 2048 + 16 * g);
        h8 = ld_stream(gb + 2048 + 16 * (g + 8));
    } else {
        d4 = __ldg(reinterpret_cast<const uint2*>(gb + 2048) + lane);
    }
    int C[3][4];
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int k = 0; k < 4; ++k) C[p][k] = 0;
    // x digits of all eight chunks first (independent registers, so the
    // loads overlap); only the 8 owning lanes load, the rest keep zeros
    fg += g;
    uint4 bf[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) bf[c] = (ldA || ldB) ? __ldg(fg + c * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint32_t w0 = word(A[c >> 1], 2 * (c & 1)), w1 = word(A[c >> 1], 2 * (c & 1) + 1);
        const uint32_t a0 = w0 & 0x0F0F0F0Fu, a1 = (w0 >> 4) & 0x0F0F0F0Fu;
        const uint32_t a2 = w1 & 0x0F0F0F0Fu, a3 = (w1 >> 4) & 0x0F0F0F0Fu;
        mma_u8s8(C[0], a0, a1, a2, a3, ldA ? bf[c].x : 0u, ldB ? bf[c].x : 0u);
        mma_u8s8(C[1], a0, a1, a2, a3, ldA ? bf[c].y : 0u, ldB ? bf[c].y : 0u);
        mma_u8s8(C[2], a0, a1, a2, a3, ldA ? bf[c].z : 0u, ldB ? bf[c].z : 0u);
    }
    // C[p][0]: (row g, block 2t)  [1]: (g, 2t+1)  [2]: (g+8, 2t)  [3]: (g+8, 2t+1).
    // |D2| <= 64, so the combined integer fits int32: 32 * 15 * (64 * 65536 + 128 * 257) < 2^31.
    float T[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) T[k] = static_cast<float>(C[2][k] * 65536 + C[1][k] * 256 + C[0][k]);
    const float2 sc2 = __ldg(reinterpret_cast<const float2*>(sc_) + t);
    const float2 xs2 = __ldg(reinterpret_cast<const float2*>(xs_) + t);
    const float s0 = sc2.x, s1 = sc2.y, x0 = xs2.x, x1 = xs2.y;
    if (TYPE == T_Q4_K) {
        // six-bit scales / mins of sub-blocks 2t, 2t+1 (kquants.h:204-212), four per word
        const int sh = 16 * (t & 1);
        float sc[2][2], mn[2][2], d[2], dm[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 hh = h ? h8 : h0;
            const uint32_t scw = t < 2 ? (hh.y & 0x3F3F3F3Fu) : ((hh.w & 0x0F0F0F0Fu) | ((hh.y >> 2) & 0x30303030u));
            const uint32_t mw = t < 2 ? (hh.z & 0x3F3F3F3Fu)
                                      : (((hh.w >> 4) & 0x0F0F0F0Fu) | ((hh.z >> 2) & 0x30303030u));
            sc[h][0] = static_cast<float>((scw >> sh) & 0xFFu);
            sc[h][1] = static_cast<float>((scw >> (sh + 8)) & 0xFFu);
            mn[h][0] = static_cast<float>((mw >> sh) & 0xFFu);
            mn[h][1] = static_cast<float>((mw >> (sh + 8)) & 0xFFu);
            d[h] = h2f(hh.x);
            dm[h] = h2f(hh.x >> 16);
        }
        y0 = fmaf(d[0], fmaf(sc[0][0] * s0, T[0], sc[0][1] * s1 * T[1]),
                  fmaf(-dm[0], fmaf(mn[0][0], x0, mn[0][1] * x1), y0));
        y8 = fmaf(d[1], fmaf(sc[1][0] * s0, T[2], sc[1][1] * s1 * T[3]),
                  fmaf(-dm[1], fmaf(mn[1][0], x0, mn[1][1] * x1), y8));
    } else {
        // value = (q - 8) * d; d of (g, 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1)
        const float dg0 = h2f(d4.x), dg1 = h2f(d4.x >> 16), d80 = h2f(d4.y), d81 = h2f(d4.y >> 16);
        y0 = fmaf(dg0, fmaf(s0, T[0], -8.0f * x0), fmaf(dg1, fmaf(s1, T[1], -8.0f * x1), y0));
        y8 = fmaf(d80, fmaf(s0, T[2], -8.0f * x0), fmaf(d81, fmaf(s1, T[3], -8.0f * x1), y8));
    }
}

template <int TYPE>
__global__ void __launch_bounds__(kGemvThreads, 3) gemv_mma_kernel(const GemvArgs a) {
    __shared__ float red[kWarps][MMA_TILE_ROWS];
    __shared__ int64_t next_tile;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int64_t tile_bytes = a.ngroups * MMA_GROUP_BYTES;
    const bool bsrc = (g & 3) == t;  // this lane supplies a B (x digit) fragment
    const bool ldA = bsrc && g < 4, ldB = bsrc && g >= 4;
    uint4 bA = make_uint4(0, 0, 0, 0), bB = make_uint4(0, 0, 0, 0);

    // the first tile is static: start its weights towards L2 before waiting on xprep
    int64_t tile = blockIdx.x;
    if (lane == 0 && tile < a.ntiles)
        for (int d = 0; d < kPrefetch; ++d) {
            const int64_t gi = warp + int64_t(d) * kWarps;
            if (gi < a.ngroups) prefetch_l2(a.W + tile * tile_bytes + gi * MMA_GROUP_BYTES, MMA_GROUP_BYTES);
        }
    pdl_release();
    pdl_wait();  // x digits and the tile queue come from xprep_kernel

    while (tile < a.ntiles) {  // `tile` is CTA-uniform, so every thread runs the same iterations
        if (threadIdx.x == 0) next_tile = static_cast<int64_t>(gridDim.x) + atomicAdd(a.queue, 1);
        const uint8_t* tb = a.W + tile * tile_bytes;
        float y0 = 0.f, y8 = 0.f;
        for (int64_t gi = warp; gi < a.ngroups; gi += kWarps) {
            const int64_t ahead = gi + int64_t(kPrefetch) * kWarps;
            if (lane == 0 && ahead < a.ngroups) prefetch_l2(tb + ahead * MMA_GROUP_BYTES, MMA_GROUP_BYTES);
            group_dot<TYPE>(tb + gi * MMA_GROUP_BYTES, a.frags + gi * 64, a.scale + gi * 8, a.xsum + gi * 8, lane, g,
                            t, ldA, ldB, bA, bB, y0, y8);
        }
        y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
        y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
        if (t == 0) {
            red[warp][g] = y0;
            red[warp][g + 8] = y8;
        }
        __syncthreads();
        const int64_t nt = next_tile;
        if (threadIdx.x < MMA_TILE_ROWS) {
            float acc = 0.f;
            const int nw = static_cast<int>(a.ngroups < kWarps ? a.ngroups : kWarps);
            for (int w = 0; w < nw; ++w) acc += red[w][threadIdx.x];
            a.y[tile * MMA_TILE_ROWS + threadIdx.x] = acc;
        }
        // warm L2 with the next tile's first groups of this warp
        if (lane == 0 && nt < a.ntiles)
            for (int d = 0; d < kPrefetch; ++d) {
                const int64_t gi = warp + int64_t(d) * kWarps;
                if (gi < a.ngroups) prefetch_l2(a.W + nt * tile_bytes + gi * MMA_GROUP_BYTES, MMA_GROUP_BYTES);
            }
        __syncthreads();
        tile = nt;
    }
}

// ---------------------------------------------------------------------------
// repack between GGUF rows and the MMA layout: one warp per (tile, group),
// the group's 16 x 144 GGUF bytes staged in shared memory.
// ---------------------------------------------------------------------------
template <bool kPack>
__global__ void __launch_bounds__(128) mma_repack_kernel(int type, const uint8_t* __restrict__ src,
                                                         uint8_t* __restrict__ dst, int64_t K, int64_t ntiles) {
    __shared__ __align__(16) uint8_t stage[4][MMA_GROUP_BYTES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t ngroups = K / 256, row_bytes = ngroups * 144;
    const int64_t total = ntiles * ngroups;
    for (int64_t item = blockIdx.x * 4 + warp; item < total; item += int64_t(gridDim.x) * 4) {
        const int64_t tile = item / ngroups, gi = item % ngroups;
        uint8_t* st = stage[warp];
        const int64_t tbase = tile * MMA_TILE_ROWS * row_bytes;
        if (kPack) {
            for (int i = lane; i < MMA_GROUP_BYTES; i += 32) {
                const int r = i / 144, o = i % 144;
                st[i] = src[tbase + r * row_bytes + gi * 144 + o];
            }
            __syncwarp();
            // lane-local part of mma_pack_group: this lane's 64 A bytes
            const int g = lane >> 2, t = lane & 3;
            const uint8_t* r0 = st + g * 144;
            const uint8_t* r8 = st + (g + 8) * 144;
            uint8_t* out = dst + tbase + gi * MMA_GROUP_BYTES;
            for (int c = 0; c < 8; ++c)
                for (int kind = 0; kind < 2; ++kind) {
                    const int blk = t + 4 * kind;
                    uint32_t w = 0;
                    for (int j = 0; j < 4; ++j) {
                        const int v = 32 * blk + 4 * c + j;
                        w |= (q4_of(type, r0, 0, v) | (q4_of(type, r8, 0, v) << 4)) << (8 * j);
                    }
                    *reinterpret_cast<uint32_t*>(out + ((c >> 1) * 32 + lane) * 16 + 8 * (c & 1) + 4 * kind) = w;
                }
            if (type == T_Q4_K) {
                for (int i = lane; i < 256; i += 32) out[2048 + i] = st[(i >> 4) * 144 + (i & 15)];
            } else {
                for (int i = lane; i < 128; i += 32) {  // [g][t][h] fp16
                    const int h = i & 3, tt = (i >> 2) & 3, gg = i >> 4;
                    const int row = gg + 8 * (h >> 1), blk = 2 * tt + (h & 1);
                    out[2048 + 2 * i] = st[row * 144 + blk * 18];
                    out[2048 + 2 * i + 1] = st[row * 144 + blk * 18 + 1];
                }
            }
            __syncwarp();
        } else {
            const uint8_t* in = src + tbase + gi * MMA_GROUP_BYTES;
            for (int i = lane; i < MMA_GROUP_BYTES; i += 32) st[i] = in[i];
            __syncwarp();
            // rebuild GGUF bytes: each lane produces whole GGUF bytes (two nibbles)
            for (int i = lane; i < MMA_GROUP_BYTES; i += 32) {
                const int r = i / 144, o = i % 144;
                uint8_t v;
                if (type == T_Q4_K && o < 16) {
                    v = st[2048 + 16 * r + o];
                } else if (type == T_Q4_0 && (o % 18) < 2) {
                    const int blk = o / 18, gg = r & 7, h = 2 * (r >> 3) + (blk & 1), tt = blk >> 1;
                    v = st[2048 + ((gg * 4 + tt) * 4 + h) * 2 + (o % 18)];
                } else {
                    // the two values stored in this GGUF byte
                    int vals[2];
                    if (type == T_Q4_K) {
                        const int qb = o - 16, jp = qb >> 5, oo = qb & 31;  // sub-blocks 2jp (low), 2jp+1 (high)
                        vals[0] = 32 * (2 * jp) + oo;
                        vals[1] = 32 * (2 * jp + 1) + oo;
                    } else {
                        const int blk = o / 18, qb = o % 18 - 2;
                        vals[0] = 32 * blk + qb;
                        vals[1] = 32 * blk + qb + 16;
                    }
                    const int g = r & 7, half = r >> 3;
                    uint32_t byte = 0;
                    for (int n = 0; n < 2; ++n) {
                        const int vv = vals[n], blk = vv >> 5, within = vv & 31, c = within >> 2, j = within & 3;
                        const int t = blk & 3, kind = blk >> 2, ln = 4 * g + t;
                        const uint32_t w = *reinterpret_cast<const uint32_t*>(st + ((c >> 1) * 32 + ln) * 16 +
                                                                              8 * (c & 1) + 4 * kind);
                        const uint32_t q = (w >> (8 * j + 4 * half)) & 0xFu;
                        byte |= q << (4 * n);
                    }
                    v = static_cast<uint8_t>(byte);
                }
                dst[tbase + r * row_bytes + gi * 144 + o] = v;
            }
            __syncwarp();
        }
    }
}

// per-(device, stream) double-buffered x-digit scratch for the launcher API
struct ScratchEntry {
    int dev;
    cudaStream_t stream;
    void* ptr[2];
    size_t bytes;
    int next;
};

std::mutex g_scratch_mtx;
ScratchEntry g_scratch[64];
int g_scratch_n = 0;

}  // namespace

// Scratch of one MMA GEMV launch: x digits (1 KiB per 256 values), block
// scales and sums (per 32 values) and the tile queue counter, which
// xprep_kernel zeroes at the start of every launch.
ScratchLayout scratch_layout(int64_t N, int64_t K) {
    (void)N;
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    ScratchLayout L;
    const int64_t ngroups = K / 256;
    L.frags = 0;
    L.scale = up(L.frags + static_cast<size_t>(ngroups) * 1024);
    L.xsum = up(L.scale + static_cast<size_t>(K / 32) * sizeof(float));
    L.queue = up(L.xsum + static_cast<size_t>(K / 32) * sizeof(float));
    L.total = up(L.queue + sizeof(int));
    return L;
}

size_t xprep_bytes(int64_t N, int64_t K) { return scratch_layout(N, K).total; }

cudaError_t mma_repack_launch(int type, const void* raw, void* packed, int64_t N, int64_t K, bool pack,
                              cudaStream_t stream) {
    if (layout_kind(type, N, K) != 1) return cudaErrorInvalidValue;
    const int64_t ntiles = N / MMA_TILE_ROWS, items = ntiles * (K / 256);
    const int64_t blocks = (items + 3) / 4 < 65536 ? (items + 3) / 4 : 65536;
    if (pack)
        mma_repack_kernel<true><<<unsigned(blocks), 128, 0, stream>>>(type, static_cast<const uint8_t*>(raw),
                                                                     static_cast<uint8_t*>(packed), K, ntiles);
    else
        mma_repack_kernel<false><<<unsigned(blocks), 128, 0, stream>>>(type, static_cast<const uint8_t*>(raw),
                                                                      static_cast<uint8_t*>(packed), K, ntiles);
    return cudaGetLastError();
}

cudaError_t gemv_mma_launch(int type, const void* W, const float* x, float* y, int64_t N, int64_t K,
                            void* scratch, cudaStream_t stream, bool pdl) {
    const ScratchLayout L = scratch_layout(N, K);
    uint8_t* base = static_cast<uint8_t*>(scratch);
    GemvArgs a;
    a.W = static_cast<const uint8_t*>(W);
    a.frags = reinterpret_cast<const uint4*>(base + L.frags);
    a.scale = reinterpret_cast<const float*>(base + L.scale);
    a.xsum = reinterpret_cast<const float*>(base + L.xsum);
    a.y = y;
    a.queue = reinterpret_cast<int*>(base + L.queue);
    a.N = N;
    a.K = K;
    a.ntiles = N / MMA_TILE_ROWS;
    a.ngroups = K / 256;

    static int s_sms[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 16) return cudaErrorInvalidDevice;
    if (s_sms[dev] == 0) cudaDeviceGetAttribute(&s_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int sms = s_sms[dev] > 0 ? s_sms[dev] : 148;

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cudaLaunchConfig_t cp = {};
    const int64_t nblk = K / 32;
    cp.gridDim = dim3(static_cast<unsigned>((nblk + 1) / 2));  // one warp per 32-value block
    cp.blockDim = dim3(64);
    cp.stream = stream;
    cp.attrs = attr;
    cp.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cp, xprep_kernel, x, K, base + L.frags, reinterpret_cast<float*>(base + L.scale),
                                       reinterpret_cast<float*>(base + L.xsum), a.queue);
    if (e != cudaSuccess) return e;

    int64_t blocks = a.ntiles < int64_t(sms) * 3 ? a.ntiles : int64_t(sms) * 3;
    cudaLaunchConfig_t cg = {};
    cg.gridDim = dim3(static_cast<unsigned>(blocks < 1 ? 1 : blocks));
    cg.blockDim = dim3(kGemvThreads);
    cg.stream = stream;
    cudaLaunchAttribute attr2[1];
    attr2[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr2[0].val.programmaticStreamSerializationAllowed = 1;  // overlap the L2 warm-up with xprep
    cg.attrs = attr2;
    cg.numAttrs = 1;
    if (type == T_Q4_K) return cudaLaunchKernelEx(&cg, gemv_mma_kernel<T_Q4_K>, a);
    if (type == T_Q4_0) return cudaLaunchKernelEx(&cg, gemv_mma_kernel<T_Q4_0>, a);
    return cudaErrorInvalidValue;
}

// Scratch for launcher calls that bring none: two slots per (device, stream),
// alternated so that a GEMV reading one slot can overlap (PDL) the next call's
// x preparation writing the other.  Grown on demand (must not happen inside
// stream capture: the first call for a new, larger K allocates).
void* launcher_scratch(cudaStream_t stream, int64_t N, int64_t K) {
    const size_t need = xprep_bytes(N, K);
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_scratch_mtx);
    ScratchEntry* e = nullptr;
    for (int i = 0; i < g_scratch_n; ++i)
        if (g_scratch[i].dev == dev && g_scratch[i].stream == stream) e = &g_scratch[i];
    if (!e) {
        if (g_scratch_n >= 64) return nullptr;
        e = &g_scratch[g_scratch_n++];
        *e = ScratchEntry{dev, stream, {nullptr, nullptr}, 0, 0};
    }
    if (e->bytes < need) {
        size_t cap = need < (1u << 20) ? (1u << 20) : need;
        for (int s = 0; s < 2; ++s) {
            if (e->ptr[s]) cudaFree(e->ptr[s]);
            e->ptr[s] = nullptr;
            if (cudaMalloc(&e->ptr[s], cap) != cudaSuccess || cudaMemset(e->ptr[s], 0, cap) != cudaSuccess) {
                e->bytes = 0;
                return nullptr;
            }
        }
        e->bytes = cap;
    }
    void* p = e->ptr[e->next];
    e->next ^= 1;
    return p;
}

}  // namespace xb
