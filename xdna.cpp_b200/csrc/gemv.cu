// Dequant-GEMV kernels for sm_100a: y[N] = W[N,K] x[K], W in the stripe-tile
// layout of formats.cuh, x and y F32.  M = 1 is a bandwidth-bound contraction
// (about 3.6 flop per weight byte), so there are no tensor cores here.
//
// Work split.  One warp owns one tile of TILE_ROWS rows at a time; its lanes
// stride over the row's units (32 or 128 values each).  For every unit a lane
// loads the 16-byte payload pieces of all the tile's rows (coalesced 512-byte
// warp loads, L1 no-allocate), reads the matching slice of x once from shared
// memory and applies it to every row (x reuse = TILE_ROWS), unpacks the quant
// bits in registers and accumulates in F32.  A warp-shuffle reduction finishes
// each tile.  x is staged once per CTA into shared memory with a 16-byte pad per
// unit so the lanes' 128-bit reads are bank-conflict free; IQ grids live in
// shared memory.
//
// Small unsigned integers become floats with the 2^23 magic: the byte is
// placed in the mantissa of 0x4B000000 by one byte_perm and the bias (2^23 plus
// the format's zero point) is removed by one FADD, exactly.
//
// Programmatic dependent launch: every kernel waits on griddepcontrol before
// touching x or y and releases its dependents immediately, so a chain of
// GEMVs (a decode step) overlaps launch latency.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "formats.cuh"
#include "gemv.cuh"
#include "iq_tables.h"  // generated at build time from the gguf package

namespace xb {

namespace {

constexpr int kThreads = 256;
constexpr int kItemRows = 2;  // rows per warp work item (x reuse factor)
static_assert(TILE_ROWS % kItemRows == 0, "items must not straddle tiles");
constexpr int kWarps = kThreads / 32;
constexpr float kMagic = 8388608.0f;  // 2^23

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned int*>(p));
}
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned short*>(p));
}
__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}
__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
// float(2^23 + byte i of w)
__device__ __forceinline__ float bmag(uint32_t w, int i) {
    return __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7440u + i)));
}
// 16 consecutive floats of x from shared memory
__device__ __forceinline__ void load_x16(const float* xs, float (&xv)[16]) {
    const float4* p = reinterpret_cast<const float4*>(xs);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 v = p[k];
        xv[4 * k + 0] = v.x;
        xv[4 * k + 1] = v.y;
        xv[4 * k + 2] = v.z;
        xv[4 * k + 3] = v.w;
    }
}
// sum_{i<16} (byte_i(w[0..3]) - off) * xv[i]  for four words of byte values
__device__ __forceinline__ float dot16_bytes(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                             float off, const float (&xv)[16]) {
    const uint32_t w[4] = {w0, w1, w2, w3};
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        s0 = fmaf(bmag(w[k], 0) - off, xv[4 * k + 0], s0);
        s1 = fmaf(bmag(w[k], 1) - off, xv[4 * k + 1], s1);
        s0 = fmaf(bmag(w[k], 2) - off, xv[4 * k + 2], s0);
        s1 = fmaf(bmag(w[k], 3) - off, xv[4 * k + 3], s1);
    }
    return s0 + s1;
}

// ---------------------------------------------------------------------------
// shared-memory layout helpers
// ---------------------------------------------------------------------------
template <int UV>
struct XLayout {
    static constexpr int kStride = UV + 4;  // floats per unit incl. 16-byte pad
};

struct SmemPtrs {
    const float* xs;    // staged x, padded per unit
    const float* xs32;  // per-32-value sums of x (Q4_K / Q5_K)
    const uint32_t* grid32;
    const uint2* grid64;
};

// ---------------------------------------------------------------------------
// Per-format unit decoders.  Each accumulates, for rows r < trt of the tile,
// the dot product of unit u with x into acc[r].
// ---------------------------------------------------------------------------
template <int TR, int P>
struct Pieces {
    uint4 v[TR][P];
};

// The rows a warp works on: rows r0 .. r0 + nr - 1 of a stripe tile holding
// trt rows (the kernel's register tile is kItemRows <= TILE_ROWS rows).
struct RowCtx {
    const uint8_t* tile;
    int trt;
    int r0;
    int nr;
};

// Q4_0: unit = one block (32 values).  value = (q - 8) * d.
struct DecQ4_0 {
    static constexpr int kType = T_Q4_0, kUV = 32, kP = 1, kNeedXsum = 0;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        float xl[16], xh[16];
        load_x16(xu, xl);
        load_x16(xu + 16, xh);
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            const float d = h2f(ld_u16(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, u)));
            const uint4 q = pc.v[r][0];
            const float s_lo = dot16_bytes(q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q.z & 0x0F0F0F0Fu,
                                           q.w & 0x0F0F0F0Fu, kMagic + 8.0f, xl);
            const float s_hi = dot16_bytes((q.x >> 4) & 0x0F0F0F0Fu, (q.y >> 4) & 0x0F0F0F0Fu,
                                           (q.z >> 4) & 0x0F0F0F0Fu, (q.w >> 4) & 0x0F0F0F0Fu,
                                           kMagic + 8.0f, xh);
            acc[r] = fmaf(d, s_lo + s_hi, acc[r]);
        }
    }
};

// 6-bit scale/min pair j (0..7) of a K-quant super-block (kquants.h:204-212).
__device__ __forceinline__ void scale_min_k4(int j, const uint32_t (&s)[3], float& sc, float& m) {
    auto byte = [&](int i) -> uint32_t { return (s[i >> 2] >> (8 * (i & 3))) & 0xffu; };
    uint32_t d, mm;
    if (j < 4) {
        d = byte(j) & 63u;
        mm = byte(j + 4) & 63u;
    } else {
        d = (byte(j + 4) & 0x0fu) | ((byte(j - 4) >> 6) << 4);
        mm = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
    sc = static_cast<float>(d);
    m = static_cast<float>(mm);
}

// Q4_K / Q5_K: unit h of a super-block = values 128h..128h+127 = qs bytes
// [64h, 64h+64) = pieces 0..3.  Piece p holds qs[64h+16p .. +16]: low
// nibbles are values 64(p/2) + 16(p%2) + i, high nibbles 32 further on.
// Q5_K's piece 4 holds the transposed qh planes W[2*jj + n].
template <bool kFive>
struct DecQ45_K {
    static constexpr int kType = kFive ? T_Q5_K : T_Q4_K, kUV = 128, kP = kFive ? 5 : 4, kNeedXsum = 1;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        const int64_t b = u >> 1;
        const int h = static_cast<int>(u & 1);
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        const float* xsum = sm.xs32 + u * 4;
        float dsc[TR][4], dmn[TR][4];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            const uint32_t dd = ld_u32(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, b));
            const float d = h2f(dd), dmin = h2f(dd >> 16);
            const uint8_t* ap = rc.tile + tile_aux_off(g, rc.trt, rc.r0 + r, b);
            const uint32_t s[3] = {ld_u32(ap), ld_u32(ap + 4), ld_u32(ap + 8)};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float sc, m;
                scale_min_k4(4 * h + k, s, sc, m);
                dsc[r][k] = d * sc;
                dmn[r][k] = dmin * m;
            }
        }
        float S[TR][4];
#pragma unroll
        for (int r = 0; r < TR; ++r)
#pragma unroll
            for (int k = 0; k < 4; ++k) S[r][k] = 0.f;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int jj = p >> 1, half = p & 1;
            float xl[16], xh[16];
            load_x16(xu + 64 * jj + 16 * half, xl);
            load_x16(xu + 64 * jj + 32 + 16 * half, xh);
#pragma unroll
            for (int r = 0; r < TR; ++r) {
                if (r >= rc.nr) break;
                const uint4 q = pc.v[r][p];
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const uint32_t w = word(q, wi);
                    lo[wi] = w & 0x0F0F0F0Fu;
                    hi[wi] = (w >> 4) & 0x0F0F0F0Fu;
                    if constexpr (kFive) {
                        const int k = 4 * half + wi;
                        const uint32_t w0 = word(pc.v[r][4], 2 * jj + 0);
                        const uint32_t w1 = word(pc.v[r][4], 2 * jj + 1);
                        lo[wi] |= ((w0 >> k) & 0x01010101u) << 4;
                        hi[wi] |= ((w1 >> k) & 0x01010101u) << 4;
                    }
                }
                S[r][2 * jj] += dot16_bytes(lo[0], lo[1], lo[2], lo[3], kMagic, xl);
                S[r][2 * jj + 1] += dot16_bytes(hi[0], hi[1], hi[2], hi[3], kMagic, xh);
            }
        }
        const float x0 = xsum[0], x1 = xsum[1], x2 = xsum[2], x3 = xsum[3];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            float a = acc[r];
            a = fmaf(dsc[r][0], S[r][0], a);
            a = fmaf(dsc[r][1], S[r][1], a);
            a = fmaf(dsc[r][2], S[r][2], a);
            a = fmaf(dsc[r][3], S[r][3], a);
            a = fmaf(-dmn[r][0], x0, a);
            a = fmaf(-dmn[r][1], x1, a);
            a = fmaf(-dmn[r][2], x2, a);
            a = fmaf(-dmn[r][3], x3, a);
            acc[r] = a;
        }
    }
};

// Q3_K 16 six-bit scales from the 12-byte record (kquants.h:366-373);
// returns scale index i in 0..15.
__device__ __forceinline__ int q3k_scale(const uint32_t (&a)[3], int i) {
    const uint32_t kmask1 = 0x03030303u, kmask2 = 0x0f0f0f0fu;
    uint32_t w;
    switch (i >> 2) {
        case 0: w = (a[0] & kmask2) | (((a[2] >> 0) & kmask1) << 4); break;
        case 1: w = (a[1] & kmask2) | (((a[2] >> 2) & kmask1) << 4); break;
        case 2: w = ((a[0] >> 4) & kmask2) | (((a[2] >> 4) & kmask1) << 4); break;
        default: w = ((a[1] >> 4) & kmask2) | (((a[2] >> 6) & kmask1) << 4); break;
    }
    return static_cast<int>((w >> (8 * (i & 3))) & 0xffu);
}

// Q3_K: unit h: pieces 0,1 = qs[32h + 16s + i] (s = piece), bits 2*j2 give the
// low two bits of value 32*j2 + 16s + i; piece 2 = transposed hmask planes
// H[j2].  value = (q2 | hbit << 2) - 4, scale index 8h + 2*j2 + s.
struct DecQ3_K {
    static constexpr int kType = T_Q3_K, kUV = 128, kP = 3, kNeedXsum = 0;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        const int64_t b = u >> 1;
        const int h = static_cast<int>(u & 1);
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        float dl[TR][8];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            const float d = h2f(ld_u16(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, b)));
            const uint8_t* ap = rc.tile + tile_aux_off(g, rc.trt, rc.r0 + r, b);
            const uint32_t a[3] = {ld_u32(ap), ld_u32(ap + 4), ld_u32(ap + 8)};
#pragma unroll
            for (int k = 0; k < 8; ++k) dl[r][k] = d * static_cast<float>(q3k_scale(a, 8 * h + k) - 32);
        }
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                float xv[16];
                load_x16(xu + 32 * j2 + 16 * s, xv);
#pragma unroll
                for (int r = 0; r < TR; ++r) {
                    if (r >= rc.nr) break;
                    const uint4 q = pc.v[r][s];
                    const uint32_t H = word(pc.v[r][2], j2);
                    uint32_t v[4];
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi) {
                        const int k = 4 * s + wi;
                        v[wi] = ((word(q, wi) >> (2 * j2)) & 0x03030303u) | (((H >> k) & 0x01010101u) << 2);
                    }
                    acc[r] = fmaf(dl[r][2 * j2 + s], dot16_bytes(v[0], v[1], v[2], v[3], kMagic + 4.0f, xv), acc[r]);
                }
            }
        }
    }
};

// Q6_K: unit h: pieces 0..3 = ql[64h + 16p + i], pieces 4,5 = qh[32h + 16(p%2) + i].
// Low nibble of ql piece p is value 32(p/2) + 16(p%2) + i (sub-block p), high
// nibble is 64 further on (sub-block 4 + p); qh supplies bits 4,5 from bit
// pair 2m, m = p/2 (+2 for high).  value = q6 - 32, int8 scale per 16 values.
struct DecQ6_K {
    static constexpr int kType = T_Q6_K, kUV = 128, kP = 6, kNeedXsum = 0;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        const int64_t b = u >> 1;
        const int h = static_cast<int>(u & 1);
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        float dl[TR][8];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            const float d = h2f(ld_u16(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, b)));
            const uint8_t* ap = rc.tile + tile_aux_off(g, rc.trt, rc.r0 + r, b);
            const uint32_t s0 = ld_u32(ap + 8 * h), s1 = ld_u32(ap + 8 * h + 4);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t sw = k < 4 ? s0 : s1;
                const int sc = static_cast<int>(static_cast<int8_t>((sw >> (8 * (k & 3))) & 0xffu));
                dl[r][k] = d * static_cast<float>(sc);
            }
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int m = p >> 1;
            float xl[16], xh[16];
            load_x16(xu + 32 * m + 16 * (p & 1), xl);
            load_x16(xu + 64 + 32 * m + 16 * (p & 1), xh);
#pragma unroll
            for (int r = 0; r < TR; ++r) {
                if (r >= rc.nr) break;
                const uint4 ql = pc.v[r][p];
                const uint4 qh = pc.v[r][4 + (p & 1)];
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const uint32_t w = word(ql, wi), hw = word(qh, wi);
                    lo[wi] = (w & 0x0F0F0F0Fu) | (((hw >> (2 * m)) & 0x03030303u) << 4);
                    hi[wi] = ((w >> 4) & 0x0F0F0F0Fu) | (((hw >> (2 * m + 4)) & 0x03030303u) << 4);
                }
                float a = acc[r];
                a = fmaf(dl[r][p], dot16_bytes(lo[0], lo[1], lo[2], lo[3], kMagic + 32.0f, xl), a);
                a = fmaf(dl[r][4 + p], dot16_bytes(hi[0], hi[1], hi[2], hi[3], kMagic + 32.0f, xh), a);
                acc[r] = a;
            }
        }
    }
};

// byte-wise 16-entry table lookup: t0..t3 hold entries 0..15 as bytes; q holds
// four 4-bit indices in the low nibble of each byte.
__device__ __forceinline__ uint32_t lut16(uint32_t q, uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3) {
    const uint32_t s = q | (q >> 4);                    // idx0|idx1<<4 in byte 0, idx2|idx3<<4 in byte 2
    const uint32_t s16 = __byte_perm(s, 0u, 0x4420u);   // four 4-bit selectors
    const uint32_t s7 = s16 & 0x7777u;
    const uint32_t lo = __byte_perm(t0, t1, s7);
    const uint32_t hi = __byte_perm(t2, t3, s7);
    const uint32_t pick = ((s16 >> 1) & 0x4444u) | 0x3210u;
    return __byte_perm(lo, hi, pick);
}

// IQ4_XS: unit h: piece p = sub-block ib = 4h + p (qs[16 ib + i]); low nibble
// value 32p + i, high nibble 32p + 16 + i.  value = kvalues[q] * d * (ls - 32).
struct DecIQ4_XS {
    static constexpr int kType = T_IQ4_XS, kUV = 128, kP = 4, kNeedXsum = 0;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        // kvalues + 128 as bytes (all in 1..241)
        constexpr uint32_t t0 = XB_IQ4NL_U8_0, t1 = XB_IQ4NL_U8_1, t2 = XB_IQ4NL_U8_2, t3 = XB_IQ4NL_U8_3;
        const int64_t b = u >> 1;
        const int h = static_cast<int>(u & 1);
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        float dl[TR][4];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            const uint32_t dd = ld_u32(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, b));  // d | scales_h << 16
            const float d = h2f(dd);
            const uint32_t sh = dd >> 16;
            const uint32_t sl = ld_u32(rc.tile + tile_aux_off(g, rc.trt, rc.r0 + r, b));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ib = 4 * h + k;
                const int ls = static_cast<int>(((sl >> (4 * ib)) & 0x0fu) | (((sh >> (2 * ib)) & 3u) << 4));
                dl[r][k] = d * static_cast<float>(ls - 32);
            }
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            float xl[16], xh[16];
            load_x16(xu + 32 * p, xl);
            load_x16(xu + 32 * p + 16, xh);
#pragma unroll
            for (int r = 0; r < TR; ++r) {
                if (r >= rc.nr) break;
                const uint4 q = pc.v[r][p];
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const uint32_t w = word(q, wi);
                    lo[wi] = lut16(w & 0x0F0F0F0Fu, t0, t1, t2, t3);
                    hi[wi] = lut16((w >> 4) & 0x0F0F0F0Fu, t0, t1, t2, t3);
                }
                const float s = dot16_bytes(lo[0], lo[1], lo[2], lo[3], kMagic + 128.0f, xl) +
                                dot16_bytes(hi[0], hi[1], hi[2], hi[3], kMagic + 128.0f, xh);
                acc[r] = fmaf(dl[r][p], s, acc[r]);
            }
        }
    }
};

// Signed 4-value dot with a 4-byte grid entry: sum_c grid_c * (+-1) * x_c,
// sign bit c of `sbits`.
__device__ __forceinline__ float grid4_dot(uint32_t gw, uint32_t sbits, const float* xv) {
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float gv = bmag(gw, c) - kMagic;
        const float xs = __int_as_float(__float_as_int(xv[c]) ^ static_cast<int>(((sbits >> c) & 1u) << 31));
        s = fmaf(gv, xs, s);
    }
    return s;
}

// IQ3_S: unit h, sub-block sb (ib = 4h + sb): grid indices qs[8 ib + gi] (unit
// bytes 8 sb + gi, pieces 0,1) with bit gi of qh[ib] as bit 8; sign byte
// 4 sb + gi/2 of piece 2, bits 4(gi%2)+c.  db = d (1 + 2 s).
struct DecIQ3_S {
    static constexpr int kType = T_IQ3_S, kUV = 128, kP = 3, kNeedXsum = 0;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        const int64_t b = u >> 1;
        const int h = static_cast<int>(u & 1);
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        uint32_t qhw[TR], scw[TR];
        float d[TR];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            d[r] = h2f(ld_u16(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, b)));
            const uint8_t* ap = rc.tile + tile_aux_off(g, rc.trt, rc.r0 + r, b);
            qhw[r] = ld_u32(ap + 4 * h);  // qh[4h .. 4h+3]
            scw[r] = ld_u32(ap + 8);      // scales[0..3]
        }
#pragma unroll
        for (int sb = 0; sb < 4; ++sb) {
            const int ib = 4 * h + sb;
            float xv[32];
            load_x16(xu + 32 * sb, *reinterpret_cast<float(*)[16]>(&xv[0]));
            load_x16(xu + 32 * sb + 16, *reinterpret_cast<float(*)[16]>(&xv[16]));
#pragma unroll
            for (int r = 0; r < TR; ++r) {
                if (r >= rc.nr) break;
                const uint32_t qa = word(pc.v[r][sb >> 1], 2 * (sb & 1));
                const uint32_t qb = word(pc.v[r][sb >> 1], 2 * (sb & 1) + 1);
                const uint32_t sg = word(pc.v[r][2], sb);
                const uint32_t qh = (qhw[r] >> (8 * sb)) & 0xffu;
                float s = 0.f;
#pragma unroll
                for (int gi = 0; gi < 8; ++gi) {
                    const uint32_t qb8 = ((gi < 4 ? qa : qb) >> (8 * (gi & 3))) & 0xffu;
                    const uint32_t idx = qb8 | (((qh >> gi) & 1u) << 8);
                    const uint32_t gw = sm.grid32[idx];
                    const uint32_t sbits = (sg >> (8 * (gi >> 1) + 4 * (gi & 1))) & 0x0fu;
                    s += grid4_dot(gw, sbits, &xv[4 * gi]);
                }
                const float sc = static_cast<float>((scw[r] >> (4 * ib)) & 0x0fu);
                acc[r] = fmaf(d[r] * (1.0f + 2.0f * sc), s, acc[r]);
            }
        }
    }
};

// IQ3_XXS: unit h, sub-block sb: grid indices qs bytes 8 sb + gi (pieces 0,1);
// aux word sb of piece 2 = 4 x 7-bit sign index | scale << 28.  The eighth
// sign bit of each byte makes the number of negative signs even.
struct DecIQ3_XXS {
    static constexpr int kType = T_IQ3_XXS, kUV = 128, kP = 3, kNeedXsum = 0;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        const int64_t b = u >> 1;
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        float d[TR];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            d[r] = h2f(ld_u16(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, b)));
        }
#pragma unroll
        for (int sb = 0; sb < 4; ++sb) {
            float xv[32];
            load_x16(xu + 32 * sb, *reinterpret_cast<float(*)[16]>(&xv[0]));
            load_x16(xu + 32 * sb + 16, *reinterpret_cast<float(*)[16]>(&xv[16]));
#pragma unroll
            for (int r = 0; r < TR; ++r) {
                if (r >= rc.nr) break;
                const uint32_t qa = word(pc.v[r][sb >> 1], 2 * (sb & 1));
                const uint32_t qb = word(pc.v[r][sb >> 1], 2 * (sb & 1) + 1);
                const uint32_t aux = word(pc.v[r][2], sb);
                float s = 0.f;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    const uint32_t s7 = (aux >> (7 * l)) & 127u;
                    const uint32_t signs = s7 | ((__popc(s7) & 1u) << 7);
                    const uint32_t qw = l < 2 ? qa : qb;
                    const uint32_t i1 = (qw >> (16 * (l & 1))) & 0xffu;
                    const uint32_t i2 = (qw >> (16 * (l & 1) + 8)) & 0xffu;
                    s += grid4_dot(sm.grid32[i1], signs & 0x0fu, &xv[8 * l]);
                    s += grid4_dot(sm.grid32[i2], signs >> 4, &xv[8 * l + 4]);
                }
                const float db = d[r] * (0.5f + static_cast<float>(aux >> 28)) * 0.5f;
                acc[r] = fmaf(db, s, acc[r]);
            }
        }
    }
};

// IQ2_S: unit h, sub-block sb (ib = 4h + sb): grid index qs byte 4 sb + l
// (piece 0) | ((qh[ib] >> 2l) & 3) << 8 into the 1024 x 8 grid; sign byte
// 4 sb + l of piece 1; scale nibble 0 for l < 2, nibble 1 for l >= 2,
// db = d (0.5 + s) / 4.
struct DecIQ2_S {
    static constexpr int kType = T_IQ2_S, kUV = 128, kP = 2, kNeedXsum = 0;
    template <int TR>
    static __device__ __forceinline__ void unit(const Geometry& g, const RowCtx& rc, int64_t u,
                                                const Pieces<TR, kP>& pc, const SmemPtrs& sm, float (&acc)[TR]) {
        const int64_t b = u >> 1;
        const int h = static_cast<int>(u & 1);
        const float* xu = sm.xs + u * XLayout<kUV>::kStride;
        uint32_t qhw[TR], scw[TR];
        float d[TR];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (r >= rc.nr) break;
            d[r] = h2f(ld_u16(rc.tile + tile_d_off(g, rc.trt, rc.r0 + r, b)));
            const uint8_t* ap = rc.tile + tile_aux_off(g, rc.trt, rc.r0 + r, b);
            qhw[r] = ld_u32(ap + 4 * h);      // qh[4h .. 4h+3]
            scw[r] = ld_u32(ap + 8 + 4 * h);  // scales[4h .. 4h+3]
        }
#pragma unroll
        for (int sb = 0; sb < 4; ++sb) {
            float xv[32];
            load_x16(xu + 32 * sb, *reinterpret_cast<float(*)[16]>(&xv[0]));
            load_x16(xu + 32 * sb + 16, *reinterpret_cast<float(*)[16]>(&xv[16]));
#pragma unroll
            for (int r = 0; r < TR; ++r) {
                if (r >= rc.nr) break;
                const uint32_t qw = word(pc.v[r][0], sb);
                const uint32_t sg = word(pc.v[r][1], sb);
                const uint32_t qh = (qhw[r] >> (8 * sb)) & 0xffu;
                const uint32_t sc = (scw[r] >> (8 * sb)) & 0xffu;
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    const uint32_t idx = ((qw >> (8 * l)) & 0xffu) | (((qh >> (2 * l)) & 3u) << 8);
                    const uint2 gw = sm.grid64[idx];
                    const uint32_t sb8 = (sg >> (8 * l)) & 0xffu;
                    const float t = grid4_dot(gw.x, sb8 & 0x0fu, &xv[8 * l]) +
                                    grid4_dot(gw.y, sb8 >> 4, &xv[8 * l + 4]);
                    if (l < 2) s0 += t; else s1 += t;
                }
                const float db0 = d[r] * (0.5f + static_cast<float>(sc & 0x0fu)) * 0.25f;
                const float db1 = d[r] * (0.5f + static_cast<float>(sc >> 4)) * 0.25f;
                acc[r] = fmaf(db0, s0, fmaf(db1, s1, acc[r]));
            }
        }
    }
};

// ---------------------------------------------------------------------------
// the tile kernel
// ---------------------------------------------------------------------------
template <class D>
__host__ __device__ constexpr int grid_words() {
    return D::kType == T_IQ3_S ? 512 : (D::kType == T_IQ3_XXS ? 256 : (D::kType == T_IQ2_S ? 2048 : 0));
}

template <class D>
size_t smem_bytes(int64_t K) {
    const int64_t nu = K / D::kUV;
    size_t bytes = static_cast<size_t>(nu) * XLayout<D::kUV>::kStride * sizeof(float);
    if (D::kNeedXsum) bytes += static_cast<size_t>(K / 32) * sizeof(float);
    bytes = (bytes + 15) & ~size_t(15);
    bytes += static_cast<size_t>(grid_words<D>()) * sizeof(uint32_t);
    return bytes;
}

template <class D>
__global__ void __launch_bounds__(kThreads, 2) gemv_tiles_kernel(const uint8_t* __restrict__ W,
                                                              const float* __restrict__ x,
                                                              float* __restrict__ y, int64_t N, int64_t K) {
    constexpr int TR = kItemRows;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const Geometry g = make_geometry(D::kType, N, K);
    float* xs = reinterpret_cast<float*>(smem_raw);
    float* xs32 = xs + g.nu * XLayout<D::kUV>::kStride;
    size_t off = static_cast<size_t>(g.nu) * XLayout<D::kUV>::kStride * sizeof(float);
    if (D::kNeedXsum) off += static_cast<size_t>(K / 32) * sizeof(float);
    off = (off + 15) & ~size_t(15);
    uint32_t* grid = reinterpret_cast<uint32_t*>(smem_raw + off);

    pdl_release();
    pdl_wait();

    // stage x (K is a multiple of 32, so of 4)
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int64_t i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = __ldg(x4 + i);
        const int64_t e = 4 * i;
        float* dst = xs + (e / D::kUV) * XLayout<D::kUV>::kStride + (e % D::kUV);
        *reinterpret_cast<float4*>(dst) = v;
    }
    if constexpr (grid_words<D>() > 0) {
        const uint32_t* src = D::kType == T_IQ3_S ? kIq3sGrid
                              : (D::kType == T_IQ3_XXS ? kIq3xxsGrid
                                                       : reinterpret_cast<const uint32_t*>(kIq2sGrid));
        for (int i = threadIdx.x; i < grid_words<D>(); i += blockDim.x) grid[i] = src[i];
    }
    __syncthreads();
    if constexpr (D::kNeedXsum) {
        for (int64_t s = threadIdx.x; s < K / 32; s += blockDim.x) {
            const int64_t e = 32 * s;
            const float* p = xs + (e / D::kUV) * XLayout<D::kUV>::kStride + (e % D::kUV);
            float a = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) a += p[i];
            xs32[s] = a;
        }
        __syncthreads();
    }

    SmemPtrs sm{xs, xs32, grid, reinterpret_cast<const uint2*>(grid)};
    const int lane = threadIdx.x & 31;
    const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    const int64_t total_warps = static_cast<int64_t>(gridDim.x) * kWarps;

    const int64_t nitems = (N + kItemRows - 1) / kItemRows;
    for (int64_t it = warp_global; it < nitems; it += total_warps) {
        const int64_t row = it * kItemRows;
        const int64_t t = row / TILE_ROWS;
        RowCtx rc;
        rc.trt = static_cast<int>(N - t * TILE_ROWS < TILE_ROWS ? N - t * TILE_ROWS : TILE_ROWS);
        rc.r0 = static_cast<int>(row - t * TILE_ROWS);
        rc.nr = static_cast<int>(N - row < kItemRows ? N - row : kItemRows);
        rc.tile = W + t * TILE_ROWS * g.row_bytes;
        float acc[TR];
#pragma unroll
        for (int r = 0; r < TR; ++r) acc[r] = 0.f;
        for (int64_t u = lane; u < g.nu; u += 32) {
            Pieces<TR, D::kP> pc;
#pragma unroll
            for (int r = 0; r < TR; ++r)
#pragma unroll
                for (int p = 0; p < D::kP; ++p)
                    pc.v[r][p] = r < rc.nr ? ld_stream(rc.tile + tile_payload_off(g, rc.trt, p, rc.r0 + r, u))
                                           : make_uint4(0, 0, 0, 0);
            D::template unit<TR>(g, rc, u, pc, sm, acc);
        }
#pragma unroll
        for (int r = 0; r < TR; ++r) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < TR; ++r)
                if (r < rc.nr) y[row + r] = acc[r];
        }
    }
}

// Per-device launch geometry of one kernel instantiation, cached so that a
// launch costs one cudaGetDevice plus the launch itself.
struct LaunchCache {
    std::mutex mtx;
    int sms[kMaxDevices] = {};
    size_t smem_set[kMaxDevices] = {};
    // last few (smem bytes -> resident CTAs per SM) answers per device
    size_t occ_smem[kMaxDevices][4] = {};
    int occ_val[kMaxDevices][4] = {};
    int occ_next[kMaxDevices] = {};
};

template <class D>
cudaError_t launch_typed(const uint8_t* W, const float* x, float* y, int64_t N, int64_t K, cudaStream_t stream,
                         const LaunchOpts& opts) {
    static LaunchCache cache;
    const size_t smem = smem_bytes<D>(K);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    int sms = 0, per_sm = 0;
    {
        std::lock_guard<std::mutex> lk(cache.mtx);
        if (cache.sms[dev] == 0) {
            e = cudaDeviceGetAttribute(&cache.sms[dev], cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return e;
        }
        sms = cache.sms[dev];
        if (smem > cache.smem_set[dev]) {
            e = cudaFuncSetAttribute(gemv_tiles_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            cache.smem_set[dev] = smem;
        }
        for (int i = 0; i < 4; ++i)
            if (cache.occ_smem[dev][i] == smem && cache.occ_val[dev][i] > 0) per_sm = cache.occ_val[dev][i];
        if (per_sm == 0) {
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_tiles_kernel<D>, kThreads, smem);
            if (e != cudaSuccess) return e;
            if (per_sm <= 0) return cudaErrorInvalidConfiguration;
            const int slot = cache.occ_next[dev];
            cache.occ_next[dev] = (slot + 1) & 3;
            cache.occ_smem[dev][slot] = smem;
            cache.occ_val[dev][slot] = per_sm;
        }
    }
    const int64_t nitems = (N + kItemRows - 1) / kItemRows;
    int64_t blocks = (nitems + kWarps - 1) / kWarps;
    const int64_t cap = static_cast<int64_t>(sms) * per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = opts.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_tiles_kernel<D>, W, x, y, N, K);
}

}  // namespace

cudaError_t gemv_launch(int type, const void* W, const float* x, float* y, int64_t N, int64_t K,
                        cudaStream_t stream, const LaunchOpts& opts) {
    if (N == 0) return cudaSuccess;
    if (layout_kind(type, N, K) == 1) {
        void* scratch = opts.scratch ? opts.scratch : launcher_scratch(stream, N, K);
        if (!scratch) return cudaErrorMemoryAllocation;
        return gemv_mma_launch(type, W, x, y, N, K, scratch, stream, opts.pdl, opts.feed, opts.x_ready, opts.classic);
    }
    const uint8_t* w = static_cast<const uint8_t*>(W);
    switch (type) {
        case T_Q4_0: return launch_typed<DecQ4_0>(w, x, y, N, K, stream, opts);
        case T_Q4_K: return launch_typed<DecQ45_K<false>>(w, x, y, N, K, stream, opts);
        case T_Q5_K: return launch_typed<DecQ45_K<true>>(w, x, y, N, K, stream, opts);
        case T_Q3_K: return launch_typed<DecQ3_K>(w, x, y, N, K, stream, opts);
        case T_Q6_K: return launch_typed<DecQ6_K>(w, x, y, N, K, stream, opts);
        case T_IQ4_XS: return launch_typed<DecIQ4_XS>(w, x, y, N, K, stream, opts);
        case T_IQ3_S: return launch_typed<DecIQ3_S>(w, x, y, N, K, stream, opts);
        case T_IQ3_XXS: return launch_typed<DecIQ3_XXS>(w, x, y, N, K, stream, opts);
        case T_IQ2_S: return launch_typed<DecIQ2_S>(w, x, y, N, K, stream, opts);
        default: return cudaErrorInvalidValue;
    }
}

size_t gemv_smem_bytes(int type, int64_t K) {
    switch (type) {
        case T_Q4_0: return smem_bytes<DecQ4_0>(K);
        case T_Q4_K: return smem_bytes<DecQ45_K<false>>(K);
        case T_Q5_K: return smem_bytes<DecQ45_K<true>>(K);
        case T_Q3_K: return smem_bytes<DecQ3_K>(K);
        case T_Q6_K: return smem_bytes<DecQ6_K>(K);
        case T_IQ4_XS: return smem_bytes<DecIQ4_XS>(K);
        case T_IQ3_S: return smem_bytes<DecIQ3_S>(K);
        case T_IQ3_XXS: return smem_bytes<DecIQ3_XXS>(K);
        case T_IQ2_S: return smem_bytes<DecIQ2_S>(K);
        default: return 0;
    }
}

}  // namespace xb
