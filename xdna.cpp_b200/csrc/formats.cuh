// Weight formats of the decode-GEMV path and the B200 "stripe tile" layout.
//
// GGUF block formats (byte layouts, reference include/xdna/kquants.h:50-160 and
// include/xdna/q4_0_reference.h:11-35; IQ3_XXS / IQ2_S as gguf 0.19.0
// gguf/quants.py:901-1056) are split, per tile of TILE_ROWS rows, into three
// regions so the GEMV kernel can stream them with 16-byte loads:
//
//   payload : quant bits, in 16-byte pieces ordered [piece][row][unit]  so the
//             32 lanes of a warp, each owning one "unit" of a row, read 512
//             contiguous bytes per load instruction;
//   aux     : per-block sub-scale records (A bytes), ordered [row][block];
//   d       : per-block fp16 super-scales (D bytes), ordered [row][block].
//
// A unit is UNIT_VALS consecutive values of a row (32 for Q4_0, 128 = half a
// super-block otherwise).  The tile occupies exactly rows * row_bytes bytes,
// the same span as the GGUF rows it holds, so the repack is an in-place
// permutation of each tile and tensor offsets/sizes are unchanged.
// Q5_K's qh and Q3_K's hmask bit planes are transposed during the repack into
// per-unit 16-byte pieces (see pack_block); every other byte moves unchanged.
// Scales are kept bit-exact (fp16 / 6-bit / int8), unlike the reference's
// lossy BF16 column prepack (src/xdna-q4-prepack.cpp:564-600).
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define XB_HD __host__ __device__ __forceinline__
#else
#define XB_HD inline
#endif

namespace xb {

// ggml type ids (reference include/xdna/ggml-xdna.h:19-48)
enum : int {
    T_Q4_0 = 2, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14,
    T_IQ3_XXS = 18, T_IQ3_S = 21, T_IQ2_S = 22, T_IQ4_XS = 23,
};

// Rows per stripe tile.  Eight rows make every tile start on a 16-byte
// boundary for all nine formats (8 x an even block size is a multiple of 16),
// which the kernels' 16-byte loads require.
constexpr int TILE_ROWS = 8;

struct FormatInfo {
    int type;
    int block_vals;   // values per GGUF block
    int block_bytes;  // bytes per GGUF block
    int unit_vals;    // values per GEMV unit
    int pieces;       // 16-byte payload pieces per unit
    int a_bytes;      // aux record bytes per block
    int d_bytes;      // d record bytes per block
};

XB_HD FormatInfo format_info(int type) {
    switch (type) {
        //                   type       bv   bb  uv  pc  a   d
        case T_Q4_0:    return {T_Q4_0,    32,  18, 32,  1, 0,  2};
        case T_Q4_K:    return {T_Q4_K,   256, 144, 128, 4, 12, 4};
        case T_Q5_K:    return {T_Q5_K,   256, 176, 128, 5, 12, 4};
        case T_Q3_K:    return {T_Q3_K,   256, 110, 128, 3, 12, 2};
        case T_Q6_K:    return {T_Q6_K,   256, 210, 128, 6, 16, 2};
        case T_IQ4_XS:  return {T_IQ4_XS, 256, 136, 128, 4, 4,  4};
        case T_IQ3_S:   return {T_IQ3_S,  256, 110, 128, 3, 12, 2};
        case T_IQ3_XXS: return {T_IQ3_XXS,256,  98, 128, 3, 0,  2};
        case T_IQ2_S:   return {T_IQ2_S,  256,  82, 128, 2, 16, 2};
        default:        return {0, 0, 0, 0, 0, 0, 0};
    }
}

XB_HD bool type_supported(int type) { return format_info(type).block_vals != 0; }

// Geometry of one weight matrix [N rows x K values].
struct Geometry {
    FormatInfo f;
    int64_t N, K;
    int64_t nb;         // blocks per row
    int64_t nu;         // units per row
    int64_t row_bytes;  // GGUF bytes per row
    int64_t ntiles;
};

XB_HD Geometry make_geometry(int type, int64_t N, int64_t K) {
    Geometry g;
    g.f = format_info(type);
    g.N = N;
    g.K = K;
    g.nb = g.f.block_vals ? K / g.f.block_vals : 0;
    g.nu = g.f.unit_vals ? K / g.f.unit_vals : 0;
    g.row_bytes = g.nb * g.f.block_bytes;
    g.ntiles = (N + TILE_ROWS - 1) / TILE_ROWS;
    return g;
}

// Byte offsets inside a tile holding `tr` rows.
XB_HD int64_t tile_payload_off(const Geometry& g, int tr, int piece, int row, int64_t unit) {
    return ((int64_t(piece) * tr + row) * g.nu + unit) * 16;
}
XB_HD int64_t tile_aux_off(const Geometry& g, int tr, int row, int64_t block) {
    return int64_t(g.f.pieces) * tr * g.nu * 16 + (int64_t(row) * g.nb + block) * g.f.a_bytes;
}
XB_HD int64_t tile_d_off(const Geometry& g, int tr, int row, int64_t block) {
    return int64_t(g.f.pieces) * tr * g.nu * 16 + int64_t(tr) * g.nb * g.f.a_bytes +
           (int64_t(row) * g.nb + block) * g.f.d_bytes;
}

// ---------------------------------------------------------------------------
// Per-block repack.  `blk` is one GGUF block; the unit pieces, aux and d
// records it produces are written through the three output pointers:
//   pieces[u][p] (u < units per block), aux (a_bytes), d (d_bytes).
// unpack_block is the exact inverse.
// ---------------------------------------------------------------------------

// Bit (8*i + k) of word jj of the transposed plane = bit `bit` of src[4*k + i]
// (k: 4-byte word index 0..7 within a 32-byte group, i: byte within word).
XB_HD uint32_t transpose_plane(const uint8_t* src32, int bit) {
    uint32_t w = 0;
    for (int k = 0; k < 8; ++k)
        for (int i = 0; i < 4; ++i)
            w |= uint32_t((src32[4 * k + i] >> bit) & 1u) << (8 * i + k);
    return w;
}

XB_HD void untranspose_plane(uint32_t w, uint8_t* dst32, int bit) {
    for (int k = 0; k < 8; ++k)
        for (int i = 0; i < 4; ++i)
            dst32[4 * k + i] = uint8_t(dst32[4 * k + i] | (((w >> (8 * i + k)) & 1u) << bit));
}

XB_HD void put32(uint8_t* p, uint32_t v) {
    p[0] = uint8_t(v); p[1] = uint8_t(v >> 8); p[2] = uint8_t(v >> 16); p[3] = uint8_t(v >> 24);
}
XB_HD uint32_t get32(const uint8_t* p) {
    return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}
XB_HD void copy_bytes(uint8_t* dst, const uint8_t* src, int n) {
    for (int i = 0; i < n; ++i) dst[i] = src[i];
}

// pieces: array of (units per block) * pieces * 16 bytes, unit-major.
XB_HD void pack_block(int type, const uint8_t* blk, uint8_t* pieces, uint8_t* aux, uint8_t* d) {
    switch (type) {
        case T_Q4_0:  // d(2) qs(16)
            copy_bytes(d, blk, 2);
            copy_bytes(pieces, blk + 2, 16);
            break;
        case T_Q4_K:  // d dmin(4) scales(12) qs(128)
            copy_bytes(d, blk, 4);
            copy_bytes(aux, blk + 4, 12);
            for (int h = 0; h < 2; ++h) copy_bytes(pieces + h * 64, blk + 16 + 64 * h, 64);
            break;
        case T_Q5_K:  // d dmin(4) scales(12) qh(32) qs(128)
            copy_bytes(d, blk, 4);
            copy_bytes(aux, blk + 4, 12);
            for (int h = 0; h < 2; ++h) {
                uint8_t* u = pieces + h * 80;
                copy_bytes(u, blk + 48 + 64 * h, 64);
                for (int jj = 0; jj < 2; ++jj)
                    for (int n = 0; n < 2; ++n)
                        put32(u + 64 + 4 * (2 * jj + n), transpose_plane(blk + 16, 2 * (2 * h + jj) + n));
            }
            break;
        case T_Q3_K:  // hmask(32) qs(64) scales(12) d(2)
            copy_bytes(d, blk + 108, 2);
            copy_bytes(aux, blk + 96, 12);
            for (int h = 0; h < 2; ++h) {
                uint8_t* u = pieces + h * 48;
                copy_bytes(u, blk + 32 + 32 * h, 32);
                for (int j2 = 0; j2 < 4; ++j2) put32(u + 32 + 4 * j2, transpose_plane(blk, 4 * h + j2));
            }
            break;
        case T_Q6_K:  // ql(128) qh(64) scales(16) d(2)
            copy_bytes(d, blk + 208, 2);
            copy_bytes(aux, blk + 192, 16);
            for (int h = 0; h < 2; ++h) {
                uint8_t* u = pieces + h * 96;
                copy_bytes(u, blk + 64 * h, 64);
                copy_bytes(u + 64, blk + 128 + 32 * h, 32);
            }
            break;
        case T_IQ4_XS:  // d(2) scales_h(2) scales_l(4) qs(128)
            copy_bytes(d, blk, 4);
            copy_bytes(aux, blk + 4, 4);
            for (int h = 0; h < 2; ++h) copy_bytes(pieces + h * 64, blk + 8 + 64 * h, 64);
            break;
        case T_IQ3_S:  // d(2) qs(64) qh(8) signs(32) scales(4)
            copy_bytes(d, blk, 2);
            copy_bytes(aux, blk + 66, 8);
            copy_bytes(aux + 8, blk + 106, 4);
            for (int h = 0; h < 2; ++h) {
                uint8_t* u = pieces + h * 48;
                copy_bytes(u, blk + 2 + 32 * h, 32);
                copy_bytes(u + 32, blk + 74 + 16 * h, 16);
            }
            break;
        case T_IQ3_XXS:  // d(2) qs(64) scales_signs(32)
            copy_bytes(d, blk, 2);
            for (int h = 0; h < 2; ++h) {
                uint8_t* u = pieces + h * 48;
                copy_bytes(u, blk + 2 + 32 * h, 32);
                copy_bytes(u + 32, blk + 66 + 16 * h, 16);
            }
            break;
        case T_IQ2_S:  // d(2) qs(32) signs(32) qh(8) scales(8)
            copy_bytes(d, blk, 2);
            copy_bytes(aux, blk + 66, 16);
            for (int h = 0; h < 2; ++h) {
                uint8_t* u = pieces + h * 32;
                copy_bytes(u, blk + 2 + 16 * h, 16);
                copy_bytes(u + 16, blk + 34 + 16 * h, 16);
            }
            break;
        default:
            break;
    }
}

XB_HD void unpack_block(int type, const uint8_t* pieces, const uint8_t* aux, const uint8_t* d, uint8_t* blk) {
    switch (type) {
        case T_Q4_0:
            copy_bytes(blk, d, 2);
            copy_bytes(blk + 2, pieces, 16);
            break;
        case T_Q4_K:
            copy_bytes(blk, d, 4);
            copy_bytes(blk + 4, aux, 12);
            for (int h = 0; h < 2; ++h) copy_bytes(blk + 16 + 64 * h, pieces + h * 64, 64);
            break;
        case T_Q5_K:
            copy_bytes(blk, d, 4);
            copy_bytes(blk + 4, aux, 12);
            for (int i = 0; i < 32; ++i) blk[16 + i] = 0;
            for (int h = 0; h < 2; ++h) {
                const uint8_t* u = pieces + h * 80;
                copy_bytes(blk + 48 + 64 * h, u, 64);
                for (int jj = 0; jj < 2; ++jj)
                    for (int n = 0; n < 2; ++n)
                        untranspose_plane(get32(u + 64 + 4 * (2 * jj + n)), blk + 16, 2 * (2 * h + jj) + n);
            }
            break;
        case T_Q3_K:
            copy_bytes(blk + 108, d, 2);
            copy_bytes(blk + 96, aux, 12);
            for (int i = 0; i < 32; ++i) blk[i] = 0;
            for (int h = 0; h < 2; ++h) {
                const uint8_t* u = pieces + h * 48;
                copy_bytes(blk + 32 + 32 * h, u, 32);
                for (int j2 = 0; j2 < 4; ++j2) untranspose_plane(get32(u + 32 + 4 * j2), blk, 4 * h + j2);
            }
            break;
        case T_Q6_K:
            copy_bytes(blk + 208, d, 2);
            copy_bytes(blk + 192, aux, 16);
            for (int h = 0; h < 2; ++h) {
                const uint8_t* u = pieces + h * 96;
                copy_bytes(blk + 64 * h, u, 64);
                copy_bytes(blk + 128 + 32 * h, u + 64, 32);
            }
            break;
        case T_IQ4_XS:
            copy_bytes(blk, d, 4);
            copy_bytes(blk + 4, aux, 4);
            for (int h = 0; h < 2; ++h) copy_bytes(blk + 8 + 64 * h, pieces + h * 64, 64);
            break;
        case T_IQ3_S:
            copy_bytes(blk, d, 2);
            copy_bytes(blk + 66, aux, 8);
            copy_bytes(blk + 106, aux + 8, 4);
            for (int h = 0; h < 2; ++h) {
                const uint8_t* u = pieces + h * 48;
                copy_bytes(blk + 2 + 32 * h, u, 32);
                copy_bytes(blk + 74 + 16 * h, u + 32, 16);
            }
            break;
        case T_IQ3_XXS:
            copy_bytes(blk, d, 2);
            for (int h = 0; h < 2; ++h) {
                const uint8_t* u = pieces + h * 48;
                copy_bytes(blk + 2 + 32 * h, u, 32);
                copy_bytes(blk + 66 + 16 * h, u + 32, 16);
            }
            break;
        case T_IQ2_S:
            copy_bytes(blk, d, 2);
            copy_bytes(blk + 66, aux, 16);
            for (int h = 0; h < 2; ++h) {
                const uint8_t* u = pieces + h * 32;
                copy_bytes(blk + 2 + 16 * h, u, 16);
                copy_bytes(blk + 34 + 16 * h, u + 16, 16);
            }
            break;
        default:
            break;
    }
}

// Repack (or unpack) one block (row r of a tile with tr rows, block b) between
// a GGUF tile `raw` and a stripe tile `tile`.  Both point at the tile start.
XB_HD void repack_one(const Geometry& g, int tr, int r, int64_t b, const uint8_t* raw, uint8_t* tile) {
    const FormatInfo& f = g.f;
    uint8_t pieces[2 * 6 * 16];
    uint8_t aux[16];
    uint8_t d[4];
    pack_block(f.type, raw + r * g.row_bytes + b * f.block_bytes, pieces, aux, d);
    const int upb = f.block_vals / f.unit_vals;
    for (int uu = 0; uu < upb; ++uu)
        for (int p = 0; p < f.pieces; ++p)
            copy_bytes(tile + tile_payload_off(g, tr, p, r, b * upb + uu), pieces + (uu * f.pieces + p) * 16, 16);
    if (f.a_bytes) copy_bytes(tile + tile_aux_off(g, tr, r, b), aux, f.a_bytes);
    copy_bytes(tile + tile_d_off(g, tr, r, b), d, f.d_bytes);
}

XB_HD void unrepack_one(const Geometry& g, int tr, int r, int64_t b, const uint8_t* tile, uint8_t* raw) {
    const FormatInfo& f = g.f;
    uint8_t pieces[2 * 6 * 16];
    uint8_t aux[16] = {0};
    uint8_t d[4];
    const int upb = f.block_vals / f.unit_vals;
    for (int uu = 0; uu < upb; ++uu)
        for (int p = 0; p < f.pieces; ++p)
            copy_bytes(pieces + (uu * f.pieces + p) * 16, tile + tile_payload_off(g, tr, p, r, b * upb + uu), 16);
    if (f.a_bytes) copy_bytes(aux, tile + tile_aux_off(g, tr, r, b), f.a_bytes);
    copy_bytes(d, tile + tile_d_off(g, tr, r, b), f.d_bytes);
    unpack_block(f.type, pieces, aux, d, raw + r * g.row_bytes + b * f.block_bytes);
}

// ---------------------------------------------------------------------------
// MMA layout (Q4_0 and Q4_K when N % 16 == 0 and K % 256 == 0).
//
// The integer tensor-core GEMV (gemv_mma.cu) computes 16 rows x 256 values
// ("a group": eight 32-value blocks) with mma.m16n8k32: the weights are the
// u8 A operand, x is three signed-byte digit planes in a block-diagonal B
// operand whose column n holds block n, so each C column is one block's dot
// product.  A tile holds 16 rows; a group of a tile is 2304 bytes (16 rows x
// 144 / 16 rows x 8 blocks x 18), laid out as
//   A   : [4 chunk pairs][32 lanes][16 B]: lane (g = lane / 4, t = lane % 4)
//         holds, for chunks c = 2i, 2i + 1, two words: word 0 = block t,
//         word 1 = block t + 4; byte j of a word = value 4c + j of that block
//         with row g in the low nibble and row g + 8 in the high nibble
//         (exactly the m16n8k32 A fragment after one mask / shift);
//   hdr : 256 B.  Q4_K: the 16 rows' 16-byte headers {d, dmin, scales[12]}.
//         Q4_0: [g][t][4 x fp16] = d(g, 2t), d(g, 2t+1), d(g+8, 2t), d(g+8, 2t+1)
//         (the blocks whose C columns lane (g, t) owns).
// ---------------------------------------------------------------------------
constexpr int MMA_TILE_ROWS = 16;
constexpr int MMA_MAX_SEGMENTS = 4;  // matrices sharing x in one MMA GEMV launch
constexpr int MMA_GROUP_BYTES = 2304;  // Q4_0 / Q4_K group (16 rows x 144 B)

// Q5_K adds a 512-byte high-bit plane between the nibbles and the header:
//   [0, 2048)    nibbles, as Q4_K;
//   [2048, 2560) per lane 16 B, word i for chunks 2i and 2i+1: bit 8j + 4 + k
//                (chunk 2i) or 8j + k (chunk 2i+1) is the fifth bit of value j
//                of A register k (a0 row g / a1 row g+8 of block t, a2 / a3 of
//                block t+4), so one shift and one mask put it at bit 4;
//   [2560, 2816) the 16 rows' 16-byte headers, as Q4_K.
//
// Q6_K (16-value sub-blocks with int8 scales; 6-bit q) uses 16-value B
// blocks: chunk cc (0..7) covers values 4 (cc % 4) .. +3 of the 16-value
// blocks 8 (cc / 4) + column, so chunks 0-3 and 4-7 are two sets of 8 blocks.
//   [0, 2048)    low nibbles, swizzled as Q4_K (column t / t+4 of each chunk);
//   [2048, 3072) per lane 32 B: word cc holds the high two bits of value j of
//                A register k at bits 8j + 2k, 8j + 2k + 1;
//   [3072, 3328) per lane 8 int8 scales: rows g, g+8 (4 bytes each) x sets 0, 1
//                (2 bytes each) x blocks 2t, 2t+1 of the set;
//   [3328, 3360) the 16 rows' fp16 d.
//
// Q3_K (3-bit q = low pair + 4 * high bit, 6-bit scales per 16 values) uses the
// same 16-value chunk order as Q6_K:
//   [0, 1024)    per lane 32 B: word c holds the low pair of value j of A
//                register k at bits 8j + 2k, 8j + 2k + 1;
//   [1024, 1536) per lane 16 B: word i holds the high bit of value j of
//                register k of chunk 2i (bit 8j + k) and 2i + 1 (bit 8j + 4 + k);
//   [1536, 1664) per lane 4 B: low nibbles of its 8 scales, [1664, 1728) per
//                lane 2 B: their high pairs (scale order as Q6_K's int8 scales);
//   [1728, 1760) the 16 rows' fp16 d.
//
// IQ4_XS (4-bit indices into the 16 IQ4_NL values, 6-bit scales per 32):
//   [0, 2048)    per lane and chunk pair 16 B; word 2 (c % 2) holds the codes
//                of A registers a0 (bits 0-15) and a1 (bits 16-31) of chunk c,
//                word 2 (c % 2) + 1 those of a2 / a3, one 4-bit code per value
//                in value order (byte_perm selector form).  code = the index
//                with bits 2 and 3 swapped (iq4_code), which pairs codes i and
//                i + 8 on values of one sign for the two-table decode;
//   [2048, 2176) the 16 rows' first 8 block bytes {d, scales_h, scales_l[4]}.
//
// IQ3_S (9-bit indices into the 512-entry grid, one per 4 values, a sign bit
// per value, 4-bit scales per 32): A register k of chunk c is grid entry
// 8 (block) + c of its row, so each register is one lookup:
//   [0, 1024)    per lane 32 B: word c, byte k = the entry's low 8 index bits;
//   [1024, 1536) per lane 16 B: word c / 2, bits 16 (c % 2) + 4 k .. + 3 = the
//                register's 4 sign bits, in value order;
//   [1536, 1664) per lane 4 B: bit 4 c + k = the entry's index bit 8;
//   [1664, 1696) the 16 rows' fp16 d;  [1696, 1760) the 16 rows' scales[4].
//
// IQ3_XXS (8-bit indices into the 256-entry grid, one per 4 values; per 8
// values a 7-bit sign index whose 8th sign makes the count even; 4-bit scales
// per 32): register k of chunk c is grid entry 8 (block) + c:
//   [0, 1024)    per lane 32 B: word c, byte k = the entry's grid index;
//   [1024, 1536) per lane 16 B: word p (chunk pair 2p, 2p + 1), bits 7 k .. + 6
//                = the pair's 7-bit sign index for register k; bits 28-31 = the
//                scale of (row g + 8 (p % 2), block 2t + p / 2);
//   [1536, 1568) the 16 rows' fp16 d.
//
// IQ2_S (10-bit indices into the 1024-entry grid, one per 8 values; a sign
// bit per value; 4-bit scales per 16): 16-value x blocks as Q6_K; chunks 2q
// and 2q + 1 of register k share one grid entry (low and high 4 values):
//   [0, 512)     per lane 16 B: byte 4 q + k = the entry's low index byte;
//   [512, 1024)  per lane 16 B: byte 4 q + k = the entry's 8 sign bits;
//   [1024, 1152) per lane 4 B: bits 2 (4 q + k) .. + 1 = the index bits 8-9;
//   [1152, 1280) per lane 4 B: nibble 4 st + 2 h + b = the scale of row g + 8 h,
//                16-value block 8 st + 2 t + b;
//   [1280, 1312) the 16 rows' fp16 d.
XB_HD int mma_group_bytes(int type) {
    switch (type) {
        case T_Q5_K: return 2816;
        case T_Q6_K: return 3360;
        case T_Q3_K:
        case T_IQ3_S: return 1760;
        case T_IQ4_XS: return 2176;
        case T_IQ3_XXS: return 1568;
        case T_IQ2_S: return 1312;
        default: return MMA_GROUP_BYTES;
    }
}
XB_HD int mma_header_off(int type) { return type == T_Q5_K ? 2560 : (type == T_Q6_K ? 3072 : 2048); }
// GGUF bytes of one row's 256-value group (8 Q4_0 blocks or one K super-block)
XB_HD int mma_row_group_bytes(int type) { return mma_group_bytes(type) / MMA_TILE_ROWS; }
// x blocks (B columns) of 16 values instead of 32
XB_HD bool mma_blk16(int type) { return type == T_Q6_K || type == T_Q3_K || type == T_IQ2_S; }

XB_HD int layout_kind(int type, int64_t N, int64_t K) {
    return ((type == T_Q4_0 || type == T_Q4_K || type == T_Q5_K || type == T_Q6_K || type == T_Q3_K ||
             type == T_IQ4_XS || type == T_IQ3_S || type == T_IQ3_XXS || type == T_IQ2_S) &&
            N > 0 && K > 0 && N % MMA_TILE_ROWS == 0 && K % 256 == 0)
               ? 1
               : 0;
}

// IQ4_XS layout code of an index (an involution: also the index of a code)
XB_HD uint32_t iq4_code(uint32_t q) { return (q & 3u) | (((q >> 3) & 1u) << 2) | (((q >> 2) & 1u) << 3); }
// IQ4_XS index of value v: qs[16 ib + j % 16] nibble j / 16 of sub-block ib = v / 32
XB_HD const uint8_t* iq4_idx(const uint8_t* row, int64_t gi, int v, int* shift) {
    const int ib = v >> 5, j = v & 31;
    *shift = 4 * (j >> 4);
    return row + gi * 136 + 8 + 16 * ib + (j & 15);
}

// Q3_K: low pair / high bit of value v, and the 6-bit scale i of a row's group
XB_HD const uint8_t* q3_lo(const uint8_t* row, int64_t gi, int v, int* shift) {
    const int n = v >> 7, j = (v >> 5) & 3, half = (v >> 4) & 1, l = v & 15;
    *shift = 2 * j;
    return row + gi * 110 + 32 + 32 * n + 16 * half + l;
}
XB_HD const uint8_t* q3_hi(const uint8_t* row, int64_t gi, int v, int* bit) {
    const int n = v >> 7, j = (v >> 5) & 3, half = (v >> 4) & 1, l = v & 15;
    *bit = 4 * n + j;
    return row + gi * 110 + 16 * half + l;
}
XB_HD uint32_t q3_scale(const uint8_t* row, int64_t gi, int i) {
    const uint8_t* s12 = row + gi * 110 + 96;
    const int q = i >> 2, r = i & 3;
    const uint32_t lo = (s12[4 * (q & 1) + r] >> (4 * (q >> 1))) & 0xFu;
    const uint32_t hi = (s12[8 + r] >> (2 * q)) & 3u;
    return lo | (hi << 4);
}
XB_HD void q3_set_scale(uint8_t* row, int64_t gi, int i, uint32_t v) {
    uint8_t* s12 = row + gi * 110 + 96;
    const int q = i >> 2, r = i & 3;
    uint8_t* pl = s12 + 4 * (q & 1) + r;
    const int sl = 4 * (q >> 1);
    *pl = uint8_t((*pl & ~(0xFu << sl)) | ((v & 0xFu) << sl));
    uint8_t* ph = s12 + 8 + r;
    *ph = uint8_t((*ph & ~(3u << (2 * q))) | (((v >> 4) & 3u) << (2 * q)));
}

// value index (0..255) of lane (g, t)'s A register `kind` (0: column t,
// 1: column t + 4), chunk c, byte j
XB_HD int mma_value(int type, int c, int t, int kind, int j) {
    if (mma_blk16(type)) return 16 * (8 * (c >> 2) + t + 4 * kind) + 4 * (c & 3) + j;
    return 32 * (t + 4 * kind) + 4 * c + j;
}
// Q6_K: low nibble byte / shift and high-pair byte / shift of value v
XB_HD const uint8_t* q6_lo(const uint8_t* row, int64_t gi, int v, int* shift) {
    const int n = v >> 7, qd = (v >> 5) & 3, l = v & 31;
    *shift = 4 * (qd >> 1);
    return row + gi * 210 + 64 * n + l + 32 * (qd & 1);
}
XB_HD const uint8_t* q6_hi(const uint8_t* row, int64_t gi, int v, int* shift) {
    const int n = v >> 7, qd = (v >> 5) & 3, l = v & 31;
    *shift = 2 * qd;
    return row + gi * 210 + 128 + 32 * n + l;
}

// Byte and bit of the low 4 bits of value v (0..255) in a row's group gi:
// Q4_K / Q5_K super-blocks keep 64-value pairs of sub-blocks in 32 bytes (low
// nibbles = sub-block 2i, high = 2i+1); Q4_0 blocks keep value o (high nibble
// for o >= 16) in byte o % 16 after the 2-byte scale.
XB_HD const uint8_t* q4_byte(int type, const uint8_t* row, int64_t gi, int v, int* shift) {
    if (type == T_Q6_K) return q6_lo(row, gi, v, shift);
    if (type == T_Q4_0) {
        const int o = v & 31;
        *shift = 4 * (o >> 4);
        return row + (gi * 8 + (v >> 5)) * 18 + 2 + (o & 15);
    }
    const int qs = type == T_Q5_K ? 48 : 16;
    *shift = 4 * ((v >> 5) & 1);
    return row + gi * mma_row_group_bytes(type) + qs + 32 * (v >> 6) + (v & 31);
}
XB_HD uint32_t q4_of(int type, const uint8_t* row, int64_t gi, int v) {
    int sh;
    const uint8_t* p = q4_byte(type, row, gi, v, &sh);
    return (*p >> sh) & 0xFu;
}
// Q5_K fifth bit of value v: qh[v % 32] bit 2 * (v / 64) + (v / 32) % 2
XB_HD const uint8_t* q5_hbyte(const uint8_t* row, int64_t gi, int v, int* bit) {
    *bit = 2 * (v >> 6) + ((v >> 5) & 1);
    return row + gi * 176 + 16 + (v & 31);
}
// bit of Q5_K high-plane word (chunk c, A register k, value j)
XB_HD int q5_plane_bit(int c, int k, int j) { return 8 * j + ((c & 1) ? 0 : 4) + k; }

// One group (gi) of one 16-row tile: GGUF rows (tile row 0 at `raw`, stride
// row_bytes) -> MMA layout at `out` (2304 bytes), or the inverse.
// IQ3_S grid entry e (0..63) of a row's group gi: the low index byte, the
// index bit 8 and the 4 sign bits of its values (block bytes: d, qs[64],
// qh[8], signs[32], scales[4])
XB_HD uint8_t* iq3s_qs(uint8_t* row, int64_t gi, int e) { return row + gi * 110 + 2 + e; }
XB_HD uint8_t* iq3s_qh(uint8_t* row, int64_t gi, int e) { return row + gi * 110 + 66 + (e >> 3); }
XB_HD uint8_t* iq3s_sg(uint8_t* row, int64_t gi, int e) { return row + gi * 110 + 74 + (e >> 1); }

// IQ3_XXS block bytes: d, qs[64], then 8 words (4 x 7-bit sign index | scale << 28)
XB_HD uint8_t* iq3xxs_word(uint8_t* row, int64_t gi, int blk) { return row + gi * 98 + 66 + 4 * blk; }
// IQ2_S block bytes: d, qs[32], signs[32], qh[8], scales[8]; entry e covers values 8e .. 8e + 7
XB_HD uint8_t* iq2s_at(uint8_t* row, int64_t gi, int off) { return row + gi * 82 + off; }

XB_HD void mma_pack_group(int type, const uint8_t* raw, int64_t row_bytes, int64_t gi, uint8_t* out) {
    uint8_t* rw = const_cast<uint8_t*>(raw);
    if (type == T_IQ3_XXS) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int c = 0; c < 8; ++c)
                for (int k = 0; k < 4; ++k)
                    out[lane * 32 + 4 * c + k] =
                        *(rw + (g + 8 * (k & 1)) * row_bytes + gi * 98 + 2 + 8 * (t + 4 * (k >> 1)) + c);
            for (int p = 0; p < 4; ++p) {
                uint32_t w = 0;
                for (int k = 0; k < 4; ++k) {
                    const uint32_t aux = get32(iq3xxs_word(rw + (g + 8 * (k & 1)) * row_bytes, gi, t + 4 * (k >> 1)));
                    w |= ((aux >> (7 * p)) & 127u) << (7 * k);
                }
                const uint32_t aux = get32(iq3xxs_word(rw + (g + 8 * (p & 1)) * row_bytes, gi, 2 * t + (p >> 1)));
                w |= aux & 0xF0000000u;
                put32(out + 1024 + lane * 16 + 4 * p, w);
            }
        }
        for (int r = 0; r < 16; ++r) copy_bytes(out + 1536 + 2 * r, raw + r * row_bytes + gi * 98, 2);
        return;
    }
    if (type == T_IQ2_S) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            uint32_t hw = 0, sw = 0;
            for (int q = 0; q < 4; ++q)
                for (int k = 0; k < 4; ++k) {
                    uint8_t* row = rw + (g + 8 * (k & 1)) * row_bytes;
                    const int e = 2 * (8 * (q >> 1) + t + 4 * (k >> 1)) + (q & 1);
                    out[lane * 16 + 4 * q + k] = *iq2s_at(row, gi, 2 + e);
                    out[512 + lane * 16 + 4 * q + k] = *iq2s_at(row, gi, 34 + e);
                    hw |= ((static_cast<uint32_t>(*iq2s_at(row, gi, 66 + (e >> 2))) >> (2 * (e & 3))) & 3u)
                          << (2 * (4 * q + k));
                }
            for (int st = 0; st < 2; ++st)
                for (int h = 0; h < 2; ++h)
                    for (int b = 0; b < 2; ++b) {
                        const int B = 8 * st + 2 * t + b;
                        const uint32_t sc = *iq2s_at(rw + (g + 8 * h) * row_bytes, gi, 74 + (B >> 1));
                        sw |= ((sc >> (4 * (B & 1))) & 0xFu) << (4 * (4 * st + 2 * h + b));
                    }
            put32(out + 1024 + lane * 4, hw);
            put32(out + 1152 + lane * 4, sw);
        }
        for (int r = 0; r < 16; ++r) copy_bytes(out + 1280 + 2 * r, raw + r * row_bytes + gi * 82, 2);
        return;
    }
    if (type == T_IQ3_S) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            uint32_t hw = 0;
            uint32_t sw[4] = {0, 0, 0, 0};
            for (int c = 0; c < 8; ++c)
                for (int k = 0; k < 4; ++k) {
                    uint8_t* row = const_cast<uint8_t*>(raw) + (g + 8 * (k & 1)) * row_bytes;
                    const int e = 8 * (t + 4 * (k >> 1)) + c;
                    out[lane * 32 + 4 * c + k] = *iq3s_qs(row, gi, e);
                    hw |= static_cast<uint32_t>((*iq3s_qh(row, gi, e) >> (e & 7)) & 1u) << (4 * c + k);
                    sw[c >> 1] |= static_cast<uint32_t>((*iq3s_sg(row, gi, e) >> (4 * (e & 1))) & 0xFu)
                                  << (16 * (c & 1) + 4 * k);
                }
            for (int i = 0; i < 4; ++i) put32(out + 1024 + lane * 16 + 4 * i, sw[i]);
            put32(out + 1536 + lane * 4, hw);
        }
        for (int r = 0; r < 16; ++r) {
            copy_bytes(out + 1664 + 2 * r, raw + r * row_bytes + gi * 110, 2);
            copy_bytes(out + 1696 + 4 * r, raw + r * row_bytes + gi * 110 + 106, 4);
        }
        return;
    }
    if (type == T_IQ4_XS) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int c = 0; c < 8; ++c)
                for (int half = 0; half < 2; ++half) {  // word: registers (a0, a1) or (a2, a3)
                    uint32_t w = 0;
                    for (int k2 = 0; k2 < 2; ++k2) {
                        const int k = 2 * half + k2;  // a0 row g / a1 row g+8 of column t, a2 / a3 of t + 4
                        const uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                        for (int j = 0; j < 4; ++j) {
                            int sh;
                            const uint8_t* p = iq4_idx(row, gi, mma_value(type, c, t, k >> 1, j), &sh);
                            w |= iq4_code((*p >> sh) & 0xFu) << (16 * k2 + 4 * j);
                        }
                    }
                    put32(out + ((c >> 1) * 32 + lane) * 16 + 8 * (c & 1) + 4 * half, w);
                }
        }
        for (int r = 0; r < 16; ++r) copy_bytes(out + 2048 + 8 * r, raw + r * row_bytes + gi * 136, 8);
        return;
    }
    if (type == T_Q3_K) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int c = 0; c < 8; ++c) {
                uint32_t lw = 0;
                for (int k = 0; k < 4; ++k) {
                    const uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                    for (int j = 0; j < 4; ++j) {
                        int sh;
                        const uint8_t* lb = q3_lo(row, gi, mma_value(type, c, t, k >> 1, j), &sh);
                        lw |= static_cast<uint32_t>((*lb >> sh) & 3u) << (8 * j + 2 * k);
                    }
                }
                put32(out + lane * 32 + 4 * c, lw);
            }
            for (int i = 0; i < 4; ++i) {
                uint32_t hw = 0;
                for (int c = 2 * i; c < 2 * i + 2; ++c)
                    for (int k = 0; k < 4; ++k) {
                        const uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                        for (int j = 0; j < 4; ++j) {
                            int bit;
                            const uint8_t* hb = q3_hi(row, gi, mma_value(type, c, t, k >> 1, j), &bit);
                            hw |= static_cast<uint32_t>((*hb >> bit) & 1u) << (8 * j + 4 * (c & 1) + k);
                        }
                    }
                put32(out + 1024 + lane * 16 + 4 * i, hw);
            }
            uint32_t lo = 0, hi = 0;
            for (int i = 0; i < 8; ++i) {  // i = 4 h + 2 set + b
                const int h = i >> 2, st = (i >> 1) & 1, b = i & 1;
                const uint32_t sc = q3_scale(raw + (g + 8 * h) * row_bytes, gi, 8 * st + 2 * t + b);
                lo |= (sc & 0xFu) << (4 * i);
                hi |= ((sc >> 4) & 3u) << (2 * i);
            }
            put32(out + 1536 + 4 * lane, lo);
            out[1664 + 2 * lane] = uint8_t(hi & 0xFFu);
            out[1664 + 2 * lane + 1] = uint8_t(hi >> 8);
        }
        for (int r = 0; r < 16; ++r) copy_bytes(out + 1728 + 2 * r, raw + r * row_bytes + gi * 110 + 108, 2);
        return;
    }
    for (int lane = 0; lane < 32; ++lane) {
        const int g = lane >> 2, t = lane & 3;
        const uint8_t* r0 = raw + g * row_bytes;
        const uint8_t* r8 = raw + (g + 8) * row_bytes;
        for (int c = 0; c < 8; ++c)
            for (int kind = 0; kind < 2; ++kind) {
                uint32_t w = 0;
                for (int j = 0; j < 4; ++j) {
                    const int v = mma_value(type, c, t, kind, j);
                    w |= (q4_of(type, r0, gi, v) | (q4_of(type, r8, gi, v) << 4)) << (8 * j);
                }
                put32(out + ((c >> 1) * 32 + lane) * 16 + 8 * (c & 1) + 4 * kind, w);
            }
    }
    if (type == T_Q6_K) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int c = 0; c < 8; ++c) {
                uint32_t w = 0;
                for (int k = 0; k < 4; ++k) {
                    const uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                    for (int j = 0; j < 4; ++j) {
                        int sh;
                        const uint8_t* hb = q6_hi(row, gi, mma_value(type, c, t, k >> 1, j), &sh);
                        w |= static_cast<uint32_t>((*hb >> sh) & 3u) << (8 * j + 2 * k);
                    }
                }
                put32(out + 2048 + lane * 32 + 4 * c, w);
            }
            for (int h = 0; h < 2; ++h)
                for (int st = 0; st < 2; ++st)
                    for (int b = 0; b < 2; ++b)
                        out[3072 + lane * 8 + 4 * h + 2 * st + b] =
                            raw[(g + 8 * h) * row_bytes + gi * 210 + 192 + 8 * st + 2 * t + b];
        }
        for (int r = 0; r < 16; ++r) copy_bytes(out + 3328 + 2 * r, raw + r * row_bytes + gi * 210 + 208, 2);
        return;
    }
    if (type == T_Q5_K) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int i = 0; i < 4; ++i) {
                uint32_t w = 0;
                for (int c = 2 * i; c < 2 * i + 2; ++c)
                    for (int k = 0; k < 4; ++k) {
                        const uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                        const int blk = t + 4 * (k >> 1);
                        for (int j = 0; j < 4; ++j) {
                            int bit;
                            const uint8_t* hb = q5_hbyte(row, gi, 32 * blk + 4 * c + j, &bit);
                            w |= static_cast<uint32_t>((*hb >> bit) & 1u) << q5_plane_bit(c, k, j);
                        }
                    }
                put32(out + 2048 + lane * 16 + 4 * i, w);
            }
        }
    }
    uint8_t* hdr = out + mma_header_off(type);
    if (type == T_Q4_K || type == T_Q5_K) {
        for (int r = 0; r < 16; ++r)
            copy_bytes(hdr + 16 * r, raw + r * row_bytes + gi * mma_row_group_bytes(type), 16);
    } else {
        for (int g = 0; g < 8; ++g)
            for (int t = 0; t < 4; ++t)
                for (int h = 0; h < 4; ++h) {
                    const int row = g + 8 * (h >> 1), blk = 2 * t + (h & 1);
                    copy_bytes(hdr + ((g * 4 + t) * 4 + h) * 2, raw + row * row_bytes + (gi * 8 + blk) * 18, 2);
                }
    }
}

XB_HD void mma_unpack_group(int type, const uint8_t* in, int64_t row_bytes, int64_t gi, uint8_t* raw) {
    if (type == T_IQ3_XXS) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int c = 0; c < 8; ++c)
                for (int k = 0; k < 4; ++k)
                    *(raw + (g + 8 * (k & 1)) * row_bytes + gi * 98 + 2 + 8 * (t + 4 * (k >> 1)) + c) =
                        in[lane * 32 + 4 * c + k];
            for (int p = 0; p < 4; ++p) {
                const uint32_t w = get32(in + 1024 + lane * 16 + 4 * p);
                for (int k = 0; k < 4; ++k) {
                    uint8_t* a = iq3xxs_word(raw + (g + 8 * (k & 1)) * row_bytes, gi, t + 4 * (k >> 1));
                    const uint32_t m = 127u << (7 * p);
                    put32(a, (get32(a) & ~m) | (((w >> (7 * k)) & 127u) << (7 * p)));
                }
                uint8_t* a = iq3xxs_word(raw + (g + 8 * (p & 1)) * row_bytes, gi, 2 * t + (p >> 1));
                put32(a, (get32(a) & 0x0FFFFFFFu) | (w & 0xF0000000u));
            }
        }
        for (int r = 0; r < 16; ++r) copy_bytes(raw + r * row_bytes + gi * 98, in + 1536 + 2 * r, 2);
        return;
    }
    if (type == T_IQ2_S) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            const uint32_t hw = get32(in + 1024 + lane * 4), sw = get32(in + 1152 + lane * 4);
            for (int q = 0; q < 4; ++q)
                for (int k = 0; k < 4; ++k) {
                    uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                    const int e = 2 * (8 * (q >> 1) + t + 4 * (k >> 1)) + (q & 1);
                    *iq2s_at(row, gi, 2 + e) = in[lane * 16 + 4 * q + k];
                    *iq2s_at(row, gi, 34 + e) = in[512 + lane * 16 + 4 * q + k];
                    uint8_t* h = iq2s_at(row, gi, 66 + (e >> 2));
                    const int sh = 2 * (e & 3);
                    *h = uint8_t((*h & ~(3u << sh)) | (((hw >> (2 * (4 * q + k))) & 3u) << sh));
                }
            for (int st = 0; st < 2; ++st)
                for (int h = 0; h < 2; ++h)
                    for (int b = 0; b < 2; ++b) {
                        const int B = 8 * st + 2 * t + b;
                        uint8_t* sc = iq2s_at(raw + (g + 8 * h) * row_bytes, gi, 74 + (B >> 1));
                        const int sh = 4 * (B & 1);
                        *sc = uint8_t((*sc & ~(0xFu << sh)) | (((sw >> (4 * (4 * st + 2 * h + b))) & 0xFu) << sh));
                    }
        }
        for (int r = 0; r < 16; ++r) copy_bytes(raw + r * row_bytes + gi * 82, in + 1280 + 2 * r, 2);
        return;
    }
    if (type == T_IQ3_S) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            const uint32_t hw = get32(in + 1536 + lane * 4);
            for (int c = 0; c < 8; ++c) {
                const uint32_t sw = get32(in + 1024 + lane * 16 + 4 * (c >> 1));
                for (int k = 0; k < 4; ++k) {
                    uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                    const int e = 8 * (t + 4 * (k >> 1)) + c;
                    *iq3s_qs(row, gi, e) = in[lane * 32 + 4 * c + k];
                    uint8_t* h = iq3s_qh(row, gi, e);
                    *h = uint8_t((*h & ~(1u << (e & 7))) | (((hw >> (4 * c + k)) & 1u) << (e & 7)));
                    uint8_t* sg = iq3s_sg(row, gi, e);
                    const int sh = 4 * (e & 1);
                    *sg = uint8_t((*sg & ~(0xFu << sh)) | (((sw >> (16 * (c & 1) + 4 * k)) & 0xFu) << sh));
                }
            }
        }
        for (int r = 0; r < 16; ++r) {
            copy_bytes(raw + r * row_bytes + gi * 110, in + 1664 + 2 * r, 2);
            copy_bytes(raw + r * row_bytes + gi * 110 + 106, in + 1696 + 4 * r, 4);
        }
        return;
    }
    if (type == T_IQ4_XS) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int c = 0; c < 8; ++c)
                for (int half = 0; half < 2; ++half) {
                    const uint32_t w = get32(in + ((c >> 1) * 32 + lane) * 16 + 8 * (c & 1) + 4 * half);
                    for (int k2 = 0; k2 < 2; ++k2) {
                        const int k = 2 * half + k2;
                        uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                        for (int j = 0; j < 4; ++j) {
                            int sh;
                            uint8_t* p = const_cast<uint8_t*>(iq4_idx(row, gi, mma_value(type, c, t, k >> 1, j), &sh));
                            const uint32_t q = iq4_code((w >> (16 * k2 + 4 * j)) & 0xFu);
                            *p = uint8_t((*p & ~(0xFu << sh)) | (q << sh));
                        }
                    }
                }
        }
        for (int r = 0; r < 16; ++r) copy_bytes(raw + r * row_bytes + gi * 136, in + 2048 + 8 * r, 8);
        return;
    }
    if (type == T_Q3_K) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int c = 0; c < 8; ++c) {
                const uint32_t lw = get32(in + lane * 32 + 4 * c);
                const uint32_t hw = get32(in + 1024 + lane * 16 + 4 * (c >> 1));
                for (int k = 0; k < 4; ++k) {
                    uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                    for (int j = 0; j < 4; ++j) {
                        const int v = mma_value(type, c, t, k >> 1, j);
                        int sh, bit;
                        uint8_t* lb = const_cast<uint8_t*>(q3_lo(row, gi, v, &sh));
                        *lb = uint8_t((*lb & ~(3u << sh)) | (((lw >> (8 * j + 2 * k)) & 3u) << sh));
                        uint8_t* hb = const_cast<uint8_t*>(q3_hi(row, gi, v, &bit));
                        const uint32_t hv = (hw >> (8 * j + 4 * (c & 1) + k)) & 1u;
                        *hb = uint8_t((*hb & ~(1u << bit)) | (hv << bit));
                    }
                }
            }
            const uint32_t lo = get32(in + 1536 + 4 * lane);
            const uint32_t hi = in[1664 + 2 * lane] | (uint32_t(in[1664 + 2 * lane + 1]) << 8);
            for (int i = 0; i < 8; ++i) {
                const int h = i >> 2, st = (i >> 1) & 1, b = i & 1;
                q3_set_scale(raw + (g + 8 * h) * row_bytes, gi, 8 * st + 2 * t + b,
                             ((lo >> (4 * i)) & 0xFu) | (((hi >> (2 * i)) & 3u) << 4));
            }
        }
        for (int r = 0; r < 16; ++r) copy_bytes(raw + r * row_bytes + gi * 110 + 108, in + 1728 + 2 * r, 2);
        return;
    }
    const uint8_t* hdr = in + mma_header_off(type);
    if (type == T_Q6_K) {
        for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            for (int h = 0; h < 2; ++h)
                for (int st = 0; st < 2; ++st)
                    for (int b = 0; b < 2; ++b)
                        raw[(g + 8 * h) * row_bytes + gi * 210 + 192 + 8 * st + 2 * t + b] =
                            in[3072 + lane * 8 + 4 * h + 2 * st + b];
            for (int c = 0; c < 8; ++c) {
                const uint32_t w = get32(in + 2048 + lane * 32 + 4 * c);
                for (int k = 0; k < 4; ++k) {
                    uint8_t* row = raw + (g + 8 * (k & 1)) * row_bytes;
                    for (int j = 0; j < 4; ++j) {
                        int sh;
                        uint8_t* hb = const_cast<uint8_t*>(q6_hi(row, gi, mma_value(type, c, t, k >> 1, j), &sh));
                        const uint32_t hv = (w >> (8 * j + 2 * k)) & 3u;
                        *hb = uint8_t((*hb & ~(3u << sh)) | (hv << sh));
                    }
                }
            }
        }
        for (int r = 0; r < 16; ++r) copy_bytes(raw + r * row_bytes + gi * 210 + 208, in + 3328 + 2 * r, 2);
    } else if (type == T_Q4_K || type == T_Q5_K) {
        for (int r = 0; r < 16; ++r)
            copy_bytes(raw + r * row_bytes + gi * mma_row_group_bytes(type), hdr + 16 * r, 16);
    } else {
        for (int g = 0; g < 8; ++g)
            for (int t = 0; t < 4; ++t)
                for (int h = 0; h < 4; ++h) {
                    const int row = g + 8 * (h >> 1), blk = 2 * t + (h & 1);
                    copy_bytes(raw + row * row_bytes + (gi * 8 + blk) * 18, hdr + ((g * 4 + t) * 4 + h) * 2, 2);
                }
    }
    for (int lane = 0; lane < 32; ++lane) {
        const int g = lane >> 2, t = lane & 3;
        for (int c = 0; c < 8; ++c)
            for (int kind = 0; kind < 2; ++kind) {
                const uint32_t w = get32(in + ((c >> 1) * 32 + lane) * 16 + 8 * (c & 1) + 4 * kind);
                for (int j = 0; j < 4; ++j) {
                    const int v = mma_value(type, c, t, kind, j);
                    const uint32_t b = (w >> (8 * j)) & 0xFFu;
                    for (int half = 0; half < 2; ++half) {
                        uint8_t* row = raw + (g + 8 * half) * row_bytes;
                        const uint32_t q = (b >> (4 * half)) & 0xFu;
                        int sh;
                        uint8_t* p = const_cast<uint8_t*>(q4_byte(type, row, gi, v, &sh));
                        *p = uint8_t((*p & ~(0xFu << sh)) | (q << sh));
                        if (type == T_Q5_K) {
                            const int k = half + 2 * kind;
                            const uint32_t hw = get32(in + 2048 + lane * 16 + 4 * (c >> 1));
                            int bit;
                            uint8_t* hb = const_cast<uint8_t*>(q5_hbyte(row, gi, v, &bit));
                            const uint32_t hv = (hw >> q5_plane_bit(c, k, j)) & 1u;
                            *hb = uint8_t((*hb & ~(1u << bit)) | (hv << bit));
                        }
                    }
                }
            }
    }
}

}  // namespace xb
