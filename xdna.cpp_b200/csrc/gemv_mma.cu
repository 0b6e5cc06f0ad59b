// Integer tensor-core GEMV for all nine claimed formats on sm_100a: Q4_0, Q3_K, Q4_K, Q5_K, Q6_K, IQ4_XS,
// IQ3_S, IQ3_XXS and IQ2_S.
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
//     streaming load per lane yields two chunks' A fragments with one mask
//     per register (rows g+8 are used in place as 16 q and scaled back in the
//     integer combine); the x digits (B) come from L1, written once per launch
//     by xprep_kernel in a per-lane slot layout that needs no selects.
//
// Accumulation: exact int32 inside a block, F32 across blocks (the products
// never round, so the result is at least as accurate as the reference's
// sequential F32 dot).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <mutex>

#include "formats.cuh"
#include "gemv.cuh"
#include "iq_tables.h"  // generated at build time from the gguf package

namespace xb {
namespace {


__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded waits on the peers' flags: 1 s of %globaltimer.
constexpr uint64_t kGatherWaitNs = 1000000000ull;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
// An integer 0 <= v < 2^23 as a float, exactly: its bits under the exponent
// of 2^23, less 2^23 (a logic and a float instruction; no conversion pipe).
__device__ __forceinline__ float u23f(uint32_t v) { return __int_as_float(0x4B000000u | v) - 8388608.0f; }
__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

__device__ __forceinline__ void mma_s8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Work split and scratch.
//
// The GEMV's unit of work is one (16-row tile, 256-value group) pair, the
// format's group bytes of the MMA layout (2304 for Q4_0 / Q4_K); units are
// numbered tile-major, so unit u lives at W + u * group bytes.  In unit mode
// each warp of the grid takes one contiguous, equal-sized range of units
// (warp w: [w U / NW, (w + 1) U / NW)), so every warp streams the same number
// of bytes whatever N and K are: no partial waves, no idle SMs on short
// matrices.  Small launches run in tile mode instead (struct Split below):
// whole tiles per CTA, so step 2 below never happens.  A tile whose groups are
// split across warps is combined in two levels, always adding in a fixed
// order (deterministic results):
//   1. each contributor writes its 16 partial rows to shared memory (two
//      slots per warp: a warp can share only its first and its last tile) and
//      counts itself in with a shared-memory atomic; the CTA's last
//      contributor adds the CTA's partials in warp order;
//   2. if the tile also has contributors in other CTAs (only a CTA's first
//      and last tile can), that warp writes the CTA's sum to global memory
//      and counts in at the tile's global counter; the last CTA adds the
//      CTAs' sums in CTA order.  Otherwise it writes y directly.
// Only tiles that cross a CTA boundary pay for a device-scope fence and atomic.
//
// Scratch of one launch (all offsets 256-byte aligned):
//   frags   per group, per chunk c (32 values of each of the 8 blocks), per
//           block b: a 32-byte B-fragment slot: {b0,b1} of digit planes 0
//           and 1, then, in an even chunk's slot, {b0,b1} of plane 2 of
//           this chunk and of the next (an odd chunk's last 16 bytes are
//           unused), so a chunk pair takes three 16-byte loads.
//           Block b < 4 is supplied by lane (g = b, t = b) in register b0,
//           block b >= 4 by lane (g = b, t = b - 4) in register b1; the other
//           register of the pair is zero, so the kernel needs no selects.
//   zeros   kZeroBytes of zeros: the B "slots" of the 24 lanes that supply nothing
//   scale   2^e per 32-value block;  xsum  sum of the block's x
//   count   one arrival counter per tile, the CTA completion counter and one
//           per 32-value chunk of a feeding output (cleared by xprep_kernel,
//           or by the previous launch when it prepared x)
//   partial kMaxCtas CTAs * 2 slots * 16 floats (level-2 CTA sums)
// ---------------------------------------------------------------------------
// One CTA of 24 warps per SM: warps of one CTA are scheduled as equals,
// while of three 8-warp CTAs on an SM the one that started first finished
// about 2.5 us (10 %) before the last, leaving the SM short of loads in flight
// at the end of every launch.
constexpr int kWarps = 24;
constexpr int kGemvThreads = kWarps * 32;
constexpr int kCtasPerSm = 1;
constexpr int kMaxCtas = 512;        // bounds the partial-slot area
constexpr int kPrefetch = 2;         // groups ahead per warp (bulk L2 prefetch; 2 measured ahead of 4 and 8)
constexpr int kSlotBytes = 32;
constexpr int kChunkFragBytes = 8 * kSlotBytes;       // 8 blocks
constexpr int kGroupFragBytes = 8 * kChunkFragBytes;  // 8 chunks: 2 KiB per 256 values
// The zero B fragments of the 24 lanes that supply no x block: one group's
// worth of zero slots, so that those lanes step through it with the same
// constant chunk stride as the supplying lanes through the x fragments, and
// every fragment load of a group takes an immediate offset from one address.
constexpr int kZeroBytes = kGroupFragBytes;

__device__ __forceinline__ uint32_t digit_word(uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3, int plane) {
    // byte `plane` of each of four lanes' packed digits, in value order
    const uint32_t sel = 0x0040u | (static_cast<uint32_t>(plane) * 0x0011u);
    return __byte_perm(__byte_perm(v0, v1, sel), __byte_perm(v2, v3, sel), 0x5410);
}

// x preparation of 32 consecutive values x[32 w32 + lane] held one per lane
// (one 32-value block, or two 16-value blocks when BL = 16): the block scale
// 2^e, the block sum and the three digit planes, written to the fragment slots.
// BL = values per x block (B column): 32, or 16 for the formats with
// 16-value sub-blocks (chunks 0-3 then cover blocks 0-7, chunks 4-7 blocks
// 8-15 of the group).
// Peer copies of a prepared x (row-sharded chains): the same bytes also go to
// every other rank's scratch slot, at the same offset from that rank's
// exchange base (pb[p]) as from this rank's (pb[rank]).
struct PeerDest {
    const float* const* pb;  // nullptr: none
    int world, rank;
};
template <typename T>
__device__ __forceinline__ T* at_peer(const PeerDest& d, int p, T* local) {
    const char* mine = reinterpret_cast<const char*>(__ldg(reinterpret_cast<const unsigned long long*>(d.pb) + d.rank));
    const char* theirs = reinterpret_cast<const char*>(__ldg(reinterpret_cast<const unsigned long long*>(d.pb) + p));
    return reinterpret_cast<T*>(const_cast<char*>(theirs) + (reinterpret_cast<const char*>(local) - mine));
}

template <int BL>
__device__ __forceinline__ void prep_x32(float v, int64_t w32, int lane, uint8_t* __restrict__ frags,
                                         float* __restrict__ scale, float* __restrict__ xsum,
                                         const PeerDest pd = PeerDest{nullptr, 0, 0}) {
    const int64_t b = (w32 * 32 + lane) / BL;  // this lane's block
    // a block holding an infinity or a NaN gets a NaN scale and sum, so every
    // output it reaches is NaN, as in an F32 dot product (the fixed-point
    // digits cannot carry it)
    const uint32_t nonfinite = __ballot_sync(0xffffffffu, !isfinite(v));
    const bool bad = BL == 32 ? nonfinite != 0u : ((nonfinite >> (lane & 16)) & 0xFFFFu) != 0u;
    float m = isfinite(v) ? fabsf(v) : 0.f, s = v;
#pragma unroll
    for (int o = BL / 2; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    int E = 0;
    if (m > 0.f) frexpf(m, &E);  // m < 2^E
    int e = m > 0.f ? E - 22 : 0;
    e = e < -120 ? -120 : (e > 120 ? 120 : e);
    const int X = isfinite(v) ? __float2int_rn(v * ldexpf(1.0f, -e)) : 0;  // |X| <= 2^22
    const int d0 = ((X + 128) & 255) - 128;
    const int X1 = (X - d0) >> 8;
    const int d1 = ((X1 + 128) & 255) - 128;
    const int d2 = (X1 - d1) >> 8;                        // |d2| <= 64
    const uint32_t mine = (static_cast<uint32_t>(d0) & 0xFFu) | ((static_cast<uint32_t>(d1) & 0xFFu) << 8) |
                          ((static_cast<uint32_t>(d2) & 0xFFu) << 16);
    const uint32_t n1 = __shfl_down_sync(0xffffffffu, mine, 1);
    const uint32_t n2 = __shfl_down_sync(0xffffffffu, mine, 2);
    const uint32_t n3 = __shfl_down_sync(0xffffffffu, mine, 3);
    if ((lane & 3) == 0) {  // values 4c' .. 4c' + 3 of the block, c' = (lane % BL) / 4
        const uint32_t D0 = digit_word(mine, n1, n2, n3, 0);
        const uint32_t D1 = digit_word(mine, n1, n2, n3, 1);
        const uint32_t D2 = digit_word(mine, n1, n2, n3, 2);
        constexpr int kPerGroup = 256 / BL;
        const int64_t gi = b / kPerGroup;
        const int jb = static_cast<int>(b % kPerGroup);
        const int blk = jb & 7;                                          // B column
        const int c = (BL == 32 ? 0 : 4 * (jb >> 3)) + (lane % BL) / 4;  // chunk
        // planes 0 and 1 to the chunk's slot; plane 2 to the last 16 bytes of
        // the chunk pair's even slot, first half for the even chunk (load_b)
        uint8_t* sb = frags + gi * kGroupFragBytes + c * kChunkFragBytes + blk * kSlotBytes;
        uint4* slot = reinterpret_cast<uint4*>(sb);
        uint2* p2 = reinterpret_cast<uint2*>((c & 1) ? sb - kChunkFragBytes + 24 : sb + 16);
        const uint4 s0 = blk < 4 ? make_uint4(D0, 0u, D1, 0u) : make_uint4(0u, D0, 0u, D1);
        const uint2 s1 = blk < 4 ? make_uint2(D2, 0u) : make_uint2(0u, D2);
        *slot = s0;
        *p2 = s1;
        if (pd.pb)
            for (int p = 0; p < pd.world; ++p)
                if (p != pd.rank) {
                    *at_peer(pd, p, slot) = s0;
                    *at_peer(pd, p, p2) = s1;
                }
    }
    if (lane % BL == 0) {
        const float sv = bad ? __int_as_float(0x7fc00000) : ldexpf(1.0f, e);
        const float xv = bad ? __int_as_float(0x7fc00000) : s;
        scale[b] = sv;
        xsum[b] = xv;
        if (pd.pb)
            for (int p = 0; p < pd.world; ++p)
                if (p != pd.rank) {
                    *at_peer(pd, p, scale + b) = sv;
                    *at_peer(pd, p, xsum + b) = xv;
                }
    }
}

// x preparation: one warp per 32 values (lane j = value j); also clears the
// counters (ncount ints) of the GEMV that follows.
template <int BL>
__global__ void __launch_bounds__(64) xprep_kernel(const float* __restrict__ x, int64_t K, uint8_t* __restrict__ frags,
                                                    uint8_t* __restrict__ zeros, float* __restrict__ scale,
                                                    float* __restrict__ xsum, int* __restrict__ count,
                                                    int64_t ncount) {
    pdl_release();
    pdl_wait();
    const int64_t gtid = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    const int64_t nthr = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = gtid; i < ncount; i += nthr) count[i] = 0;
    for (int64_t i = gtid; i < kZeroBytes / 4; i += nthr) reinterpret_cast<uint32_t*>(zeros)[i] = 0u;
    const int lane = threadIdx.x & 31;
    const int64_t nw = K / 32;
    for (int64_t w32 = gtid >> 5; w32 < nw; w32 += nthr >> 5) prep_x32<BL>(x[w32 * 32 + lane], w32, lane, frags, scale, xsum);
}

// One launch covers up to kMaxSegs weight matrices that share x (and K):
// their 16-row tiles are numbered one after the other, matrix s owning tiles
// [tile_end[s-1], tile_end[s]).
constexpr int kMaxSegs = MMA_MAX_SEGMENTS;

struct GemvArgs {
    const uint8_t* W[kMaxSegs];
    float* y[kMaxSegs];
    int64_t tile_end[kMaxSegs];
    int nseg;
    const uint8_t* frags;
    const uint8_t* zeros;
    const float* scale;
    const float* xsum;
    int* count;
    float* partial;
    int64_t ngroups, units, nwarps;
    int tile_mode;  // small launch: each CTA takes whole tiles (see Split)
    int cta_tiles;  // bound on the tiles one CTA's units touch (shared-memory counters)
    bool xchg;      // row-sharded launch: also store rows into the peers' exchange buffers
    PeerExchange x;
    int* done;      // CTAs finished (cleared with the counters), for the completion flags
    // feed: tiles [f_t0, f_t1) (output f_y) are the next launch's x; its
    // fragments, scales and sums go to f_frags / f_scale / f_xsum; f_chunk
    // counts the two tiles of each 32-value chunk in (f_bl = 0: no feed)
    uint8_t* f_frags;
    float* f_scale;
    float* f_xsum;
    int* f_chunk;
    const float* f_y;
    int64_t f_t0, f_t1;
    int f_bl;
    int* f_count;       // the next launch's counters (f_ncount ints) and zero slot, cleared here
    int64_t f_ncount;
    uint32_t* f_zeros;
    int* err;           // set when a bounded wait (shared-memory ring) runs out
    // row-sharded chain (ShardChain): the feed also goes to the peers; this
    // launch waits for the peers' previous epoch and assembles the previous
    // launch's outputs (prev) before computing
    const float* const* f_pbase;
    int64_t f_ch0;      // the fed output's first 32-value chunk in the full vector (this rank's rows)
    int wait_peers;
    int nprev;
    GatherSeg prev[kMaxSegs];
};

// Matrix s of a (global) tile, and that matrix's first tile, weights and
// output; constant-index selects keep the parameter arrays in the constant
// bank (no dynamically indexed copy of the arguments).
struct SegRef {
    const uint8_t* W;
    float* y;
    int64_t first_tile, end_tile, xo;
};
__device__ __forceinline__ SegRef seg_ref(const GemvArgs& a, int64_t tile) {
    SegRef r{a.W[0], a.y[0], 0, a.tile_end[0], a.x.xo[0]};
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < a.nseg && tile >= a.tile_end[i - 1])
            r = SegRef{a.W[i], a.y[i], a.tile_end[i - 1], a.tile_end[i], a.x.xo[i]};
    return r;
}

// Output row `row` (0..15) of global tile `tile`: to y, and for a sharded
// launch to the same place of every peer's exchange buffer (NVLink stores).
// hoff: the launch's exchange data half (sharded launches)
__device__ __forceinline__ void emit(const GemvArgs& a, float* ty, int tile, int row, float v, int64_t hoff) {
    ty[row] = v;
    if (a.xchg) {
        const SegRef sr = seg_ref(a, tile);
        const int64_t n_local = (sr.end_tile - sr.first_tile) * MMA_TILE_ROWS;
        const int64_t off = hoff + sr.xo + a.x.rank * n_local + (tile - sr.first_tile) * MMA_TILE_ROWS + row;
#pragma unroll
        for (int p = 0; p < kMaxPeers; ++p)
            if (p < a.x.world && p != a.x.rank) a.x.peer_data[p][off] = v;
    }
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// The peers' flags of a finished sharded launch, raised by the CTA that
// counted in last: one system-scope release fence (cumulative over every
// CTA's stores, which it observed through the completion counter) followed
// by plain system-scope stores, so the flags of all peers share one fence.
__device__ __forceinline__ void raise_peer_flags(const PeerExchange& x, uint32_t e) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int p = 0; p < x.world; ++p)
        if (p != x.rank) st_relaxed_sys(x.peer_flags[p] + x.rank, e);
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// A warp counts in at *p once: every lane's earlier stores are released
// with lane 0's atomic (the warp barrier orders them before it), and every
// lane's later loads are ordered after it.  Returns the old count to all
// lanes.  One acquire-release atomic in place of a fence on each side.
__device__ __forceinline__ int warp_count_in(int* p) {
    __syncwarp();
    int prev = 0;
    if ((threadIdx.x & 31) == 0) prev = atom_add_acq_rel_gpu(p, 1);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    __syncwarp();
    return prev;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// bytes of one (16-row tile, 256-value group) unit of format TYPE
template <int TYPE>
constexpr int kUnitBytes =
    TYPE == T_Q5_K ? 2816
                   : (TYPE == T_Q6_K ? 3360
                                     : ((TYPE == T_Q3_K || TYPE == T_IQ3_S)
                                            ? 1760
                                            : (TYPE == T_IQ4_XS ? 2176
                                                                : (TYPE == T_IQ3_XXS ? 1568
                                                                                     : (TYPE == T_IQ2_S ? 1312
                                                                                                        : MMA_GROUP_BYTES)))));
template <int TYPE>
constexpr int kHeaderOff = TYPE == T_Q5_K ? 2560 : 2048;
template <int TYPE>
constexpr int kXBlocks = (TYPE == T_Q6_K || TYPE == T_Q3_K || TYPE == T_IQ2_S) ? 16 : 8;  // x blocks per 256 values

template <int TYPE>
__device__ __forceinline__ const uint8_t* unit_weights(const GemvArgs& a, int64_t u) {
    const int64_t tile = u / a.ngroups;
    const SegRef r = seg_ref(a, tile);
    return r.W + ((tile - r.first_tile) * a.ngroups + (u - tile * a.ngroups)) * kUnitBytes<TYPE>;
}

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
// first warp of the split whose range holds unit u
__device__ __forceinline__ int64_t warp_of(int64_t u, int64_t U, int64_t NW) { return ((u + 1) * NW + U - 1) / U - 1; }

// Unit ranges of the warps.  Unit mode: warp w of the NW working warps takes
// [w U / NW, (w + 1) U / NW), an equal share whatever N and K are (inline in
// the kernel).  Tile mode (small launches, where the cross-CTA combine would
// be a large part of the time; this struct): CTA c of NC takes whole tiles
// [c T / NC, (c + 1) T / NC) and its warps split that CTA's units, so no tile
// spans two CTAs.
struct Split {
    int U, ng, NW, T, NC;
    // U <= 64 units per SM, so 32-bit unsigned arithmetic is exact
    static __device__ __forceinline__ int mdiv(int a, int b, int c) {
        return static_cast<int>(static_cast<uint32_t>(a) * static_cast<uint32_t>(b) / static_cast<uint32_t>(c));
    }
    static __device__ __forceinline__ int inv(int u, int n, int parts) {  // warp_of in 32 bits
        return static_cast<int>((static_cast<uint32_t>(u + 1) * parts + n - 1) / static_cast<uint32_t>(n)) - 1;
    }
    __device__ __forceinline__ int cta_unit0(int c) const { return mdiv(c, T, NC) * ng; }
    // A CTA's units go to its first ceil(units / 2) warps (at most all of
    // them): about two units per warp, and consecutive warps, so that the
    // warps sharing a tile are always consecutive (the shared-memory combine
    // counts every warp from first to last).
    static __device__ __forceinline__ int cta_warps(int uc) { return (uc + 1) / 2 < kWarps ? (uc + 1) / 2 : kWarps; }
    __device__ __forceinline__ int warp_unit0(int w) const {
        const int c = w / kWarps, i = w - c * kWarps;
        if (c >= NC) return U;
        const int cs = cta_unit0(c), ce = cta_unit0(c + 1);
        const int nw = cta_warps(ce - cs);
        return i >= nw ? ce : cs + mdiv(i, ce - cs, nw);
    }
    // the warp whose range holds unit u
    __device__ __forceinline__ int warp_of_unit(int u) const {
        const int c = inv(u / ng, T, NC);
        const int cs = cta_unit0(c), uc = cta_unit0(c + 1) - cs;
        return c * kWarps + inv(u - cs, uc, cta_warps(uc));
    }
};

// Loads of a group's weights (W) and of the x fragments (X): from global
// memory (streaming loads for the weights, the read-only cache for the
// rest), or from a shared-memory stage filled by bulk copies.
struct LdGlobal {
    static __device__ __forceinline__ uint4 q(const uint8_t* p) { return ld_stream(p); }
    static __device__ __forceinline__ uint4 q_ro(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
    static __device__ __forceinline__ uint2 d(const uint8_t* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    static __device__ __forceinline__ uint32_t w(const uint8_t* p) {
        return __ldg(reinterpret_cast<const unsigned int*>(p));
    }
    static __device__ __forceinline__ uint32_t h(const uint8_t* p) {
        return __ldg(reinterpret_cast<const unsigned short*>(p));
    }
};
struct LdShared {
    static __device__ __forceinline__ uint4 q(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
    static __device__ __forceinline__ uint4 q_ro(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
    static __device__ __forceinline__ uint2 d(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
    static __device__ __forceinline__ uint32_t w(const uint8_t* p) { return *reinterpret_cast<const unsigned int*>(p); }
    static __device__ __forceinline__ uint32_t h(const uint8_t* p) { return *reinterpret_cast<const unsigned short*>(p); }
};

// Byte permute (prmt.b32): result byte i is byte sel[4i+2:4i] of {b, a}
// (a = bytes 0-3), or that byte's sign replicated when sel[4i+3] is set.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// B fragments of chunk c: planes 0 and 1 (q) from the chunk's slot, plane 2
// (r) from the slot of the chunk pair's even member, whose last 16 bytes
// hold plane 2 of both chunks (r2, loaded at the even chunk and kept for the
// odd one): three 16-byte loads per chunk pair.
template <class X>
__device__ __forceinline__ void load_b(const uint8_t* fb, int c, int fc, uint4& q, uint2& r, uint4& r2) {
    q = X::q_ro(fb + c * fc);
    if ((c & 1) == 0) r2 = X::q_ro(fb + c * fc + 16);
    r = (c & 1) ? make_uint2(r2.z, r2.w) : make_uint2(r2.x, r2.y);
}

// One group of 16 rows x 256 values: accumulate rows g and g+8 of this lane.
// fb: this lane's B slot of chunk 0 (or the zero slot), fc: bytes between chunks.
// Q6_K: two sets of 8 sixteen-value blocks; q = 6 bits (A = q, u8), value =
// d * sc * (q - 32) with int8 sc per 16 values, so each block adds
// d * sc * (2^e * T - 32 * xsum).
template <class W, class X>
__device__ __forceinline__ void group_dot_q6k(const uint8_t* gb, const uint8_t* fb, int fc,
                                              const float* __restrict__ sc_, const float* __restrict__ xs_, int lane,
                                              int g, int t, float& y0, float& y8) {
    uint4 A[4], H[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] = W::q(gb + (i * 32 + lane) * 16);
    H[0] = W::q(gb + 2048 + lane * 32);
    H[1] = W::q(gb + 2048 + lane * 32 + 16);
    const uint2 scw = W::d(gb + 3072 + 8 * lane);
    const float dg = h2f(W::h(gb + 3328 + 2 * g));
    const float d8 = h2f(W::h(gb + 3328 + 2 * (g + 8)));
#pragma unroll
    for (int st = 0; st < 2; ++st) {
        int C[3][4];
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int k = 0; k < 4; ++k) C[p][k] = 0;
        uint4 r2;  // plane 2 of the current chunk pair
#pragma unroll
        for (int cs = 0; cs < 4; ++cs) {
            const int c = 4 * st + cs;
            uint4 q;
            uint2 r;
            load_b<X>(fb, c, fc, q, r, r2);
            const uint32_t w0 = word(A[c >> 1], 2 * (c & 1)), w1 = word(A[c >> 1], 2 * (c & 1) + 1);
            const uint32_t hw = word(H[c >> 2], c & 3);  // bits 8j + 2k: high pair of register k
            const uint32_t a0 = (w0 & 0x0F0F0F0Fu) | ((hw << 4) & 0x30303030u);
            const uint32_t a1 = ((w0 >> 4) & 0x0F0F0F0Fu) | ((hw << 2) & 0x30303030u);
            const uint32_t a2 = (w1 & 0x0F0F0F0Fu) | (hw & 0x30303030u);
            const uint32_t a3 = ((w1 >> 4) & 0x0F0F0F0Fu) | ((hw >> 2) & 0x30303030u);
            mma_u8s8(C[0], a0, a1, a2, a3, q.x, q.y);
            mma_u8s8(C[1], a0, a1, a2, a3, q.z, q.w);
            mma_u8s8(C[2], a0, a1, a2, a3, r.x, r.y);
        }
        // |sum| <= 16 * 63 * 2^22 may pass 2^31: join the planes in F32
        float T[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            T[k] = fmaf(static_cast<float>(C[2][k]), 65536.0f, static_cast<float>(C[1][k] * 256 + C[0][k]));
        const float2 sc2 = reinterpret_cast<const float2*>(sc_ + 8 * st)[t];
        const float2 xs2 = reinterpret_cast<const float2*>(xs_ + 8 * st)[t];
        const uint32_t sg = (st ? scw.x >> 16 : scw.x), s8 = (st ? scw.y >> 16 : scw.y);
        const float kg0 = static_cast<float>(static_cast<int8_t>(sg & 0xFFu));
        const float kg1 = static_cast<float>(static_cast<int8_t>((sg >> 8) & 0xFFu));
        const float k80 = static_cast<float>(static_cast<int8_t>(s8 & 0xFFu));
        const float k81 = static_cast<float>(static_cast<int8_t>((s8 >> 8) & 0xFFu));
        const float b0 = fmaf(-32.0f, xs2.x, 0.0f), b1 = -32.0f * xs2.y;
        y0 = fmaf(dg, fmaf(kg0, fmaf(sc2.x, T[0], b0), kg1 * fmaf(sc2.y, T[1], b1)), y0);
        y8 = fmaf(d8, fmaf(k80, fmaf(sc2.x, T[2], b0), k81 * fmaf(sc2.y, T[3], b1)), y8);
    }
}

// Q3_K: two sets of 8 sixteen-value blocks; q3 = low pair + 4 * high bit
// (A = q3, u8), value = d * (sc - 32) * (q3 - 4) with 6-bit sc per 16 values.
template <class W, class X>
__device__ __forceinline__ void group_dot_q3k(const uint8_t* gb, const uint8_t* fb, int fc,
                                              const float* __restrict__ sc_, const float* __restrict__ xs_, int lane,
                                              int g, int t, float& y0, float& y8) {
    const uint4 L0 = W::q(gb + lane * 32), L1 = W::q(gb + lane * 32 + 16);
    const uint4 H = W::q(gb + 1024 + lane * 16);
    const uint32_t slo = W::w(gb + 1536 + 4 * lane);
    const uint32_t shi = W::h(gb + 1664 + 2 * lane);
    const float dg = h2f(W::h(gb + 1728 + 2 * g));
    const float d8 = h2f(W::h(gb + 1728 + 2 * (g + 8)));
#pragma unroll
    for (int st = 0; st < 2; ++st) {
        int C[3][4];
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int k = 0; k < 4; ++k) C[p][k] = 0;
        uint4 r2;  // plane 2 of the current chunk pair
#pragma unroll
        for (int cs = 0; cs < 4; ++cs) {
            const int c = 4 * st + cs;
            uint4 q;
            uint2 r;
            load_b<X>(fb, c, fc, q, r, r2);
            const uint32_t lw = word(c < 4 ? L0 : L1, c & 3);  // bits 8j + 2k: low pair of register k
            const uint32_t hw = word(H, c >> 1);                // bit 8j + 4 (c & 1) + k: high bit
            uint32_t hk[4];
            if (c & 1) {
#pragma unroll
                for (int k = 0; k < 4; ++k) hk[k] = hw >> (2 + k);
            } else {
                hk[0] = hw << 2;
                hk[1] = hw << 1;
                hk[2] = hw;
                hk[3] = hw >> 1;
            }
            const uint32_t a0 = (lw & 0x03030303u) | (hk[0] & 0x04040404u);
            const uint32_t a1 = ((lw >> 2) & 0x03030303u) | (hk[1] & 0x04040404u);
            const uint32_t a2 = ((lw >> 4) & 0x03030303u) | (hk[2] & 0x04040404u);
            const uint32_t a3 = ((lw >> 6) & 0x03030303u) | (hk[3] & 0x04040404u);
            mma_u8s8(C[0], a0, a1, a2, a3, q.x, q.y);
            mma_u8s8(C[1], a0, a1, a2, a3, q.z, q.w);
            mma_u8s8(C[2], a0, a1, a2, a3, r.x, r.y);
        }
        // |sum| <= 16 * 7 * 2^22 < 2^31: exact in int32
        float T[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) T[k] = static_cast<float>(C[2][k] * 65536 + C[1][k] * 256 + C[0][k]);
        const float2 sc2 = reinterpret_cast<const float2*>(sc_ + 8 * st)[t];
        const float2 xs2 = reinterpret_cast<const float2*>(xs_ + 8 * st)[t];
        float k6[4];  // scales (i = 4 h + 2 st + b) minus 32
#pragma unroll
        for (int hb = 0; hb < 4; ++hb) {
            const int i = 4 * (hb >> 1) + 2 * st + (hb & 1);
            const uint32_t v = ((slo >> (4 * i)) & 0xFu) | (((shi >> (2 * i)) & 3u) << 4);
            k6[hb] = u23f(v) - 32.0f;
        }
        const float b0 = -4.0f * xs2.x, b1 = -4.0f * xs2.y;
        y0 = fmaf(dg, fmaf(k6[0], fmaf(sc2.x, T[0], b0), k6[1] * fmaf(sc2.y, T[1], b1)), y0);
        y8 = fmaf(d8, fmaf(k6[2], fmaf(sc2.x, T[2], b0), k6[3] * fmaf(sc2.y, T[3], b1)), y8);
    }
}

// IQ4_XS: value = d * (ls - 32) * kvalues[q] with a 6-bit ls per 32 values
// (ggml-quants.c dequantize_row_iq4_xs).  A = kvalues[q] as s8 from two
// 8-entry byte tables held in registers.  The layout stores code = q with bits
// 2 and 3 swapped, so codes i and i + 8 name values of one sign.  prmt with a
// selector nibble below 8 copies byte i; with bit 3 set it replicates the sign
// of byte i.  XA holds the values of codes 0-7 and XB those of codes 8-15
// (complemented where the pair is negative); so for a code below 8 the XB
// lookup (code ^ 8) gives 0, for a code of 8 or more the XA lookup gives the
// pair's sign, and the XOR of the two lookups is the value either way.
// Each code word holds registers (k, k+1) as 16-bit selector halves.
__device__ __forceinline__ void iq4nl_lookup2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t x = w ^ 0x88888888u;
    lo = prmt(XB_IQ4NL_XA_0, XB_IQ4NL_XA_1, w) ^ prmt(XB_IQ4NL_XB_0, XB_IQ4NL_XB_1, x);
    hi = prmt(XB_IQ4NL_XA_0, XB_IQ4NL_XA_1, w >> 16) ^ prmt(XB_IQ4NL_XB_0, XB_IQ4NL_XB_1, x >> 16);
}

template <class W, class X>
__device__ __forceinline__ void group_dot_iq4xs(const uint8_t* gb, const uint8_t* fb, int fc,
                                                const float* __restrict__ sc_, int lane, int g, int t, float& y0,
                                                float& y8) {
    uint4 A[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] = W::q(gb + (i * 32 + lane) * 16);
    const uint2 h0 = W::d(gb + 2048 + 8 * g);  // {d | scales_h << 16, scales_l}
    const uint2 h8 = W::d(gb + 2048 + 8 * (g + 8));
    int C[3][4];
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int k = 0; k < 4; ++k) C[p][k] = 0;
    uint4 r2;  // plane 2 of the current chunk pair
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 q;
        uint2 r;
        load_b<X>(fb, c, fc, q, r, r2);
        uint32_t a0, a1, a2, a3;
        iq4nl_lookup2(word(A[c >> 1], 2 * (c & 1)), a0, a1);
        iq4nl_lookup2(word(A[c >> 1], 2 * (c & 1) + 1), a2, a3);
        mma_s8s8(C[0], a0, a1, a2, a3, q.x, q.y);
        mma_s8s8(C[1], a0, a1, a2, a3, q.z, q.w);
        mma_s8s8(C[2], a0, a1, a2, a3, r.x, r.y);
    }
    // |sum| <= 32 * 127 * 2^23 passes 2^31: join the planes in F32
    float T[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        T[k] = fmaf(static_cast<float>(C[2][k]), 65536.0f, static_cast<float>(C[1][k] * 256 + C[0][k]));
    const float2 sc2 = __ldg(reinterpret_cast<const float2*>(sc_) + t);
    // six-bit scales of sub-blocks 2t, 2t+1: low nibbles at bit 4 ib of
    // scales_l, high pairs at bit 2 ib of scales_h
    float k6[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint2 hh = h ? h8 : h0;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const int ib = 2 * t + b;
            const uint32_t ls = ((hh.y >> (4 * ib)) & 0xFu) | (((hh.x >> (16 + 2 * ib)) & 3u) << 4);
            k6[h][b] = u23f(ls) - 32.0f;
        }
    }
    y0 = fmaf(h2f(h0.x), fmaf(k6[0][0] * sc2.x, T[0], k6[0][1] * sc2.y * T[1]), y0);
    y8 = fmaf(h2f(h8.x), fmaf(k6[1][0] * sc2.x, T[2], k6[1][1] * sc2.y * T[3]), y8);
}

// Grid lookups of the IQ3 formats go to shared memory at random entries, and
// 32 lanes reading random words of one table conflict on its banks (about 4
// wavefronts per load instead of 1).  So each CTA holds several copies of a
// grid, interleaved word by word: entry e of copy j sits at word
// e * copies + j, and lane l reads copy l % copies, in bank l % 32 when there
// are 32 copies.  Static shared memory stops at 48 KiB per CTA: IQ3_XXS
// (256 entries) gets 32 copies, IQ3_S (512 entries) 16 (two lanes per bank),
// in 32 KiB each.
constexpr int kIq3sCopies = 16;
constexpr int kIq3xxsCopies = 32;
template <int TYPE>
constexpr size_t kGridSmem = TYPE == T_IQ3_S     ? 512 * kIq3sCopies * 4
                             : TYPE == T_IQ3_XXS ? 256 * kIq3xxsCopies * 4
                             : TYPE == T_IQ2_S   ? 1024 * 8
                                                 : 0;

// IQ3_S: value = d * (1 + 2 s) * grid[idx] * sign with a 4-bit s per 32
// values (ggml-quants.c dequantize_row_iq3_s).  Each A register is one grid
// entry (4 unsigned magnitudes 1..15) read from the lane's copy of the
// 512-entry grid, with its 4 sign bits applied per byte: the bits are spread
// to the bytes' top bits by a multiply, prmt's sign-replicate mode widens
// them to 0x00 / 0xFF masks m, and (g ^ m) + (m & 1) negates the masked bytes
// (no carry between bytes: every magnitude is at least 1).
__shared__ uint32_t s_iq3s_grid[512 * kIq3sCopies];

// four unsigned magnitudes g (each >= 1) with 4 sign bits applied, as s8
__device__ __forceinline__ uint32_t signed4(uint32_t g, uint32_t s4) {
    const uint32_t m = prmt(s4 * 0x10204080u, 0u, 0xBA98u);
    return (g ^ m) + (m & 0x01010101u);
}
__device__ __forceinline__ uint32_t iq3s_reg(uint32_t iw, uint32_t hw, uint32_t sw, int k, int lane) {
    const uint32_t idx = ((iw >> (8 * k)) & 0xFFu) | (((hw >> k) & 1u) << 8);
    return signed4(s_iq3s_grid[idx * kIq3sCopies + (lane & (kIq3sCopies - 1))], (sw >> (4 * k)) & 0xFu);
}

template <class W, class X>
__device__ __forceinline__ void group_dot_iq3s(const uint8_t* gb, const uint8_t* fb, int fc,
                                               const float* __restrict__ sc_, int lane, int g, int t, float& y0,
                                               float& y8) {
    const uint4 I0 = W::q(gb + lane * 32), I1 = W::q(gb + lane * 32 + 16);
    const uint4 S = W::q(gb + 1024 + lane * 16);
    const uint32_t qh = W::w(gb + 1536 + 4 * lane);
    const float dg = h2f(W::h(gb + 1664 + 2 * g));
    const float d8 = h2f(W::h(gb + 1664 + 2 * (g + 8)));
    const uint32_t sg = W::w(gb + 1696 + 4 * g);
    const uint32_t s8 = W::w(gb + 1696 + 4 * (g + 8));
    int C[3][4];
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int k = 0; k < 4; ++k) C[p][k] = 0;
    uint4 r2;  // plane 2 of the current chunk pair
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 q;
        uint2 r;
        load_b<X>(fb, c, fc, q, r, r2);
        const uint32_t iw = word(c < 4 ? I0 : I1, c & 3);
        const uint32_t sw = word(S, c >> 1) >> (16 * (c & 1));
        const uint32_t hw = qh >> (4 * c);
        const uint32_t a0 = iq3s_reg(iw, hw, sw, 0, lane), a1 = iq3s_reg(iw, hw, sw, 1, lane);
        const uint32_t a2 = iq3s_reg(iw, hw, sw, 2, lane), a3 = iq3s_reg(iw, hw, sw, 3, lane);
        mma_s8s8(C[0], a0, a1, a2, a3, q.x, q.y);
        mma_s8s8(C[1], a0, a1, a2, a3, q.z, q.w);
        mma_s8s8(C[2], a0, a1, a2, a3, r.x, r.y);
    }
    // |sum| <= 32 * 15 * 2^23 passes 2^31: join the planes in F32
    float T[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        T[k] = fmaf(static_cast<float>(C[2][k]), 65536.0f, static_cast<float>(C[1][k] * 256 + C[0][k]));
    const float2 sc2 = __ldg(reinterpret_cast<const float2*>(sc_) + t);
    // scales of blocks 2t (low nibble) and 2t + 1 (high nibble) are byte t of the row's scales
    const uint32_t bg = (sg >> (8 * t)) & 0xFFu, b8 = (s8 >> (8 * t)) & 0xFFu;
    const float kg0 = u23f(2u * (bg & 0xFu) + 1u), kg1 = u23f(2u * (bg >> 4) + 1u);
    const float k80 = u23f(2u * (b8 & 0xFu) + 1u), k81 = u23f(2u * (b8 >> 4) + 1u);
    y0 = fmaf(dg, fmaf(kg0 * sc2.x, T[0], kg1 * sc2.y * T[1]), y0);
    y8 = fmaf(d8, fmaf(k80 * sc2.x, T[2], k81 * sc2.y * T[3]), y8);
}

// IQ3_XXS: value = d * (0.5 + s) / 2 * grid[q] * sign with a 4-bit s per 32
// values (gguf quants.py IQ3_XXS).  As IQ3_S, one shared-memory grid entry
// (256 entries, magnitudes 4..62, one copy per lane) per A register; the 8
// signs of 8 values are a 7-bit index plus the bit that makes the count of
// negatives even.
__shared__ uint32_t s_iq3xxs_grid[256 * kIq3xxsCopies];

template <class W, class X>
__device__ __forceinline__ void group_dot_iq3xxs(const uint8_t* gb, const uint8_t* fb, int fc,
                                                 const float* __restrict__ sc_, int lane, int g, int t, float& y0,
                                                 float& y8) {
    const uint4 I0 = W::q(gb + lane * 32), I1 = W::q(gb + lane * 32 + 16);
    const uint4 SS = W::q(gb + 1024 + lane * 16);
    const float dg = h2f(W::h(gb + 1536 + 2 * g));
    const float d8 = h2f(W::h(gb + 1536 + 2 * (g + 8)));
    int C[3][4];
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int k = 0; k < 4; ++k) C[p][k] = 0;
    uint4 r2;  // plane 2 of the current chunk pair
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 q;
        uint2 r;
        load_b<X>(fb, c, fc, q, r, r2);
        const uint32_t iw = word(c < 4 ? I0 : I1, c & 3);
        const uint32_t w = word(SS, c >> 1);
        uint32_t a[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t si = (w >> (7 * k)) & 127u;
            const uint32_t sb = si | ((__popc(si) & 1u) << 7);
            a[k] = signed4(s_iq3xxs_grid[((iw >> (8 * k)) & 0xFFu) * kIq3xxsCopies + lane], (sb >> (4 * (c & 1))) & 0xFu);
        }
        mma_s8s8(C[0], a[0], a[1], a[2], a[3], q.x, q.y);
        mma_s8s8(C[1], a[0], a[1], a[2], a[3], q.z, q.w);
        mma_s8s8(C[2], a[0], a[1], a[2], a[3], r.x, r.y);
    }
    // |sum| <= 32 * 62 * 2^23 passes 2^31: join the planes in F32
    float T[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        T[k] = fmaf(static_cast<float>(C[2][k]), 65536.0f, static_cast<float>(C[1][k] * 256 + C[0][k]));
    const float2 sc2 = __ldg(reinterpret_cast<const float2*>(sc_) + t);
    // scales (top nibble of word p): p = 0 (g, 2t), 1 (g+8, 2t), 2 (g, 2t+1), 3 (g+8, 2t+1)
    const float kg0 = 0.5f * (0.5f + u23f(SS.x >> 28));
    const float k80 = 0.5f * (0.5f + u23f(SS.y >> 28));
    const float kg1 = 0.5f * (0.5f + u23f(SS.z >> 28));
    const float k81 = 0.5f * (0.5f + u23f(SS.w >> 28));
    y0 = fmaf(dg, fmaf(kg0 * sc2.x, T[0], kg1 * sc2.y * T[1]), y0);
    y8 = fmaf(d8, fmaf(k80 * sc2.x, T[2], k81 * sc2.y * T[3]), y8);
}

// IQ2_S: value = d * (0.5 + s) / 4 * grid[q] * sign with a 4-bit s per 16
// values (gguf quants.py IQ2_S); two sets of 8 sixteen-value blocks as Q6_K.
// A grid entry (1024 entries of 8 magnitudes 8..43, shared memory) covers
// chunks 2q and 2q + 1 of one register: one 64-bit load feeds two registers.
__shared__ unsigned long long s_iq2s_grid[1024];

template <class W, class X>
__device__ __forceinline__ void group_dot_iq2s(const uint8_t* gb, const uint8_t* fb, int fc,
                                               const float* __restrict__ sc_, int lane, int g, int t, float& y0,
                                               float& y8) {
    const uint4 IL = W::q(gb + lane * 16);
    const uint4 SG = W::q(gb + 512 + lane * 16);
    const uint32_t qh = W::w(gb + 1024 + 4 * lane);
    const uint32_t scw = W::w(gb + 1152 + 4 * lane);
    const float dg = h2f(W::h(gb + 1280 + 2 * g));
    const float d8 = h2f(W::h(gb + 1280 + 2 * (g + 8)));
#pragma unroll
    for (int st = 0; st < 2; ++st) {
        int C[3][4];
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int k = 0; k < 4; ++k) C[p][k] = 0;
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
            const int q = 2 * st + qq;
            const uint32_t il = word(IL, q), sg = word(SG, q);
            uint32_t lo[4], hi[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t idx = ((il >> (8 * k)) & 0xFFu) | (((qh >> (2 * (4 * q + k))) & 3u) << 8);
                const unsigned long long gv = s_iq2s_grid[idx];
                const uint32_t sb = (sg >> (8 * k)) & 0xFFu;
                lo[k] = signed4(static_cast<uint32_t>(gv), sb & 0xFu);
                hi[k] = signed4(static_cast<uint32_t>(gv >> 32), sb >> 4);
            }
            uint4 r2;  // plane 2 of the chunk pair (c = 4 st + 2 qq, + 1)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int c = 4 * st + 2 * qq + h;
                uint4 bq;
                uint2 br;
                load_b<X>(fb, c, fc, bq, br, r2);
                const uint32_t* a = h ? hi : lo;
                mma_s8s8(C[0], a[0], a[1], a[2], a[3], bq.x, bq.y);
                mma_s8s8(C[1], a[0], a[1], a[2], a[3], bq.z, bq.w);
                mma_s8s8(C[2], a[0], a[1], a[2], a[3], br.x, br.y);
            }
        }
        // |sum| <= 16 * 43 * 2^23 passes 2^31: join the planes in F32
        float T[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            T[k] = fmaf(static_cast<float>(C[2][k]), 65536.0f, static_cast<float>(C[1][k] * 256 + C[0][k]));
        const float2 sc2 = reinterpret_cast<const float2*>(sc_ + 8 * st)[t];
        // nibble 4 st + 2 h + b: row g + 8 h, block 8 st + 2 t + b
        const uint32_t n = scw >> (16 * st);
        const float kg0 = 0.25f * (0.5f + u23f(n & 0xFu));
        const float kg1 = 0.25f * (0.5f + u23f((n >> 4) & 0xFu));
        const float k80 = 0.25f * (0.5f + u23f((n >> 8) & 0xFu));
        const float k81 = 0.25f * (0.5f + u23f((n >> 12) & 0xFu));
        y0 = fmaf(dg, fmaf(kg0 * sc2.x, T[0], kg1 * sc2.y * T[1]), y0);
        y8 = fmaf(d8, fmaf(k80 * sc2.x, T[2], k81 * sc2.y * T[3]), y8);
    }
}

// Q4_0, Q4_K, Q5_K: one set of 8 thirty-two-value blocks, 4- or 5-bit q.
template <int TYPE, class W, class X>
__device__ __forceinline__ void group_dot_nib(const uint8_t* gb, const uint8_t* fb, int fc,
                                              const float* __restrict__ sc_, const float* __restrict__ xs_, int lane,
                                              int g, int t, float& y0, float& y8) {
    uint4 A[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] = W::q(gb + (i * 32 + lane) * 16);
    uint4 h0, h8, H;
    uint2 d4;
    if (TYPE == T_Q5_K) H = W::q(gb + 2048 + lane * 16);  // fifth bits
    if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        h0 = W::q(gb + kHeaderOff<TYPE> + 16 * g);
        h8 = W::q(gb + kHeaderOff<TYPE> + 16 * (g + 8));
    } else {
        d4 = W::d(gb + 2048 + 8 * lane);
    }
    int C[3][4];
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int k = 0; k < 4; ++k) C[p][k] = 0;
    uint4 r2;  // plane 2 of the current chunk pair
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 q;
        uint2 r;
        load_b<X>(fb, c, fc, q, r, r2);
        const uint32_t w0 = word(A[c >> 1], 2 * (c & 1)), w1 = word(A[c >> 1], 2 * (c & 1) + 1);
        uint32_t a0, a1, a2, a3;
        if (TYPE == T_Q5_K) {
            // 5-bit q: the fifth bit of register k sits at bit 4 (+k) or 0 (+k)
            // of each byte of the chunk pair's plane word
            const uint32_t hw = word(H, c >> 1);
            const uint32_t e0 = (c & 1) ? (hw << 4) : hw, e1 = (c & 1) ? (hw << 3) : (hw >> 1);
            const uint32_t e2 = (c & 1) ? (hw << 2) : (hw >> 2), e3 = (c & 1) ? (hw << 1) : (hw >> 3);
            a0 = (w0 & 0x0F0F0F0Fu) | (e0 & 0x10101010u);
            a1 = ((w0 >> 4) & 0x0F0F0F0Fu) | (e1 & 0x10101010u);
            a2 = (w1 & 0x0F0F0F0Fu) | (e2 & 0x10101010u);
            a3 = ((w1 >> 4) & 0x0F0F0F0Fu) | (e3 & 0x10101010u);
        } else {
            // rows g+8 stay in the high nibble: A = 16 q, undone in the combine below
            a0 = w0 & 0x0F0F0F0Fu;
            a1 = w0 & 0xF0F0F0F0u;
            a2 = w1 & 0x0F0F0F0Fu;
            a3 = w1 & 0xF0F0F0F0u;
        }
        mma_u8s8(C[0], a0, a1, a2, a3, q.x, q.y);
        mma_u8s8(C[1], a0, a1, a2, a3, q.z, q.w);
        mma_u8s8(C[2], a0, a1, a2, a3, r.x, r.y);
    }
    // C[p][0]: (row g, block 2t)  [1]: (g, 2t+1)  [2]: (g+8, 2t)  [3]: (g+8, 2t+1).
    // Rows g: |sum| <= 32 * 15 * (64 * 65536 + 128 * 257) < 2^31.  Rows g+8
    // carry a factor 16 in every plane (C0 a multiple of 16, so >> 4 is exact);
    // |C2| <= 32 * 240 * 64, so C2 * 4096 < 2^31 as well.
    float T[4];
    if (TYPE == T_Q5_K) {
        // |sum| can reach 32 * 31 * 2^22 > 2^31: join the planes in F32 (the
        // C2 term and the C1/C0 part are each exact; one rounding in the add)
#pragma unroll
        for (int k = 0; k < 4; ++k)
            T[k] = fmaf(static_cast<float>(C[2][k]), 65536.0f, static_cast<float>(C[1][k] * 256 + C[0][k]));
    } else {
        T[0] = static_cast<float>(C[2][0] * 65536 + C[1][0] * 256 + C[0][0]);
        T[1] = static_cast<float>(C[2][1] * 65536 + C[1][1] * 256 + C[0][1]);
        T[2] = static_cast<float>(C[2][2] * 4096 + C[1][2] * 16 + (C[0][2] >> 4));
        T[3] = static_cast<float>(C[2][3] * 4096 + C[1][3] * 16 + (C[0][3] >> 4));
    }
    const float2 sc2 = __ldg(reinterpret_cast<const float2*>(sc_) + t);
    const float2 xs2 = __ldg(reinterpret_cast<const float2*>(xs_) + t);
    const float s0 = sc2.x, s1 = sc2.y, x0 = xs2.x, x1 = xs2.y;
    if (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        // six-bit scales / mins of sub-blocks 2t, 2t+1 (kquants.h:204-212), four
        // per word; byte k of a word becomes a float as 2^23 + byte (prmt into
        // the exponent 0x4B) less 2^23, exactly, without the conversion pipe
        const uint32_t sel = 0x7540u | (2u * static_cast<uint32_t>(t & 1));
        float sc[2][2], mn[2][2], d[2], dm[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 hh = h ? h8 : h0;
            const uint32_t scw = t < 2 ? (hh.y & 0x3F3F3F3Fu) : ((hh.w & 0x0F0F0F0Fu) | ((hh.y >> 2) & 0x30303030u));
            const uint32_t mw = t < 2 ? (hh.z & 0x3F3F3F3Fu)
                                      : (((hh.w >> 4) & 0x0F0F0F0Fu) | ((hh.z >> 2) & 0x30303030u));
            sc[h][0] = __int_as_float(prmt(scw, 0x4B000000u, sel)) - 8388608.0f;
            sc[h][1] = __int_as_float(prmt(scw, 0x4B000000u, sel + 1)) - 8388608.0f;
            mn[h][0] = __int_as_float(prmt(mw, 0x4B000000u, sel)) - 8388608.0f;
            mn[h][1] = __int_as_float(prmt(mw, 0x4B000000u, sel + 1)) - 8388608.0f;
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

template <int TYPE, class W = LdGlobal, class X = LdGlobal>
__device__ __forceinline__ void group_dot(const uint8_t* gb, const uint8_t* fb, int fc, const float* __restrict__ sc_,
                                          const float* __restrict__ xs_, int lane, int g, int t, float& y0,
                                          float& y8) {
    if constexpr (TYPE == T_Q6_K)
        group_dot_q6k<W, X>(gb, fb, fc, sc_, xs_, lane, g, t, y0, y8);
    else if constexpr (TYPE == T_Q3_K)
        group_dot_q3k<W, X>(gb, fb, fc, sc_, xs_, lane, g, t, y0, y8);
    else if constexpr (TYPE == T_IQ4_XS)
        group_dot_iq4xs<W, X>(gb, fb, fc, sc_, lane, g, t, y0, y8);
    else if constexpr (TYPE == T_IQ3_S)
        group_dot_iq3s<W, X>(gb, fb, fc, sc_, lane, g, t, y0, y8);
    else if constexpr (TYPE == T_IQ3_XXS)
        group_dot_iq3xxs<W, X>(gb, fb, fc, sc_, lane, g, t, y0, y8);
    else if constexpr (TYPE == T_IQ2_S)
        group_dot_iq2s<W, X>(gb, fb, fc, sc_, lane, g, t, y0, y8);
    else
        group_dot_nib<TYPE, W, X>(gb, fb, fc, sc_, xs_, lane, g, t, y0, y8);
}

// Bounded waits of the shared-memory rings: 2 s of %globaltimer.
constexpr uint64_t kBulkWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bounded wait for the completion of the barrier phase with parity `parity`;
// false when it runs out or *abort (if given) is set.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 255u) == 0) {
            const uint64_t now = global_ns();
            if (i == 0) t0 = now;
            else if ((abort && *abort) || now - t0 > kBulkWaitNs) return false;
        }
    }
}
// Global -> shared bulk copy completing on `bar` (16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Per-warp shared-memory ring of gemv_mma_kernel's ring variant: depth (in
// units) per format, sized so that the 24 warps' rings take about 170 KiB.
template <int TYPE>
constexpr int kRingDepth = (170 * 1024 - kGridSmem<TYPE>) / (kWarps * kUnitBytes<TYPE>) > 4
                               ? 4
                               : ((170 * 1024 - kGridSmem<TYPE>) / (kWarps * kUnitBytes<TYPE>) < 1
                                      ? 1
                                      : (170 * 1024 - kGridSmem<TYPE>) / (kWarps * kUnitBytes<TYPE>));
// Bytes of the ring variant's dynamic shared memory after the partial rows
// and tile counters (offset `off`): the rings, then their barriers.
template <int TYPE>
constexpr size_t ring_bytes() {
    return size_t(kWarps) * kRingDepth<TYPE> * kUnitBytes<TYPE> + size_t(kWarps) * kRingDepth<TYPE> * 8;
}
__host__ __device__ constexpr size_t ring_offset(int cta_tiles) {
    return (size_t(kWarps) * 2 * MMA_TILE_ROWS * sizeof(float) + size_t(cta_tiles) * sizeof(int) + 127) & ~size_t(127);
}

// After a warp has written all 16 rows of `tile`: if the tile feeds the next
// launch, count it in at its 32-value chunk; the second of the chunk's two
// tiles (in any CTA) prepares the chunk as the x-preparation kernel would.
// Called once per emitted tile and kept out of line, so that it adds nothing
// to the register budget of the streaming loop.
__device__ __noinline__ void feed_next(uint8_t* frags, float* scale, float* xsum, int* chunk, const float* y, int lt,
                                      int bl, int lane, int64_t ch0, const PeerDest pd) {
    const int ch = lt >> 1;  // lt: the tile's index within the feeding output
    if (warp_count_in(chunk + ch) == 0) return;
    const float v = __ldcg(y + int64_t(ch) * 32 + lane);
    if (bl == 16)
        prep_x32<16>(v, ch0 + ch, lane, frags, scale, xsum, pd);
    else
        prep_x32<32>(v, ch0 + ch, lane, frags, scale, xsum, pd);
}

// kTiles: tile mode (a compile-time choice, so the unit-mode kernel carries
// none of its code).  kRing: the weights reach each warp through its own
// shared-memory ring instead of streaming loads: lane 0 requests the warp's
// next units with bulk copies (cp.async.bulk, completing on one mbarrier per
// slot) kRingDepth units ahead, the first ones before the programmatic-launch
// wait, and the warp reads each unit from shared memory once its barrier
// completes.  Everything else (split, combine, epilogue) is the same.
template <int TYPE, bool kTiles, bool kRing = false>
__global__ void __launch_bounds__(kGemvThreads, kCtasPerSm) gemv_mma_kernel(const GemvArgs a) {
    // unit, tile and group counts fit in 32 bits (the launcher checks)
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int U = static_cast<int>(a.units), NW = static_cast<int>(a.nwarps), ng = static_cast<int>(a.ngroups);
    const Split sp{U, ng, NW, kTiles ? U / ng : 1, static_cast<int>(gridDim.x)};  // tile mode only
    const int w = static_cast<int>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    const int u0 = kTiles ? sp.warp_unit0(w) : (w < NW ? static_cast<int>(int64_t(w) * U / NW) : 0);
    const int u1 = kTiles ? sp.warp_unit0(w + 1) : (w < NW ? static_cast<int>(int64_t(w + 1) * U / NW) : 0);
    // shared memory: per-warp partial rows (2 slots) and one arrival counter
    // per tile this CTA touches, counted from t0, the tile of its first unit
    extern __shared__ __align__(128) float s_part[];
    int* s_count = reinterpret_cast<int*>(s_part + kWarps * 2 * MMA_TILE_ROWS);
    const int t0 = kTiles ? sp.cta_unit0(static_cast<int>(blockIdx.x)) / ng
                          : static_cast<int>(int64_t(blockIdx.x) * kWarps * U / NW) / ng;
    for (int i = threadIdx.x; i < a.cta_tiles; i += blockDim.x) s_count[i] = 0;
    constexpr int UB = kUnitBytes<TYPE>;
    constexpr int D = kRing ? kRingDepth<TYPE> : 1;
    __shared__ int s_abort;
    uint8_t* ring = nullptr;
    uint64_t* rbar = nullptr;
    if constexpr (kRing) {
        uint8_t* rb = reinterpret_cast<uint8_t*>(s_part) + ring_offset(a.cta_tiles);
        const int wi = threadIdx.x >> 5;
        ring = rb + size_t(wi) * D * UB;
        rbar = reinterpret_cast<uint64_t*>(rb + size_t(kWarps) * D * UB) + wi * D;
        if (lane == 0) {
            for (int i = 0; i < D; ++i) mbar_init(rbar + i, 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        if (threadIdx.x == 0) s_abort = 0;
    }
    if constexpr (TYPE == T_IQ3_S)
        for (int i = threadIdx.x; i < 512 * kIq3sCopies; i += blockDim.x) s_iq3s_grid[i] = kIq3sGrid[i / kIq3sCopies];
    if constexpr (TYPE == T_IQ3_XXS)
        for (int i = threadIdx.x; i < 256 * kIq3xxsCopies; i += blockDim.x)
            s_iq3xxs_grid[i] = kIq3xxsGrid[i / kIq3xxsCopies];
    if constexpr (TYPE == T_IQ2_S)
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) s_iq2s_grid[i] = kIq2sGrid[i];
    __syncthreads();
    // fetch cursor of the ring (lane 0): the next unit to request, its
    // address, and the units left in its matrix from there on
    int fu = u0;
    const uint8_t* faddr = nullptr;
    int fleft = 0;
    auto request = [&](int slot) {
        if (fleft == 0) {
            const int ft = fu / ng;
            const SegRef sr = seg_ref(a, ft);
            faddr = sr.W + (int64_t(ft - static_cast<int>(sr.first_tile)) * ng + (fu - ft * ng)) * UB;
            fleft = static_cast<int>(sr.end_tile) * ng - fu;
        }
        mbar_arrive_tx(rbar + slot, UB);
        bulk_g2s(ring + slot * UB, faddr, UB, rbar + slot);
        if (fleft > 3) prefetch_l2(faddr + 3 * UB, UB);  // keep DRAM a few units ahead of the copies
        ++fu;
        faddr += UB;
        --fleft;
    };
    if constexpr (kRing) {
        // the warp's first units: weights are never written by the kernels this one overlaps
        if (lane == 0)
            for (int d = 0; d < D && fu < u1; ++d) request(d);
    } else {
        // start this warp's first weights towards L2 before waiting on xprep
        if (lane == 0)
            for (int d = 0; d < kPrefetch && u0 + d < u1; ++d)
                prefetch_l2(unit_weights<TYPE>(a, u0 + d), kUnitBytes<TYPE>);
    }
    pdl_release();
    pdl_wait();  // x digits and the zeroed tile counters come from xprep_kernel (or the previous launch)
    uint32_t xe = 0;  // sharded: this launch's epoch and exchange data half
    int64_t hoff = 0;
    if (a.xchg) {
        xe = __ldcg(a.x.epoch) + 1u;
        hoff = (xe & 1u) ? a.x.half_floats : 0;
    }
    if (a.f_bl != 0) {
        // what the x-preparation kernel would clear for the next launch; its
        // scratch slot's previous user has completed (this launch waited on it)
        const int64_t gt = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
        for (int64_t i = gt; i < a.f_ncount; i += int64_t(gridDim.x) * blockDim.x) a.f_count[i] = 0;
        for (int64_t i = gt; i < kZeroBytes / 4; i += int64_t(gridDim.x) * blockDim.x) a.f_zeros[i] = 0u;
    }
    if (a.wait_peers) {
        // Sharded chain: part of this launch's x was prepared by the peers
        // (their rows of the previous launch's output).  Their flags of the
        // previous epoch cover those stores; the wait is bounded and a
        // time-out is reported through the exchange's error word.
        __shared__ int s_peers_ok;
        if (threadIdx.x == 0) {
            int ok = 1;
            const uint32_t* fl = a.x.peer_flags[a.x.rank];
            const uint64_t w0 = global_ns();
            for (int p = 0; p < a.x.world && ok; ++p) {
                if (p == a.x.rank) continue;
                while (static_cast<int32_t>(ld_acquire_sys(fl + p) - (xe - 1u)) < 0) {
                    if (global_ns() - w0 > kGatherWaitNs) {
                        ok = 0;
                        atomicExch(a.x.err, 1);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            s_peers_ok = ok;
        }
        __syncthreads();
        if (s_peers_ok) {
            // the previous launch's peer rows -> its full outputs (this GPU's
            // exchange data of the previous epoch)
            const float* xd = a.x.peer_data[a.x.rank] + (((xe - 1u) & 1u) ? a.x.half_floats : 0);
            const int64_t gt = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
            const int64_t stride = int64_t(gridDim.x) * blockDim.x;
            for (int sg = 0; sg < a.nprev; ++sg) {
                const GatherSeg ps = a.prev[sg];
                const int64_t n_peers = ps.n_local * a.x.world;
                for (int64_t i = gt; i < n_peers; i += stride) {
                    if (i / ps.n_local == a.x.rank) continue;  // own rows: written by the previous launch
                    ps.y_full[i] = __ldcg(xd + ps.xo + i);
                }
            }
        }
    }

    const bool supplier = g == t || g == t + 4;
    const uint8_t* fb0 = supplier ? a.frags + g * kSlotBytes : a.zeros;
    constexpr int fc = kChunkFragBytes;  // the zero lanes step through kZeroBytes of zeros
    const int fg = supplier ? kGroupFragBytes : 0;
    int u = u0;
    int j = 0;  // units this warp has consumed (ring slot and phase)
    bool ok = true;
    while (u < u1) {
        const int tile = u / ng, tbeg = tile * ng;
        const int gend = (u1 - tbeg) < ng ? (u1 - tbeg) : ng;
        const uint8_t* tw;
        int pf_end;  // a matrix's tiles are contiguous: prefetch ahead up to its last unit
        {
            const SegRef sr = seg_ref(a, tile);
            tw = sr.W + static_cast<int64_t>(tile - static_cast<int>(sr.first_tile)) * ng * kUnitBytes<TYPE>;
            pf_end = (static_cast<int>(sr.end_tile) - tile) * ng;
        }
        float y0 = 0.f, y8 = 0.f;
        for (int gi = u - tbeg; gi < gend; ++gi) {
            if constexpr (kRing) {
                const int slot = j % D;
                if (!mbar_wait(rbar + slot, static_cast<uint32_t>(j / D) & 1u, &s_abort)) {
                    ok = false;
                    break;
                }
                group_dot<TYPE, LdShared, LdGlobal>(ring + slot * UB, fb0 + gi * fg, fc, a.scale + gi * kXBlocks<TYPE>,
                                                    a.xsum + gi * kXBlocks<TYPE>, lane, g, t, y0, y8);
                __syncwarp();  // every lane has read the slot: refill it
                if (lane == 0 && fu < u1) request(slot);
                ++j;
            } else {
                if (lane == 0 && tbeg + gi + kPrefetch < u1 && gi + kPrefetch < pf_end)
                    prefetch_l2(tw + (gi + kPrefetch) * kUnitBytes<TYPE>, kUnitBytes<TYPE>);
                group_dot<TYPE>(tw + gi * kUnitBytes<TYPE>, fb0 + gi * fg, fc, a.scale + gi * kXBlocks<TYPE>,
                                a.xsum + gi * kXBlocks<TYPE>, lane, g, t, y0, y8);
            }
        }
        if (!ok) break;
        y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
        y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
        float* ty;  // looked up again here so that nothing extra stays live in the loop above
        {
            const SegRef sr = seg_ref(a, tile);
            ty = sr.y + (tile - static_cast<int>(sr.first_tile)) * MMA_TILE_ROWS;
        }
        bool emitted = false;  // this warp wrote the tile's 16 rows (warp-uniform)
        if (u == tbeg && gend == ng) {  // the whole tile is this warp's
            if (t == 0) {
                emit(a, ty, tile, g, y0, hoff);
                emit(a, ty, tile, g + 8, y8, hoff);
            }
            emitted = true;
        } else {
            // the tile's contributors are global warps wa..wb; this CTA holds lo..hi of them
            const int wa = kTiles ? sp.warp_of_unit(tbeg) : static_cast<int>(warp_of(tbeg, U, NW));
            const int wb = kTiles ? sp.warp_of_unit(tbeg + ng - 1) : static_cast<int>(warp_of(tbeg + ng - 1, U, NW));
            const int cta = static_cast<int>(blockIdx.x);
            const int lo = wa > cta * kWarps ? wa : cta * kWarps;
            const int hi = wb < cta * kWarps + kWarps - 1 ? wb : cta * kWarps + kWarps - 1;
            const int slot_a = (kTiles ? sp.warp_unit0(wa) : static_cast<int>(int64_t(wa) * U / NW)) < tbeg
                                   ? 1 : 0;  // wa's last tile, else its first
            // level 1: partial rows to shared memory; the CTA's last contributor adds them
            float* mine = s_part + ((w - cta * kWarps) * 2 + (u == u0 ? 0 : 1)) * MMA_TILE_ROWS;
            if (t == 0) {
                mine[g] = y0;
                mine[g + 8] = y8;
            }
            __threadfence_block();
            __syncwarp();
            int prev = 0;
            if (lane == 0) prev = atomicAdd(s_count + (tile - t0), 1);
            prev = __shfl_sync(0xffffffffu, prev, 0);
            if (prev == hi - lo) {
                __threadfence_block();
                const int r = lane & 15;
                float acc = 0.f;
                for (int v = lo; v <= hi; ++v)  // warp order
                    acc += s_part[((v - cta * kWarps) * 2 + (v == wa ? slot_a : 0)) * MMA_TILE_ROWS + r];
                const int ca = wa / kWarps, cb = wb / kWarps;
                if (ca == cb) {  // every contributor was in this CTA
                    if (lane < MMA_TILE_ROWS) emit(a, ty, tile, r, acc, hoff);
                    emitted = true;
                } else {
                    // level 2: the CTA's sum to global memory; the last CTA adds them in CTA order.
                    // A CTA shares at most two tiles with others: its first (slot 0) and last (slot 1).
                    if (lane < MMA_TILE_ROWS) a.partial[(cta * 2 + (tile == t0 ? 0 : 1)) * MMA_TILE_ROWS + r] = acc;
                    const int gprev = warp_count_in(a.count + tile);
                    if (gprev == cb - ca) {
                        // lane (row r, half h) adds CTAs ca + h, ca + h + 2, ..., eight loads in flight
                        const int h = lane >> 4;
                        // CTA ca's first tile (unit mode only: in tile mode no tile spans CTAs)
                        const int t0a = static_cast<int>(int64_t(ca * kWarps) * U / NW) / ng;
                        float sum = 0.f;
                        for (int c0 = ca + h; c0 <= cb; c0 += 16) {
                            float part[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const int c = c0 + 2 * j;
                                const int which = (c == ca && t0a != tile) ? 1 : 0;
                                part[j] = c <= cb ? __ldcg(a.partial + (c * 2 + which) * MMA_TILE_ROWS + r) : 0.f;
                            }
#pragma unroll
                            for (int j = 0; j < 8; ++j) sum += part[j];
                        }
                        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
                        if (h == 0) emit(a, ty, tile, r, sum, hoff);
                        emitted = true;
                    }
                }
            }
        }
        if (emitted && a.f_bl != 0 && tile >= a.f_t0 && tile < a.f_t1)
            feed_next(a.f_frags, a.f_scale, a.f_xsum, a.f_chunk, a.f_y, static_cast<int>(tile - a.f_t0), a.f_bl, lane, a.f_ch0,
                      PeerDest{a.f_pbase, a.x.world, a.x.rank});
        u = tbeg + gend;
    }
    if constexpr (kRing) {
        if (!ok) {
            // a ring wait ran out (never expected): report it, let the copies
            // still in flight into this warp's slots land (bounded), and leave
            // this launch's outputs incomplete rather than hang
            if (lane == 0) {
                atomicExch(a.err, 1);
                s_abort = 1;
                for (int k = j; k < fu - u0; ++k) mbar_wait(rbar + k % D, static_cast<uint32_t>(k / D) & 1u, nullptr);
            }
            __syncwarp();
        }
    }
    if (a.xchg) {
        // Every row this CTA stored (locally and into the peers' buffers) is
        // ordered before its count-in at device scope; the last CTA to count
        // in then fences at system scope, which, being cumulative over what it
        // observed through the counter, orders all CTAs' stores before this
        // rank's flag in each peer's flag array.  (A system-scope fence in
        // every CTA cost about 8 us per launch; a fence per peer flag, on top
        // of an explicit one, about 1.7 us more at N = 2.)
        __syncthreads();
        if (threadIdx.x == 0) {
            if (atom_add_acq_rel_gpu(a.done, 1) == static_cast<int>(gridDim.x) - 1) {
                raise_peer_flags(a.x, xe);
                *a.x.epoch = xe;  // every CTA has read e - 1 (before counting in)
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Bulk-copy GEMV: the weights reach shared memory through the TMA unit
// (cp.async.bulk into an mbarrier-tracked ring), issued by one producer thread
// ahead of kCons consumer warps.  One CTA per SM.
//
// Work split.  Split mode (a tile has at least kCons groups): CTA c takes the
// contiguous unit range [c U / G, (c + 1) U / G), walked in pieces of up to
// kCons units that never cross a tile; consumer warp w computes unit w of
// each piece and keeps its rows' sums in registers across the pieces of one
// tile.  After the CTA's last piece of a tile every warp writes its 16 partial
// rows to shared memory, and one warp adds them in warp order: a tile wholly
// inside the CTA's range is written out; a tile shared with neighbouring CTAs
// (only a CTA's first and last tile can be) goes through the two-slot
// cross-CTA combine of gemv_mma_kernel, the last CTA adding the CTAs' sums in
// CTA order.  Whole-tile mode (fewer groups, kCons a multiple of the count):
// CTA c takes tiles [c T / G, (c + 1) T / G), kCons / ngroups tiles per
// piece, and tile j of a piece is warps j ngroups .. (j + 1) ngroups - 1.
// Every addition happens in an order fixed by the shape, so results are
// deterministic.
//
// Overlap.  The producer requests the first `stages` pieces before the
// programmatic-launch wait (weights are never written by the kernels this
// one overlaps), so a launch's first bytes stream in while the previous
// kernel drains.  In the staged-x variant each stage also carries the
// piece's x fragments, copied after the wait.
//
// Every wait is bounded (2 s of %globaltimer); a wait that runs out sets the
// error word and ends the CTA's work instead of hanging.
// ---------------------------------------------------------------------------
constexpr int kCons = 16;
constexpr int kBulkThreads = (kCons + 1) * 32;

struct BulkArgs {
    int whole;        // whole-tile mode
    int stages;       // ring depth
    int stage_bytes;  // one stage: kCons units of weights (+ their x fragments when staged)
    int* err;         // set when a bounded wait runs out
};

// Shared-memory layout of the bulk kernel after the ring (the host sizes it
// with the same arithmetic): the barriers full[S], empty[S], ready[2] and
// freed[2] and fin, two ints of piece description per stage, two sets of
// per-warp partial rows, a zero slot and the abort flag.
__host__ __device__ constexpr size_t bulk_bars_off(int S, int stage_bytes) { return size_t(S) * stage_bytes; }
__host__ __device__ constexpr size_t bulk_part_off(int S, int stage_bytes) {
    return (bulk_bars_off(S, stage_bytes) + 8 * (2 * size_t(S) + 5) + 8 * size_t(S) + 15) & ~size_t(15);
}
__host__ __device__ constexpr size_t bulk_smem_bytes(int S, int stage_bytes) {
    return bulk_part_off(S, stage_bytes) + 2 * kCons * MMA_TILE_ROWS * sizeof(float) + kSlotBytes + 16;
}

// CTA of a grid of G whose unit range [c U / G, (c + 1) U / G) holds unit u.
__device__ __forceinline__ int cta_of_unit(int64_t u, int64_t U, int G) {
    return static_cast<int>(((u + 1) * G + U - 1) / U - 1);
}

template <int TYPE, bool kXS>
__global__ void __launch_bounds__(kBulkThreads, 1) gemv_bulk_kernel(const GemvArgs a, const BulkArgs b) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int UB = kUnitBytes<TYPE>;
    const int S = b.stages, SB = b.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + bulk_bars_off(S, SB));
    uint64_t* empty = full + S;
    uint64_t* ready = empty + S;  // [2]: the warps' partial rows of a tile are written
    uint64_t* freed = ready + 2;  // [2]: every warp is done with those partial rows
    uint64_t* fin = freed + 2;    // every consumer warp has left its loop
    int* s_meta = reinterpret_cast<int*>(fin + 1);  // per stage: first tile (-1: end), g0 | len << 16 | last << 31
    float* s_part = reinterpret_cast<float*>(smem + bulk_part_off(S, SB));
    uint32_t* s_zero = reinterpret_cast<uint32_t*>(s_part + 2 * kCons * MMA_TILE_ROWS);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_zero + kSlotBytes / 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int ng = static_cast<int>(a.ngroups);
    const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
    const int64_t U = a.units, T = U / ng;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kCons);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(ready + i, kCons);
            mbar_init(freed + i, kCons);
        }
        mbar_init(fin, kCons);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kSlotBytes / 4) s_zero[threadIdx.x] = 0u;
    if constexpr (TYPE == T_IQ3_S)
        for (int i = threadIdx.x; i < 512 * kIq3sCopies; i += blockDim.x) s_iq3s_grid[i] = kIq3sGrid[i / kIq3sCopies];
    if constexpr (TYPE == T_IQ3_XXS)
        for (int i = threadIdx.x; i < 256 * kIq3xxsCopies; i += blockDim.x)
            s_iq3xxs_grid[i] = kIq3xxsGrid[i / kIq3xxsCopies];
    if constexpr (TYPE == T_IQ2_S)
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) s_iq2s_grid[i] = kIq2sGrid[i];
    __syncthreads();
    pdl_release();

    // this CTA's work: units [u0, u1) (split mode) or tiles [t0, t1) (whole-tile mode)
    const int64_t u0 = b.whole ? (int64_t(cta) * T / G) * ng : int64_t(cta) * U / G;
    const int64_t u1 = b.whole ? (int64_t(cta + 1) * T / G) * ng : int64_t(cta + 1) * U / G;

    if (warp == kCons) {
        // ------------------------------------------------------- producer
        if (lane != 0) return;
        int it = 0;
        bool waited = !kXS;  // only the staged-x copies depend on the previous kernel
        // after the dependency wait: the x copies and arrivals of the first n
        // pieces, whose weights were requested before it (staged-x variant)
        auto after_wait = [&](int n) {
            pdl_wait();
            waited = true;
            for (int i = 0; i < n; ++i) {
                const int m = s_meta[2 * i + 1];
                const int g0 = m & 0xFFFF, len = (m >> 16) & 0x7FFF;
                const uint32_t xbytes = static_cast<uint32_t>((b.whole ? ng : len) * kGroupFragBytes);
                mbar_arrive_tx(full + i, xbytes);
                bulk_g2s(smem + size_t(i) * SB + kCons * UB, a.frags + int64_t(b.whole ? 0 : g0) * kGroupFragBytes,
                         xbytes, full + i);
            }
        };
        for (int64_t u = u0; u < u1; ++it) {
            const int64_t tile = u / ng;
            int len, g0 = static_cast<int>(u - tile * ng);
            bool last;
            if (b.whole) {
                len = static_cast<int>(u1 - u < kCons ? u1 - u : kCons);  // whole tiles: kCons is a multiple of ng
                last = true;
            } else {
                const int64_t tend = (tile + 1) * ng;
                const int64_t e = tend < u1 ? tend : u1;
                len = static_cast<int>(e - u < kCons ? e - u : kCons);
                last = u + len == e;
            }
            const int stage = it % S;
            if (it == S && !waited) after_wait(S);
            if (it >= S && !mbar_wait(empty + stage, static_cast<uint32_t>((it / S) - 1) & 1u, s_abort)) {
                atomicExch(b.err, 1);
                *s_abort = 1;
                return;
            }
            s_meta[2 * stage] = static_cast<int>(tile);
            s_meta[2 * stage + 1] = g0 | (len << 16) | (last ? int(0x80000000u) : 0);
            uint8_t* dst = smem + size_t(stage) * SB;
            const uint32_t wbytes = static_cast<uint32_t>(len * UB);
            const uint32_t xbytes = kXS ? static_cast<uint32_t>((b.whole ? ng : len) * kGroupFragBytes) : 0u;
            if (kXS && !waited) mbar_expect_tx(full + stage, wbytes);  // the x copy and the arrival come after the wait
            else mbar_arrive_tx(full + stage, wbytes + xbytes);
            // a piece's units are contiguous in memory unless it spans two matrices (whole-tile mode)
            int done = 0;
            while (done < len) {
                const int64_t tt = (u + done) / ng;
                const SegRef sr = seg_ref(a, tt);
                const int64_t seg_end_u = sr.end_tile * ng;
                const int n = static_cast<int>(u + len < seg_end_u ? len - done : seg_end_u - (u + done));
                bulk_g2s(dst + done * UB, sr.W + ((tt - sr.first_tile) * ng + (u + done - tt * ng)) * UB,
                         static_cast<uint32_t>(n * UB), full + stage);
                done += n;
            }
            if (kXS && waited)
                bulk_g2s(dst + kCons * UB, a.frags + int64_t(b.whole ? 0 : g0) * kGroupFragBytes, xbytes, full + stage);
            u += len;
        }
        if (!waited) after_wait(it);
        // end of the work: a stage whose tile is -1 (its previous use was released above)
        const int stage = it % S;
        if (it >= S && !mbar_wait(empty + stage, static_cast<uint32_t>((it / S) - 1) & 1u, s_abort)) {
            atomicExch(b.err, 1);
            *s_abort = 1;
            return;
        }
        s_meta[2 * stage] = -1;
        mbar_arrive(full + stage);
        return;
    }

    // ----------------------------------------------------------- consumers
    pdl_wait();  // x fragments, scales, sums and cleared counters are ready
    uint32_t xe = 0;
    int64_t hoff = 0;
    if (a.xchg) {
        xe = __ldcg(a.x.epoch) + 1u;
        hoff = (xe & 1u) ? a.x.half_floats : 0;
    }
    const int ctid = warp * 32 + lane;
    if (a.f_bl != 0) {
        const int64_t gt = int64_t(cta) * (kCons * 32) + ctid;
        for (int64_t i = gt; i < a.f_ncount; i += int64_t(G) * (kCons * 32)) a.f_count[i] = 0;
        for (int64_t i = gt; i < kZeroBytes / 4; i += int64_t(G) * (kCons * 32)) a.f_zeros[i] = 0u;
    }
    const bool supplier = g == t || g == t + 4;
    const int fc = supplier ? kChunkFragBytes : 0;
    const int64_t first_tile = u0 / ng;
    bool ok = true;
    float y0 = 0.f, y8 = 0.f;
    for (int it = 0, flush = 0;; ++it) {
        const int stage = it % S;
        if (!mbar_wait(full + stage, static_cast<uint32_t>(it / S) & 1u, s_abort)) {
            ok = false;
            break;
        }
        const int tile0 = s_meta[2 * stage];
        if (tile0 < 0) break;
        const int m = s_meta[2 * stage + 1];
        const int g0 = m & 0xFFFF, len = (m >> 16) & 0x7FFF;
        const bool last = m < 0;
        if (warp < len) {
            const uint8_t* st = smem + size_t(stage) * SB;
            const int gi = b.whole ? warp % ng : g0 + warp;
            const uint8_t* fb;
            if constexpr (kXS)
                fb = supplier ? st + kCons * UB + (b.whole ? gi : warp) * kGroupFragBytes + g * kSlotBytes
                              : reinterpret_cast<const uint8_t*>(s_zero);
            else
                fb = supplier ? a.frags + int64_t(gi) * kGroupFragBytes + g * kSlotBytes : a.zeros;
            group_dot<TYPE, LdShared, typename std::conditional<kXS, LdShared, LdGlobal>::type>(
                st + warp * UB, fb, fc, a.scale + int64_t(gi) * kXBlocks<TYPE>, a.xsum + int64_t(gi) * kXBlocks<TYPE>,
                lane, g, t, y0, y8);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + stage);  // this warp is done with the stage
        if (!last) continue;
        // ---- flush: the tile(s) of this piece end here for this CTA
        const int par = flush & 1;
        if (flush >= 2 && !mbar_wait(freed + par, static_cast<uint32_t>((flush >> 1) - 1) & 1u, s_abort)) {
            ok = false;
            break;
        }
        float* part = s_part + par * kCons * MMA_TILE_ROWS;
        y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
        y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
        if (t == 0) {
            part[warp * MMA_TILE_ROWS + g] = y0;
            part[warp * MMA_TILE_ROWS + g + 8] = y8;
        }
        y0 = y8 = 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(ready + par);
        const int r = lane & 15;
        const int ntc = b.whole ? (len + ng - 1) / ng : 1;  // tiles ending in this piece
        const int reducer = b.whole ? -1 : tile0 % kCons;
        float acc = 0.f;
        int my_tile = -1;  // the tile this warp reduces
        if (b.whole) {
            if (warp % ng == 0 && warp / ng < ntc) my_tile = tile0 + warp / ng;
        } else if (warp == reducer) {
            my_tile = tile0;
        }
        if (my_tile >= 0) {
            if (!mbar_wait(ready + par, static_cast<uint32_t>(flush >> 1) & 1u, s_abort)) {
                ok = false;
                break;
            }
            const int w0 = b.whole ? warp : 0, wn = b.whole ? ng : kCons;
            for (int v = w0; v < w0 + wn; ++v) acc += part[v * MMA_TILE_ROWS + r];  // warp order
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(freed + par);
        ++flush;
        if (my_tile < 0) continue;
        const SegRef sr = seg_ref(a, my_tile);
        float* ty = sr.y + (int64_t(my_tile) - sr.first_tile) * MMA_TILE_ROWS;
        bool emitted = false;
        const int64_t ts = int64_t(my_tile) * ng;
        if (b.whole || (ts >= u0 && ts + ng <= u1)) {  // the whole tile was this CTA's
            if (lane < MMA_TILE_ROWS) emit(a, ty, my_tile, r, acc, hoff);
            emitted = true;
        } else {
            // shared with neighbouring CTAs: the CTA's sum to its slot (0: its
            // first tile, 1: its last); the last CTA adds them in CTA order
            const int ca = cta_of_unit(ts, U, G), cb = cta_of_unit(ts + ng - 1, U, G);
            if (lane < MMA_TILE_ROWS)
                a.partial[(cta * 2 + (my_tile == first_tile ? 0 : 1)) * MMA_TILE_ROWS + r] = acc;
            const int prev = warp_count_in(a.count + my_tile);
            if (prev == cb - ca) {
                float sum = 0.f;
                if (lane < MMA_TILE_ROWS)
                    for (int c2 = ca; c2 <= cb; ++c2) {
                        const int64_t ft = (int64_t(c2) * U / G) / ng;  // CTA c2's first tile
                        sum += __ldcg(a.partial + (c2 * 2 + (ft == my_tile ? 0 : 1)) * MMA_TILE_ROWS + r);
                    }
                if (lane < MMA_TILE_ROWS) emit(a, ty, my_tile, r, sum, hoff);
                emitted = true;
            }
        }
        if (emitted && a.f_bl != 0 && my_tile >= a.f_t0 && my_tile < a.f_t1)
            feed_next(a.f_frags, a.f_scale, a.f_xsum, a.f_chunk, a.f_y, static_cast<int>(my_tile - a.f_t0), a.f_bl, lane, a.f_ch0,
                      PeerDest{a.f_pbase, a.x.world, a.x.rank});
    }
    if (!ok) {
        if (lane == 0) atomicExch(b.err, 1);
        *s_abort = 1;
        return;
    }
    if (a.xchg) {
        // as in gemv_mma_kernel: every row this CTA stored is ordered before
        // its count-in; the last CTA fences at system scope once and raises
        // the peers' flags
        __syncwarp();
        if (lane == 0) mbar_arrive(fin);
        if (ctid == 0) {
            if (!mbar_wait(fin, 0u, s_abort)) {
                atomicExch(b.err, 1);
                return;
            }
            if (atom_add_acq_rel_gpu(a.done, 1) == G - 1) {
                raise_peer_flags(a.x, xe);
                *a.x.epoch = xe;
            }
        }
    }
}

// Peers' rows -> the full outputs, after every peer's flag reached `epoch`.
// Launched with programmatic dependent launch: it first waits
// (griddepcontrol.wait) for this GPU's GEMV to complete, which also makes the
// GEMV's stored epoch visible, then polls the peers' flags, so the next kernel
// sees both halves of every output.  The flag wait is bounded (1 s of
// %globaltimer); on time-out *err is set and nothing is copied, so the host
// reports an error instead of the GPU hanging.
struct GatherArgs {
    GatherSeg seg[kMaxSegs];
    int nseg;
};
// Feed of a gather: the next launch's x is gathered segment f.seg in full.
struct GatherFeed {
    int seg, bl;  // bl = 0: no feed
    uint8_t* frags;
    float* scale;
    float* xsum;
    int* count;  // the next launch's counters (ncount ints) and zero slot, cleared here
    int64_t ncount;
    uint32_t* zeros;
};
__global__ void __launch_bounds__(256) xchg_gather_kernel(const float* __restrict__ xdata, int64_t half_floats,
                                                          const uint32_t* flags, const uint32_t* epoch, int world,
                                                          int rank, const GatherArgs g, int* err, const GatherFeed f) {
    __shared__ int s_ok;
    // The GEMV has finished and stored this launch's epoch; the gather does
    // not let the next kernel start early, so the counter stays e until then.
    pdl_wait();
    const uint32_t e = __ldcg(epoch);
    if (threadIdx.x == 0) {
        int ok = 1;
        const uint64_t t0 = global_ns();
        for (int p = 0; p < world && ok; ++p) {
            if (p == rank) continue;
            while (static_cast<int32_t>(ld_acquire_sys(flags + p) - e) < 0) {
                if (global_ns() - t0 > kGatherWaitNs) {
                    ok = 0;
                    atomicExch(err, 1);
                    break;
                }
                __nanosleep(32);
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const float* xd = xdata + ((e & 1u) ? half_floats : 0);
    const int64_t gt = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    if (f.bl != 0) {
        for (int64_t i = gt; i < f.ncount; i += stride) f.count[i] = 0;
        for (int64_t i = gt; i < kZeroBytes / 4; i += stride) f.zeros[i] = 0u;
    }
    for (int s = 0; s < g.nseg; ++s) {
        const GatherSeg sg = g.seg[s];
        if (f.bl != 0 && s == f.seg) {
            // one warp per 32 values of the full output: the peers' rows are
            // copied in, and the 32 values become the next launch's x digits
            const int lane = threadIdx.x & 31;
            const int64_t nch = sg.n_local * world / 32;
            for (int64_t ch = gt >> 5; ch < nch; ch += stride >> 5) {
                const int64_t r = ch * 32 + lane;
                const int p = static_cast<int>(r / sg.n_local);
                float v;
                if (p == rank) {
                    v = __ldcg(sg.y_full + r);
                } else {
                    v = __ldcg(xd + sg.xo + r);
                    sg.y_full[r] = v;
                }
                if (f.bl == 16)
                    prep_x32<16>(v, ch, lane, f.frags, f.scale, f.xsum);
                else
                    prep_x32<32>(v, ch, lane, f.frags, f.scale, f.xsum);
            }
            continue;
        }
        for (int p = 0; p < world; ++p) {
            if (p == rank) continue;  // own rows: written by the GEMV
            float* dst = sg.y_full + p * sg.n_local;
            const float* src = xd + sg.xo + p * sg.n_local;
            for (int64_t i = gt; i < sg.n_local; i += stride) dst[i] = __ldcg(src + i);
        }
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

// SM count of the current device, looked up once per device.  Entries are
// atomics, so launcher threads that race on the first lookup of a device
// store the same value without a data race.
static int sm_count() {
    static std::atomic<int> sms[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    int v = sms[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) return -1;
        sms[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

// Counters of a launch over `ntiles` tiles: one per tile, the CTA completion
// counter, and one per 32-value chunk of an output that feeds the next launch.
// All start at zero: cleared by the x-preparation kernel, or by the launch
// before when that one prepares x.
static int64_t counter_ints(int64_t ntiles) { return ntiles + 1 + ntiles / 2 + 1; }

// Scratch of one MMA GEMV launch (layout described above the kernels).
ScratchLayout scratch_layout(int64_t N, int64_t K) {
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    ScratchLayout L;
    const size_t ngroups = static_cast<size_t>(K / 256), nblk = static_cast<size_t>(K / 32);
    const size_t ntiles = static_cast<size_t>(N / MMA_TILE_ROWS);
    L.frags = 0;
    L.zeros = up(L.frags + ngroups * kGroupFragBytes);
    L.scale = up(L.zeros + kZeroBytes);
    L.xsum = up(L.scale + 2 * nblk * sizeof(float));  // room for 16-value blocks
    L.count = up(L.xsum + 2 * nblk * sizeof(float));
    L.partial = up(L.count + counter_ints(static_cast<int64_t>(ntiles)) * sizeof(int));
    L.total = up(L.partial + size_t(kMaxCtas) * 2 * MMA_TILE_ROWS * sizeof(float));
    return L;
}

size_t xprep_bytes(int64_t N, int64_t K) { return scratch_layout(N, K).total; }

size_t gemv_scratch_bytes(int64_t N, int64_t K) { return scratch_layout(N, K).total; }

// Which GEMV kernel serves MMA-layout launches: XDNA_B200_GEMV = "classic"
// (the default: gemv_mma_kernel with streaming loads and L2 prefetch),
// "ring" (gemv_mma_kernel with a per-warp shared-memory ring filled by bulk
// copies), "bulk" (gemv_bulk_kernel, x fragments through the L1) or "bulkx"
// (gemv_bulk_kernel with the x fragments staged beside the weights).  On
// B200 the classic kernel streams fastest (Q4_K 28672 x 8192: 3758 GB/s
// against 3532 ring, 2859 bulk and 3424 bulkx; the 70B decode step 10.39 ms
// against 11.52 ring and 15.34 bulkx), so the others are opt-in.  Read once
// per process.
static int gemv_kernel_choice() {
    static const int choice = [] {
        const char* v = getenv("XDNA_B200_GEMV");
        if (v && !strcmp(v, "ring")) return 3;
        if (v && !strcmp(v, "bulk")) return 1;
        if (v && !strcmp(v, "bulkx")) return 2;
        return 0;
    }();
    return choice;
}

// Error word of the bulk kernel's bounded waits on the current device.
static __device__ int g_gemv_err;
static int* gemv_err_ptr() {
    static std::mutex m;
    static int* addr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(m);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemv_err) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<int*>(p);
    }
    return addr[dev];
}

cudaError_t gemv_error_status(int* out) {
    int* p = gemv_err_ptr();
    if (!p) return cudaErrorInvalidDevice;
    int v = 0;
    cudaError_t e = cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && v) e = cudaMemset(p, 0, sizeof(int));
    *out = v;
    return e;
}

// The kernels that run between GEMVs (x preparation, gather) take the
// shared-memory carve-out of the large-shared-memory GEMV variants, so that an
// SM need not drain to switch it and the programmatic-launch overlap is kept.
static cudaError_t match_carveouts() {
    for (const void* f : {reinterpret_cast<const void*>(xprep_kernel<16>), reinterpret_cast<const void*>(xprep_kernel<32>),
                          reinterpret_cast<const void*>(xchg_gather_kernel)}) {
        const cudaError_t e =
            cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Launch plan of the bulk kernel for one launch, or false where it does not
// apply (a tile group count below kCons that does not divide it, or no room
// for two stages).
struct BulkPlan {
    BulkArgs b;
    int grid;
    size_t smem;
};
template <int TYPE>
static bool bulk_plan(bool staged_x, int64_t ngroups, int64_t ntiles, int sms, BulkPlan* p) {
    constexpr int UB = kUnitBytes<TYPE>;
    // shared memory per CTA (227 KiB) less the static grid table of the IQ formats
    constexpr size_t kGrid = kGridSmem<TYPE>;
    const size_t budget = 227 * 1024 - kGrid - 1024;
    BulkArgs& b = p->b;
    b = BulkArgs{};
    int64_t work;  // the units (split mode) or tiles (whole-tile mode) shared among the CTAs
    if (ngroups >= 32768) return false;  // a piece's first group is kept in 16 bits
    if (ngroups >= kCons) {
        b.whole = 0;
        work = ntiles * ngroups;
    } else if (ngroups > 0 && kCons % ngroups == 0) {
        b.whole = 1;
        work = ntiles;
    } else {
        return false;
    }
    b.stage_bytes = ((kCons * UB + (staged_x ? kCons * kGroupFragBytes : 0)) + 127) & ~127;
    int S = 8;
    while (S >= 2 && bulk_smem_bytes(S, b.stage_bytes) > budget) --S;
    if (S < 2) return false;
    b.stages = S;
    p->smem = bulk_smem_bytes(S, b.stage_bytes);
    p->grid = static_cast<int>(work < sms ? work : sms);
    return p->grid <= kMaxCtas;
}

template <int TYPE, bool kXS>
static cudaError_t launch_bulk_typed(cudaLaunchConfig_t& cg, const GemvArgs& a, const BulkArgs& b) {
    static std::atomic<size_t> smem_set[kMaxDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (smem_set[dev].load() < cg.dynamicSmemBytes) {
        e = cudaFuncSetAttribute(gemv_bulk_kernel<TYPE, kXS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(cg.dynamicSmemBytes));
        if (e == cudaSuccess) e = match_carveouts();
        if (e != cudaSuccess) return e;
        smem_set[dev].store(cg.dynamicSmemBytes);
    }
    return cudaLaunchKernelEx(&cg, gemv_bulk_kernel<TYPE, kXS>, a, b);
}

// Plans and launches the bulk kernel for `type`; *used = false (nothing
// launched) where it does not apply.
static cudaError_t launch_bulk(int type, bool staged_x, const GemvArgs& a, int64_t ntiles, int sms,
                               cudaStream_t stream, bool* used) {
    BulkPlan p;
    bool ok = false;
    switch (type) {
        case T_Q4_K: ok = bulk_plan<T_Q4_K>(staged_x, a.ngroups, ntiles, sms, &p); break;
        case T_Q5_K: ok = bulk_plan<T_Q5_K>(staged_x, a.ngroups, ntiles, sms, &p); break;
        case T_Q6_K: ok = bulk_plan<T_Q6_K>(staged_x, a.ngroups, ntiles, sms, &p); break;
        case T_Q3_K: ok = bulk_plan<T_Q3_K>(staged_x, a.ngroups, ntiles, sms, &p); break;
        case T_IQ4_XS: ok = bulk_plan<T_IQ4_XS>(staged_x, a.ngroups, ntiles, sms, &p); break;
        case T_IQ3_S: ok = bulk_plan<T_IQ3_S>(staged_x, a.ngroups, ntiles, sms, &p); break;
        case T_IQ3_XXS: ok = bulk_plan<T_IQ3_XXS>(staged_x, a.ngroups, ntiles, sms, &p); break;
        case T_IQ2_S: ok = bulk_plan<T_IQ2_S>(staged_x, a.ngroups, ntiles, sms, &p); break;
        default: ok = bulk_plan<T_Q4_0>(staged_x, a.ngroups, ntiles, sms, &p); break;
    }
    *used = false;
    if (!ok) return cudaSuccess;
    p.b.err = gemv_err_ptr();
    if (!p.b.err) return cudaErrorInvalidDevice;
    cudaLaunchConfig_t cg = {};
    cg.gridDim = dim3(static_cast<unsigned>(p.grid));
    cg.blockDim = dim3(kBulkThreads);
    cg.dynamicSmemBytes = p.smem;
    cg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;  // weights are requested before the dependency wait
    cg.attrs = attr;
    cg.numAttrs = 1;
    *used = true;
#define XB_BULK(T)                                                                        \
    case T:                                                                               \
        return staged_x ? launch_bulk_typed<T, true>(cg, a, p.b) : launch_bulk_typed<T, false>(cg, a, p.b);
    switch (type) {
        XB_BULK(T_Q4_K)
        XB_BULK(T_Q5_K)
        XB_BULK(T_Q6_K)
        XB_BULK(T_Q3_K)
        XB_BULK(T_IQ4_XS)
        XB_BULK(T_IQ3_S)
        XB_BULK(T_IQ3_XXS)
        XB_BULK(T_IQ2_S)
        default: return staged_x ? launch_bulk_typed<T_Q4_0, true>(cg, a, p.b) : launch_bulk_typed<T_Q4_0, false>(cg, a, p.b);
    }
#undef XB_BULK
}

// One thread per (tile, group) through the shared host/device routines of
// formats.cuh: the repack path of the 5-bit layout (a one-time upload cost).
template <bool kPack>
__global__ void __launch_bounds__(128) mma_repack_generic_kernel(int type, const uint8_t* __restrict__ src,
                                                                 uint8_t* __restrict__ dst, int64_t K, int64_t ntiles) {
    const int64_t ngroups = K / 256, row_bytes = ngroups * mma_row_group_bytes(type);
    const int64_t gb = mma_group_bytes(type);
    for (int64_t item = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; item < ntiles * ngroups;
         item += int64_t(gridDim.x) * blockDim.x) {
        const int64_t tile = item / ngroups, gi = item % ngroups;
        const int64_t tbase = tile * MMA_TILE_ROWS * row_bytes;
        if (kPack)
            mma_pack_group(type, src + tbase, row_bytes, gi, dst + tbase + gi * gb);
        else
            mma_unpack_group(type, src + tbase + gi * gb, row_bytes, gi, dst + tbase);
    }
}

cudaError_t mma_repack_launch(int type, const void* raw, void* packed, int64_t N, int64_t K, bool pack,
                              cudaStream_t stream) {
    if (layout_kind(type, N, K) != 1) return cudaErrorInvalidValue;
    const int64_t ntiles = N / MMA_TILE_ROWS, items = ntiles * (K / 256);
    if (type != T_Q4_0 && type != T_Q4_K) {  // every other MMA format: the per-group routine
        const int64_t blocks = (items + 127) / 128 < 65536 ? (items + 127) / 128 : 65536;
        if (pack)
            mma_repack_generic_kernel<true><<<unsigned(blocks), 128, 0, stream>>>(
                type, static_cast<const uint8_t*>(raw), static_cast<uint8_t*>(packed), K, ntiles);
        else
            mma_repack_generic_kernel<false><<<unsigned(blocks), 128, 0, stream>>>(
                type, static_cast<const uint8_t*>(raw), static_cast<uint8_t*>(packed), K, ntiles);
        return cudaGetLastError();
    }
    const int64_t blocks = (items + 3) / 4 < 65536 ? (items + 3) / 4 : 65536;
    if (pack)
        mma_repack_kernel<true><<<unsigned(blocks), 128, 0, stream>>>(type, static_cast<const uint8_t*>(raw),
                                                                     static_cast<uint8_t*>(packed), K, ntiles);
    else
        mma_repack_kernel<false><<<unsigned(blocks), 128, 0, stream>>>(type, static_cast<const uint8_t*>(raw),
                                                                      static_cast<uint8_t*>(packed), K, ntiles);
    return cudaGetLastError();
}

template <int TYPE, bool kTiles, bool kRing>
static cudaError_t launch_gemv_typed(cudaLaunchConfig_t& cg, const GemvArgs& a) {
    if constexpr (kRing) {
        static std::atomic<size_t> smem_set[kMaxDevices];
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        if (smem_set[dev].load() < cg.dynamicSmemBytes) {
            e = cudaFuncSetAttribute(gemv_mma_kernel<TYPE, kTiles, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(cg.dynamicSmemBytes));
            if (e == cudaSuccess) e = match_carveouts();
            if (e != cudaSuccess) return e;
            smem_set[dev].store(cg.dynamicSmemBytes);
        }
    }
    return cudaLaunchKernelEx(&cg, gemv_mma_kernel<TYPE, kTiles, kRing>, a);
}

// Dynamic shared memory of gemv_mma_kernel for a launch touching cta_tiles
// tiles per CTA (the ring variant adds its rings and barriers).
static size_t gemv_smem(int type, int cta_tiles, bool ring) {
    const size_t base = size_t(kWarps) * 2 * MMA_TILE_ROWS * sizeof(float) + size_t(cta_tiles) * sizeof(int);
    if (!ring) return base;
    size_t rb;
    switch (type) {
        case T_Q4_K: rb = ring_bytes<T_Q4_K>(); break;
        case T_Q5_K: rb = ring_bytes<T_Q5_K>(); break;
        case T_Q6_K: rb = ring_bytes<T_Q6_K>(); break;
        case T_Q3_K: rb = ring_bytes<T_Q3_K>(); break;
        case T_IQ4_XS: rb = ring_bytes<T_IQ4_XS>(); break;
        case T_IQ3_S: rb = ring_bytes<T_IQ3_S>(); break;
        case T_IQ3_XXS: rb = ring_bytes<T_IQ3_XXS>(); break;
        case T_IQ2_S: rb = ring_bytes<T_IQ2_S>(); break;
        default: rb = ring_bytes<T_Q4_0>(); break;
    }
    return ring_offset(cta_tiles) + rb;
}

template <bool kTiles, bool kRing>
static cudaError_t launch_gemv(int type, cudaLaunchConfig_t& cg, const GemvArgs& a) {
    switch (type) {
        case T_Q4_K: return launch_gemv_typed<T_Q4_K, kTiles, kRing>(cg, a);
        case T_Q5_K: return launch_gemv_typed<T_Q5_K, kTiles, kRing>(cg, a);
        case T_Q6_K: return launch_gemv_typed<T_Q6_K, kTiles, kRing>(cg, a);
        case T_Q3_K: return launch_gemv_typed<T_Q3_K, kTiles, kRing>(cg, a);
        case T_IQ4_XS: return launch_gemv_typed<T_IQ4_XS, kTiles, kRing>(cg, a);
        case T_IQ3_S: return launch_gemv_typed<T_IQ3_S, kTiles, kRing>(cg, a);
        case T_IQ3_XXS: return launch_gemv_typed<T_IQ3_XXS, kTiles, kRing>(cg, a);
        case T_IQ2_S: return launch_gemv_typed<T_IQ2_S, kTiles, kRing>(cg, a);
        default: return launch_gemv_typed<T_Q4_0, kTiles, kRing>(cg, a);
    }
}

cudaError_t gemv_mma_launch(int type, const void* W, const float* x, float* y, int64_t N, int64_t K,
                            void* scratch, cudaStream_t stream, bool pdl, const MmaFeed* feed, bool x_ready,
                            bool classic) {
    const MmaSegment seg{W, y, N};
    return gemv_mma_multi_launch(type, &seg, 1, x, K, scratch, stream, pdl, nullptr, feed, x_ready, classic);
}

cudaError_t gemv_mma_multi_launch(int type, const MmaSegment* segs, int nseg, const float* x, int64_t K,
                                  void* scratch, cudaStream_t stream, bool pdl, const PeerExchange* xchg,
                                  const MmaFeed* feed, bool x_ready, bool classic, const ShardChain* chain) {
    if (layout_kind(type, MMA_TILE_ROWS, 256) != 1 ||
        nseg < 1 || nseg > kMaxSegs)
        return cudaErrorInvalidValue;
    if (xchg && (xchg->world < 2 || xchg->world > kMaxPeers || xchg->rank < 0 || xchg->rank >= xchg->world))
        return cudaErrorInvalidValue;
    GemvArgs a = {};
    if (xchg) {
        a.xchg = true;
        a.x = *xchg;
    }
    int64_t ntiles = 0;
    for (int s = 0; s < nseg; ++s) {
        if (layout_kind(type, segs[s].N, K) != 1) return cudaErrorInvalidValue;
        a.W[s] = static_cast<const uint8_t*>(segs[s].W);
        a.y[s] = segs[s].y;
        ntiles += segs[s].N / MMA_TILE_ROWS;
        a.tile_end[s] = ntiles;
    }
    a.nseg = nseg;
    const ScratchLayout L = scratch_layout(ntiles * MMA_TILE_ROWS, K);
    uint8_t* base = static_cast<uint8_t*>(scratch);
    const int64_t ngroups = K / 256, nblk = K / 32;
    a.frags = base + L.frags;
    a.zeros = base + L.zeros;
    a.scale = reinterpret_cast<const float*>(base + L.scale);
    a.xsum = reinterpret_cast<const float*>(base + L.xsum);
    a.count = reinterpret_cast<int*>(base + L.count);
    a.done = a.count + ntiles;
    a.partial = reinterpret_cast<float*>(base + L.partial);
    a.ngroups = ngroups;
    a.units = ntiles * ngroups;
    if (chain && (!xchg || chain->nprev < 0 || chain->nprev > kMaxSegs || (chain->nprev > 0 && !chain->prev) ||
                  (chain->feed_peers && (!feed || !chain->peer_base))))
        return cudaErrorInvalidValue;
    const bool feed_peers = chain && chain->feed_peers;
    if (chain) {
        a.wait_peers = chain->nprev > 0 ? 1 : 0;
        a.nprev = chain->nprev;
        for (int s = 0; s < chain->nprev; ++s) a.prev[s] = chain->prev[s];
    }
    if (feed) {
        // the next launch's x is segment feed->seg in full: K_next = its N
        // (times the ranks when this rank's rows go to every peer as well)
        const int64_t nf = segs[feed->seg].N, kn = feed_peers ? nf * xchg->world : nf;
        if ((xchg && !feed_peers) || !feed->next_scratch || feed->seg < 0 || feed->seg >= nseg || kn % 256 != 0 ||
            (feed_peers && nf % 32 != 0) || (feed->bl != 16 && feed->bl != 32) || feed->next_rows <= 0 ||
            feed->next_rows % MMA_TILE_ROWS != 0)
            return cudaErrorInvalidValue;
        const ScratchLayout Ln = scratch_layout(MMA_TILE_ROWS, kn);  // x offsets depend on K only
        uint8_t* nb = static_cast<uint8_t*>(feed->next_scratch);
        a.f_frags = nb + Ln.frags;
        a.f_scale = reinterpret_cast<float*>(nb + Ln.scale);
        a.f_xsum = reinterpret_cast<float*>(nb + Ln.xsum);
        a.f_chunk = a.count + ntiles + 1;
        a.f_y = segs[feed->seg].y;
        a.f_t0 = feed->seg > 0 ? a.tile_end[feed->seg - 1] : 0;
        a.f_t1 = a.tile_end[feed->seg];
        a.f_bl = feed->bl;
        const int64_t nt = feed->next_rows / MMA_TILE_ROWS;
        const ScratchLayout Lf = scratch_layout(feed->next_rows, kn);
        if (feed_peers) {
            a.f_pbase = chain->peer_base;
            a.f_ch0 = xchg->rank * nf / 32;
        }
        a.f_count = reinterpret_cast<int*>(nb + Lf.count);
        a.f_ncount = counter_ints(nt);
        a.f_zeros = reinterpret_cast<uint32_t*>(nb + Lf.zeros);
    }
    if (a.units >= (int64_t(1) << 31)) return cudaErrorInvalidValue;  // the kernel counts units in 32 bits

    const int sms = sm_count();
    if (sms <= 0) return cudaErrorInvalidDevice;
    int64_t blocks = int64_t(sms) * kCtasPerSm;
    if (blocks > kMaxCtas) blocks = kMaxCtas;
    // Tile mode up to 64 units per SM: at 11008 x 2048 it lifted the formats
    // on this path by 25-40 % (no tile spans two CTAs, so no device-scope
    // fences and atomics in the combine); large launches keep the exact split.
    a.tile_mode = a.units <= int64_t(64) * sms ? 1 : 0;
    if (a.tile_mode) {
        if (blocks > ntiles) blocks = ntiles;
        {
            const int64_t per = (ntiles + blocks - 1) / blocks;  // whole tiles per CTA, about the same for all
            blocks = (ntiles + per - 1) / per;
        }
        a.nwarps = blocks * kWarps;
        a.cta_tiles = static_cast<int>((ntiles + blocks - 1) / blocks + 2);
    } else {
        if (blocks > (a.units + kWarps - 1) / kWarps) blocks = (a.units + kWarps - 1) / kWarps;
        if (blocks < 1) blocks = 1;
        a.nwarps = blocks * kWarps < a.units ? blocks * kWarps : a.units;
        const int64_t per_warp = (a.units + a.nwarps - 1) / a.nwarps;
        a.cta_tiles = static_cast<int>((kWarps * per_warp + ngroups - 1) / ngroups + 2);
    }
    const size_t smem = size_t(kWarps) * 2 * MMA_TILE_ROWS * sizeof(float) + size_t(a.cta_tiles) * sizeof(int);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;  // beyond any shape the layout admits

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cudaLaunchConfig_t cp = {};
    int64_t xblocks = (nblk + 1) / 2;                                // one warp per 32-value block
    if ((ntiles + 63) / 64 > xblocks) xblocks = (ntiles + 63) / 64;  // and a thread per tile counter
    if (xblocks > 4096) xblocks = 4096;
    cp.gridDim = dim3(static_cast<unsigned>(xblocks));
    cp.blockDim = dim3(64);
    cp.stream = stream;
    cp.attrs = attr;
    cp.numAttrs = 1;
    if (!x_ready) {  // else the previous launch's epilogue prepared x (and the counters are clear)
        cudaError_t e = mma_blk16(type)
                            ? cudaLaunchKernelEx(&cp, xprep_kernel<16>, x, K, base + L.frags, base + L.zeros,
                                                 reinterpret_cast<float*>(base + L.scale),
                                                 reinterpret_cast<float*>(base + L.xsum), a.count, counter_ints(ntiles))
                            : cudaLaunchKernelEx(&cp, xprep_kernel<32>, x, K, base + L.frags, base + L.zeros,
                                                 reinterpret_cast<float*>(base + L.scale),
                                                 reinterpret_cast<float*>(base + L.xsum), a.count, counter_ints(ntiles));
        if (e != cudaSuccess) return e;
    }

    const int choice = classic ? 0 : gemv_kernel_choice();
    if (xchg && (choice == 1 || choice == 2)) return cudaErrorInvalidValue;  // the bulk kernel has no exchange
    if (choice == 1 || choice == 2) {
        bool used = false;
        const cudaError_t e = launch_bulk(type, choice == 2, a, ntiles, sms, stream, &used);
        if (used || e != cudaSuccess) return e;
    }
    const bool ring = choice == 3;
    a.err = gemv_err_ptr();
    if (!a.err) return cudaErrorInvalidDevice;
    cudaLaunchConfig_t cg = {};
    cg.gridDim = dim3(static_cast<unsigned>(blocks));
    cg.blockDim = dim3(kGemvThreads);
    cg.dynamicSmemBytes = gemv_smem(type, a.cta_tiles, ring);
    cg.stream = stream;
    cudaLaunchAttribute attr2[1];
    attr2[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr2[0].val.programmaticStreamSerializationAllowed = 1;  // overlap the L2 warm-up with xprep
    cg.attrs = attr2;
    cg.numAttrs = 1;
    if (ring) return a.tile_mode ? launch_gemv<true, true>(type, cg, a) : launch_gemv<false, true>(type, cg, a);
    return a.tile_mode ? launch_gemv<true, false>(type, cg, a) : launch_gemv<false, false>(type, cg, a);
}

cudaError_t xchg_gather_launch(const float* xdata, int64_t half_floats, const uint32_t* flags,
                               const uint32_t* epoch, int world, int rank, const GatherSeg* segs, int nseg, int* err,
                               cudaStream_t stream, const MmaFeed* feed) {
    if (nseg < 1 || nseg > kMaxSegs || world < 2 || world > kMaxPeers) return cudaErrorInvalidValue;
    GatherArgs g = {};
    int64_t total = 0;
    for (int s = 0; s < nseg; ++s) {
        g.seg[s] = segs[s];
        total += segs[s].n_local * world;
    }
    g.nseg = nseg;
    GatherFeed f = {};
    if (feed) {
        const int64_t kn = feed->seg >= 0 && feed->seg < nseg ? segs[feed->seg].n_local * world : 0;
        if (!feed->next_scratch || kn <= 0 || kn % 256 != 0 || (feed->bl != 16 && feed->bl != 32) ||
            feed->next_rows <= 0 || feed->next_rows % MMA_TILE_ROWS != 0)
            return cudaErrorInvalidValue;
        uint8_t* nb = static_cast<uint8_t*>(feed->next_scratch);
        const ScratchLayout Ln = scratch_layout(feed->next_rows, kn);
        f.seg = feed->seg;
        f.bl = feed->bl;
        f.frags = nb + Ln.frags;
        f.scale = reinterpret_cast<float*>(nb + Ln.scale);
        f.xsum = reinterpret_cast<float*>(nb + Ln.xsum);
        f.count = reinterpret_cast<int*>(nb + Ln.count);
        f.ncount = counter_ints(feed->next_rows / MMA_TILE_ROWS);
        f.zeros = reinterpret_cast<uint32_t*>(nb + Ln.zeros);
    }
    int64_t blocks = (total + 2047) / 2048;  // few CTAs poll the flags; each copies 8 floats per thread
    if (blocks > 32) blocks = 32;
    if (f.bl != 0) {  // and one warp per 32 values of the next launch's x, as the x-preparation kernel
        const int64_t prep = (segs[f.seg].n_local * world / 32 + 7) / 8;
        if (prep > blocks) blocks = prep < 1024 ? prep : 1024;
    }
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(static_cast<unsigned>(blocks));
    c.blockDim = dim3(256);
    c.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = attr;
    c.numAttrs = 1;
    return cudaLaunchKernelEx(&c, xchg_gather_kernel, xdata, half_floats, flags, epoch, world, rank, g, err, f);
}

// Fixed scratch of b200_gemv_noalloc: one static device array per device
// instead of buffers allocated on demand.  1 MiB holds the layout above for
// N <= 131072 rows with K <= 32768 (frags 256 KiB, counters 32 KiB, partial
// slots 64 KiB, scales and sums 8 KiB).  Nothing in it has to start zeroed:
// every launch's xprep_kernel writes the digits and clears the tile counters
// before the GEMV reads them.  It is shared by every stream of the device.
static __device__ __align__(256) unsigned char g_static_scratch[size_t(1) << 20];

size_t static_scratch_bytes() { return sizeof(g_static_scratch); }

// Device address of g_static_scratch on the current device, looked up once
// per device (cudaGetSymbolAddress) and cached.
cudaError_t static_scratch(void** out) {
    static std::mutex m;
    static void* addr[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(m);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
    }
    *out = addr[dev];
    return cudaSuccess;
}

// Scratch for launcher calls that bring none: two slots per (device, stream),
// alternated so that a GEMV reading one slot can overlap (PDL) the next call's
// x preparation writing the other.  Grown on demand (must not happen inside
// stream capture: the first call for a new, larger K allocates).
void* launcher_scratch(cudaStream_t stream, int64_t N, int64_t K) {
    const size_t need = gemv_scratch_bytes(N, K);
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
