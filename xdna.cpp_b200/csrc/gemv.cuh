// Internal launcher interface of the GEMV, repack and quantize kernels.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace xb {

// Devices a process may use with the per-device caches of this library.
constexpr int kMaxDevices = 64;

// A launch whose output segment `seg` is, in full, the x of the launch that
// follows it on the stream: its epilogue writes that x's digit fragments,
// scales and sums into the next launch's scratch (next_scratch, sized by
// xprep_bytes for the next launch) and clears that launch's counters, and the
// next launch runs with x_ready set (no x-preparation kernel).  bl = the next launch's x block: 32, or 16 for
// the types with 16-value sub-blocks.
struct MmaFeed {
    void* next_scratch = nullptr;
    int64_t next_rows = 0;  // rows of the next launch (all its segments): the counters it needs cleared
    int seg = 0;
    int bl = 32;
};

struct LaunchOpts {
    bool pdl = false;          // programmatic dependent launch (overlap with the previous kernel)
    void* scratch = nullptr;   // MMA-path scratch of gemv_scratch_bytes(N, K) (xprep_bytes(N, K) when
                               // `classic`), zeroed when new (nullptr: internal)
    bool classic = false;      // MMA path: the classic kernel only (its scratch is xprep_bytes(N, K))
    const MmaFeed* feed = nullptr;  // MMA path: this launch prepares the next launch's x
    bool x_ready = false;           // MMA path: the previous launch prepared this launch's x
};

// MMA path (gemv_mma.cu): scratch bytes for one x vector of length K, the
// launcher's internal per-(device, stream) scratch, the two kernels and the
// MMA-layout repack of whole 16-row tiles (raw / packed point at the first row).
struct ScratchLayout {
    size_t frags, zeros, scale, xsum, count, partial, total;
};
ScratchLayout scratch_layout(int64_t N, int64_t K);
size_t xprep_bytes(int64_t N, int64_t K);
// Scratch of any MMA GEMV launch over N rows: xprep_bytes plus the bulk
// kernel's split-tile chunk sums.
size_t gemv_scratch_bytes(int64_t N, int64_t K);
// Reads and clears the current device's GEMV error word (nonzero: a bounded
// wait inside a bulk-copy GEMV ran out).
cudaError_t gemv_error_status(int* out);
void* launcher_scratch(cudaStream_t stream, int64_t N, int64_t K);
// The fixed static-array scratch of b200_gemv_noalloc: its size, and its
// device address on the current device (cudaGetSymbolAddress, once per device).
size_t static_scratch_bytes();
cudaError_t static_scratch(void** out);
cudaError_t gemv_mma_launch(int type, const void* W, const float* x, float* y, int64_t N, int64_t K, void* scratch,
                            cudaStream_t stream, bool pdl, const MmaFeed* feed = nullptr, bool x_ready = false,
                            bool classic = false);
// Several MMA-layout matrices of one type that multiply the same x (same K)
// in one launch: y_s = W_s x for s < nseg <= MMA_MAX_SEGMENTS, scratch of
// xprep_bytes(sum of N_s, K).
struct MmaSegment {
    const void* W;
    float* y;
    int64_t N;
};
// Row-sharded launches (one process per GPU): besides writing its own rows of
// y, the GEMV stores them into every peer's exchange buffer (peer memory
// mapped over NVLink) and, when all its CTAs are done, raises its flag
// (= epoch) in every peer's flag array.  A gather kernel on each GPU then
// waits for the peers' flags and copies their rows into the full outputs.
// The epoch lives on the device (no launch argument changes from one launch
// to the next, so a step can be replayed as a CUDA graph): launch e reads
// e - 1 from *epoch, uses data half e % 2, and its last CTA stores e.
constexpr int kMaxPeers = 8;
struct PeerExchange {
    float* peer_data[kMaxPeers];       // each rank's exchange buffer, half 0 (half 1 follows)
    uint32_t* peer_flags[kMaxPeers];   // each rank's flag array (one word per source rank)
    int world, rank;
    int64_t half_floats;               // floats per data half
    uint32_t* epoch;                   // this rank's epoch counter (device memory)
    int64_t xo[4];                     // segment s's first float in the exchange buffer
    int* err;                          // set when a bounded wait for the peers runs out
};
// A chain of row-sharded launches without gather kernels between them: a
// launch whose output segment is the next launch's x (MmaFeed) prepares its
// own rows' part of that x into its local scratch and, over NVLink, into the
// same scratch slot of every peer (the slots sit at one offset of every
// rank's exchange region, whose base addresses `peer_base` lists in device
// memory).  The next launch then waits (bounded) until every peer's flag
// shows the previous epoch, and copies the previous launch's peer rows
// (segments `prev`, from this GPU's exchange data of the previous epoch) into
// their full outputs before it computes.
struct GatherSeg;
struct ShardChain {
    bool feed_peers = false;
    const float* const* peer_base = nullptr;  // [world]: each rank's exchange data half 0
    int nprev = 0;
    const GatherSeg* prev = nullptr;
};
cudaError_t gemv_mma_multi_launch(int type, const MmaSegment* segs, int nseg, const float* x, int64_t K,
                                  void* scratch, cudaStream_t stream, bool pdl, const PeerExchange* xchg = nullptr,
                                  const MmaFeed* feed = nullptr, bool x_ready = false, bool classic = false,
                                  const ShardChain* chain = nullptr);
// Copy the peers' rows of each segment from this GPU's exchange buffer
// (xdata: half 0) into the full outputs once every peer's flag reaches the
// launch's epoch, read from *epoch after the GEMV has stored it (a bounded
// wait: on time-out it sets *err and copies nothing).  With a feed (seg =
// index into segs) the gather also prepares that full output as the next
// launch's x, as a feeding GEMV would.
struct GatherSeg {
    float* y_full;
    int64_t n_local;
    int64_t xo;
};
cudaError_t xchg_gather_launch(const float* xdata, int64_t half_floats, const uint32_t* flags,
                               const uint32_t* epoch, int world, int rank, const GatherSeg* segs, int nseg, int* err,
                               cudaStream_t stream, const MmaFeed* feed = nullptr);
cudaError_t mma_repack_launch(int type, const void* raw, void* packed, int64_t N, int64_t K, bool pack,
                              cudaStream_t stream);

// y[N] = W[N,K] x[K]; W in the stripe-tile layout (formats.cuh), device pointers.
cudaError_t gemv_launch(int type, const void* W, const float* x, float* y, int64_t N, int64_t K,
                        cudaStream_t stream, const LaunchOpts& opts);
size_t gemv_smem_bytes(int type, int64_t K);

// GGUF rows [row0, row0 + nrows) of a matrix with N rows <-> stripe tiles.
// row0 and nrows must be tile aligned (nrows may end at N).  raw and packed
// are device pointers to row row0 (the layouts have the same byte span).
cudaError_t repack_launch(int type, const void* raw, void* packed, int64_t N, int64_t K, int64_t row0,
                          int64_t nrows, cudaStream_t stream);
cudaError_t unpack_launch(int type, const void* packed, void* raw, int64_t N, int64_t K, int64_t row0,
                          int64_t nrows, cudaStream_t stream);

// BF16 activations -> F32 (reference bf16_to_float, exact).
cudaError_t bf16_to_f32_launch(const uint16_t* src, float* dst, int64_t n, cudaStream_t stream);

// Synthetic weights: N(0, sigma) F32 from a counter-based generator, and the
// device quantisers (Q4_0: ggml quantize_row_q4_0_ref; Q4_K: this build's
// affine 6-bit scale/min fit).  Output in GGUF layout.
cudaError_t fill_normal_launch(float* out, int64_t n, uint64_t seed, float sigma, cudaStream_t stream);
cudaError_t quantize_launch(int type, const float* src, void* dst, int64_t N, int64_t K, cudaStream_t stream);
bool quantize_supported(int type);

}  // namespace xb
