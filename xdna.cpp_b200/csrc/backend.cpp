// Host runtime of the B200 decode-GEMV backend: the compat C ABI, HBM buffer
// types with a bounded pinned upload path, and the MUL_MAT graph executor.
//
// Reference counterparts:
//   src/ggml-xdna.cpp:95-147    supports_op_impl      -> supports_mul_mat()
//   src/ggml-xdna.cpp:149-308   process_mul_mat_node  -> run_node(), run_fused()
//   src/ggml-xdna.cpp:316-470   buffer / buffer-type  -> Buffer, BufferType
//   src/ggml-xdna.cpp:719-844   compat entry points   -> extern "C" section
//   src/dma_streamer.cpp:153-419 bounded 2-slot pinned staging -> Staging
//
// Compute is synchronous per call, as in the reference (caps.async = false):
// activations and outputs may be host or device pointers; host ones go
// through a pinned bounce arena on the backend's stream and outputs are
// written back before compute_graph returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <chrono>
#include <thread>

#include "../../include/ggml-b200.h"
#include "formats.cuh"
#include "gemv.cuh"
#include "nccl_shim.h"

namespace xb {

// ------------------------------------------------------------------ errors
namespace {
thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    fprintf(stderr, "[b200 error] %s\n", buf);
}

bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return false;
}

constexpr uint32_t kBackendMagic = 0x58444E41;  // "XDNA", reference src/ggml-xdna.cpp:32
constexpr uint32_t kBufferMagic = 0x58425546;   // "XBUF"
constexpr uint32_t kBuftMagic = 0x58425454;     // "XBTT"
constexpr size_t kAlignment = 4096;             // reference buft_get_alignment :407-410

int device_count() {
    static int count = -1;
    static std::once_flag once;
    std::call_once(once, [] {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        count = n;
    });
    return count;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && prev != cur) cudaSetDevice(prev);
    }
};

size_t env_size(const char* name, size_t dflt) {
    const char* v = getenv(name);
    if (!v || !*v) return dflt;
    const long long x = atoll(v);
    return x > 0 ? static_cast<size_t>(x) : dflt;
}

size_t type_size_bytes(int type, int64_t* blck) {
    // ggml block sizes for the types a buffer may hold (reference :427-448)
    *blck = 1;
    switch (type) {
        case GGML_TYPE_F32: case GGML_TYPE_I32: return 4;
        case GGML_TYPE_F16: case GGML_TYPE_BF16: case GGML_TYPE_I16: return 2;
        case GGML_TYPE_I8: return 1;
        case GGML_TYPE_I64: case GGML_TYPE_F64: return 8;
        case GGML_TYPE_Q4_1: *blck = 32; return 20;
        case GGML_TYPE_Q5_0: *blck = 32; return 22;
        case GGML_TYPE_Q5_1: *blck = 32; return 24;
        case GGML_TYPE_Q8_0: *blck = 32; return 34;
        default: {
            const FormatInfo f = format_info(type);
            if (f.block_vals) {
                *blck = f.block_vals;
                return static_cast<size_t>(f.block_bytes);
            }
            return 4;
        }
    }
}

size_t tensor_nbytes(const ggml_tensor_xdna* t) {
    int64_t blck = 1;
    const size_t ts = type_size_bytes(t->type, &blck);
    const int64_t ne0 = t->ne[0] > 0 ? t->ne[0] : 1;
    const int64_t ne1 = t->ne[1] > 0 ? t->ne[1] : 1;
    const int64_t ne2 = t->ne[2] > 0 ? t->ne[2] : 1;
    const int64_t ne3 = t->ne[3] > 0 ? t->ne[3] : 1;
    return static_cast<size_t>(ne0 / blck) * ts * static_cast<size_t>(ne1 * ne2 * ne3);
}

// ------------------------------------------------------------------ staging
// Bounded pinned upload/download path of one device: two pinned host slots and
// two device slots (slot size XDNA_B200_STAGING_MB, default 64 MiB), used
// round-robin with an event per slot -- the B200 analogue of the reference's
// 2 x 128 MiB staging ring (src/dma_streamer.cpp:165-172).
struct Staging {
    int dev = 0;
    size_t slot_bytes = 0;
    void* pinned[2] = {nullptr, nullptr};
    void* devbuf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    cudaStream_t stream = nullptr;
    int next = 0;
    std::mutex mtx;
    bool ready = false;

    bool init(int d) {
        if (ready) return true;
        dev = d;
        DeviceGuard g(dev);
        slot_bytes = env_size("XDNA_B200_STAGING_MB", 64) << 20;
        if (!cuda_ok(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "staging stream")) return false;
        for (int s = 0; s < 2; ++s) {
            if (!cuda_ok(cudaHostAlloc(&pinned[s], slot_bytes, cudaHostAllocPortable), "staging pinned alloc"))
                return false;
            if (!cuda_ok(cudaMalloc(&devbuf[s], slot_bytes), "staging device alloc")) return false;
            if (!cuda_ok(cudaEventCreateWithFlags(&done[s], cudaEventDisableTiming), "staging event")) return false;
        }
        ready = true;
        return true;
    }
    int acquire() {  // a free slot (its previous work finished)
        const int s = next;
        next ^= 1;
        cudaEventSynchronize(done[s]);
        return s;
    }
};

Staging& staging_for(int dev) {
    static std::mutex m;
    static std::map<int, std::unique_ptr<Staging>> all;
    std::lock_guard<std::mutex> lk(m);
    auto& p = all[dev];
    if (!p) p = std::make_unique<Staging>();
    return *p;
}

// ------------------------------------------------------------------ objects
struct BufferType {
    uint32_t magic = kBuftMagic;
    int dev = 0;
    bool host = false;
};

struct TensorInfo {
    int type = 0;
    int64_t K = 0, N = 0, nmat = 1;
    size_t mat_bytes = 0;
    bool packed = false;  // stripe layout (claimed quant type)
};

struct Buffer {
    uint32_t magic = kBufferMagic;
    BufferType* buft = nullptr;
    void* base = nullptr;
    size_t size = 0;
    bool owned = true;
    std::mutex mtx;
    std::map<uintptr_t, TensorInfo> tensors;  // keyed by tensor data address
};

struct BufferRegistry {
    std::mutex mtx;
    std::map<uintptr_t, Buffer*> by_base;
    void add(Buffer* b) {
        std::lock_guard<std::mutex> lk(mtx);
        by_base[reinterpret_cast<uintptr_t>(b->base)] = b;
    }
    void remove(Buffer* b) {
        std::lock_guard<std::mutex> lk(mtx);
        by_base.erase(reinterpret_cast<uintptr_t>(b->base));
    }
    Buffer* find(const void* p) {
        std::lock_guard<std::mutex> lk(mtx);
        const uintptr_t a = reinterpret_cast<uintptr_t>(p);
        auto it = by_base.upper_bound(a);
        if (it == by_base.begin()) return nullptr;
        --it;
        Buffer* b = it->second;
        return (a >= it->first && a < it->first + std::max<size_t>(b->size, 1)) ? b : nullptr;
    }
};
BufferRegistry& registry() {
    static BufferRegistry r;
    return r;
}

// Weights written into one of this backend's device buffers (repacked there).
bool resident_weights(const void* data) {
    Buffer* b = data ? registry().find(data) : nullptr;
    if (!b || b->buft->host) return false;
    std::lock_guard<std::mutex> lk(b->mtx);
    auto it = b->tensors.find(reinterpret_cast<uintptr_t>(data));
    return it != b->tensors.end() && it->second.packed;
}

BufferType* buft_instance(int dev, bool host) {
    static std::mutex m;
    static std::map<std::pair<int, bool>, std::unique_ptr<BufferType>> all;
    std::lock_guard<std::mutex> lk(m);
    auto& p = all[{dev, host}];
    if (!p) {
        p = std::make_unique<BufferType>();
        p->dev = dev;
        p->host = host;
    }
    return p.get();
}

BufferType* as_buft(void* p) {
    auto* b = static_cast<BufferType*>(p);
    return (b && b->magic == kBuftMagic) ? b : nullptr;
}
Buffer* as_buffer(void* p) {
    auto* b = static_cast<Buffer*>(p);
    return (b && b->magic == kBufferMagic) ? b : nullptr;
}

// Grow-only device / pinned arenas with bump allocation, reset when the
// stream has drained.
struct Arena {
    bool pinned = false;
    void* base = nullptr;
    size_t cap = 0, used = 0;
    void release() {
        if (base) pinned ? cudaFreeHost(base) : cudaFree(base);
        base = nullptr;
        cap = used = 0;
    }
    bool reserve(size_t bytes) {  // only when used == 0
        if (bytes <= cap) return true;
        release();
        size_t c = 1 << 20;
        while (c < bytes) c <<= 1;
        const cudaError_t e = pinned ? cudaHostAlloc(&base, c, cudaHostAllocPortable) : cudaMalloc(&base, c);
        if (e != cudaSuccess) {
            base = nullptr;
            return cuda_ok(e, pinned ? "pinned arena alloc" : "device arena alloc");
        }
        cap = c;
        return true;
    }
    void* take(size_t bytes) {
        const size_t off = (used + 255) & ~size_t(255);
        if (off + bytes > cap) return nullptr;
        used = off + bytes;
        return static_cast<char*>(base) + off;
    }
};

struct Backend {
    uint32_t magic = kBackendMagic;
    int dev = 0;
    cudaStream_t stream = nullptr;
    // row-sharded execution (ggml_backend_xdna_init_sharded)
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    std::mutex mtx;
    Arena dev_arena{false}, host_arena{true};
    // host weight matrices uploaded for the current call (see run_jobs)
    Arena wt_arena{false};
    struct PendingOut {
        void* dst;
        const void* src;
        size_t bytes;
    };
    std::vector<PendingOut> pending;
    // x-digit scratch of the MMA GEMV path: two slots, alternated per launch,
    // so that a launch can write the next launch's x digits (prepared-x chain)
    // while it reads its own
    void* xscratch[2] = {nullptr, nullptr};
    size_t xscratch_bytes = 0;
    int xscratch_next = 0;
    // Peer exchange of row-sharded MMA launches (see setup_exchange): this
    // rank's region (flag words, then two data halves used by alternate
    // launches) and every rank's region mapped into this process.
    struct Exchange {
        bool ok = false;
        char* local = nullptr;
        char* peer[kMaxPeers] = {};
        size_t cap_floats = 0;  // floats per data half
        uint32_t* epoch = nullptr;  // the device epoch counter (a word of the local flag region)
        int* err = nullptr;     // set by a gather kernel or a GEMV whose wait for the peers timed out
        size_t slot_bytes = 0;  // the two x-scratch slots after the data halves (same offsets on every rank)
        float** base_table = nullptr;  // device: each rank's data half 0 (ShardChain::peer_base)
    } xg;
    // CUDA graph of the last node list seen twice in a row with every operand
    // on this device (see compute_graph); scratch_gen invalidates it when the
    // x scratch it captured is reallocated.
    std::vector<uint64_t> graph_sig;
    bool graph_ok_sig = false;  // graph_sig was checked and is capturable
    // Device copies of MUL_MAT inputs and outputs that sit in page-locked host
    // memory (see shadow_host_operands); kept across calls, freed with the
    // backend or when more than kMaxShadows would be needed.
    struct HostShadow {
        void* host;
        size_t bytes;
        void* dev;
    };
    std::vector<HostShadow> shadows;
    // which MUL_MAT operands of the node list with signature pin_sig are
    // page-locked host memory (bit 0: src1, bit 1: dst, per node index), so
    // that a list seen again costs no pointer queries
    struct PinnedOp {
        size_t node;
        unsigned mask;
        const void* x;  // the node's src1 and dst data when classified
        const void* y;
    };
    std::vector<uint64_t> pin_sig;
    std::vector<PinnedOp> pin_ops;
    cudaGraphExec_t graph_exec = nullptr;
    uint64_t graph_gen = 0, scratch_gen = 0;
};

// A scratch slot of at least gemv_scratch_bytes(N, K); growing it drains the stream first.
void* backend_xscratch(Backend* be, int64_t N, int64_t K);

// Both x-scratch slots hold at least `need` bytes (growing them waits for
// the stream: never inside a stream capture).
bool backend_xscratch_reserve(Backend* be, size_t need) {
    if (need > be->xscratch_bytes && be->xg.ok) {
        set_error("a GEMV launch needs %zu bytes of scratch, more than the exchange region's %zu-byte slots "
                  "(XDNA_B200_XSLOT_MB)",
                  need, be->xscratch_bytes);
        return false;
    }
    if (need > be->xscratch_bytes) {
        if (cudaStreamSynchronize(be->stream) != cudaSuccess) return false;
        const size_t cap = std::max<size_t>(need, 1u << 20);
        for (int s = 0; s < 2; ++s) {
            if (be->xscratch[s]) cudaFree(be->xscratch[s]);
            be->xscratch[s] = nullptr;
            if (!cuda_ok(cudaMalloc(&be->xscratch[s], cap), "x scratch alloc") ||
                !cuda_ok(cudaMemset(be->xscratch[s], 0, cap), "x scratch clear")) {
                be->xscratch_bytes = 0;
                return false;
            }
        }
        be->xscratch_bytes = cap;
        ++be->scratch_gen;
    }
    return true;
}

void* backend_xscratch(Backend* be, int64_t N, int64_t K) {
    if (!backend_xscratch_reserve(be, gemv_scratch_bytes(N, K))) return nullptr;
    void* p = be->xscratch[be->xscratch_next];
    be->xscratch_next ^= 1;
    return p;
}

bool nccl_wait(ncclComm_t comm, ncclResult_t r, const char* what);

// Exchange regions: [flags: one uint32 per source rank, then this rank's
// epoch counter at byte 128; 256 B][half 0][half 1][x-scratch slot 0][slot 1].
// The slots are the backend's GEMV scratch: a sharded launch writes the next
// launch's x into the same slot of every rank (XDNA_B200_XSLOT_MB each,
// default 8).
constexpr size_t kXchgFlagBytes = 256;
constexpr size_t kXchgEpochOffset = 128;

void release_exchange(Backend* be) {
    Backend::Exchange& x = be->xg;
    for (int p = 0; p < kMaxPeers; ++p)
        if (x.peer[p] && x.peer[p] != x.local) cudaIpcCloseMemHandle(x.peer[p]);
    if (x.local) cudaFree(x.local);
    if (x.err) cudaFree(x.err);
    if (x.base_table) cudaFree(x.base_table);
    x = Backend::Exchange{};
}

// Allocate this rank's exchange region, swap IPC handles with the other ranks
// over NCCL and map theirs.  Any failure leaves the backend on the NCCL
// all-gather path (x.ok stays false) with the reason in the error string.
bool setup_exchange(Backend* be) {
    Backend::Exchange& x = be->xg;
    if (be->world < 2 || be->world > kMaxPeers || getenv("XDNA_B200_NO_P2P")) return false;
    const char* mb = getenv("XDNA_B200_XCHG_MB");
    const size_t half_bytes = (mb ? static_cast<size_t>(atol(mb)) : 16) << 20;
    x.cap_floats = half_bytes / sizeof(float);
    x.slot_bytes = env_size("XDNA_B200_XSLOT_MB", 8) << 20;
    const size_t bytes = kXchgFlagBytes + 2 * half_bytes + 2 * x.slot_bytes;
    bool ok = cuda_ok(cudaMalloc(&x.local, bytes), "exchange alloc") &&
              cuda_ok(cudaMemset(x.local, 0, bytes), "exchange clear") &&
              cuda_ok(cudaMalloc(&x.err, sizeof(int)), "exchange error word") &&
              cuda_ok(cudaMemset(x.err, 0, sizeof(int)), "exchange error clear") &&
              cuda_ok(cudaDeviceSynchronize(), "exchange clear sync");
    cudaIpcMemHandle_t mine;
    ok = ok && cuda_ok(cudaIpcGetMemHandle(&mine, x.local), "cudaIpcGetMemHandle");
    // every rank must take part in the handle all-gather even if its own setup
    // failed (a zero handle then tells the others to stay on NCCL)
    if (!ok) memset(&mine, 0, sizeof mine);
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    char* d = nullptr;
    std::vector<char> all(hb * be->world);
    bool gathered = cuda_ok(cudaMalloc(&d, hb * be->world), "handle buffer");
    if (gathered) {
        gathered = cuda_ok(cudaMemcpy(d + hb * be->rank, &mine, hb, cudaMemcpyHostToDevice), "handle upload");
        const NcclApi& api = nccl_api();
        const ncclResult_t r = api.AllGather(d + hb * be->rank, d, hb, ncclInt8, be->comm, be->stream);
        gathered = nccl_wait(be->comm, r, "handle all-gather") && gathered &&
                   cuda_ok(cudaStreamSynchronize(be->stream), "handle sync") &&
                   cuda_ok(cudaMemcpy(all.data(), d, hb * be->world, cudaMemcpyDeviceToHost), "handle download");
        cudaFree(d);
    }
    ok = ok && gathered;
    static const char zero[sizeof(cudaIpcMemHandle_t)] = {};
    for (int p = 0; p < be->world && ok; ++p) {
        if (p == be->rank) {
            x.peer[p] = x.local;
            continue;
        }
        if (!memcmp(all.data() + hb * p, zero, hb)) {
            ok = false;
            break;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, all.data() + hb * p, hb);
        void* ptr = nullptr;
        ok = cuda_ok(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        x.peer[p] = static_cast<char*>(ptr);
    }
    if (!ok) {
        cudaGetLastError();
        release_exchange(be);
        return false;
    }
    x.epoch = reinterpret_cast<uint32_t*>(x.local + kXchgEpochOffset);  // zero: cleared with the region
    std::vector<float*> bases(be->world);
    for (int p = 0; p < be->world; ++p) bases[p] = reinterpret_cast<float*>(x.peer[p] + kXchgFlagBytes);
    if (!cuda_ok(cudaMalloc(&x.base_table, sizeof(float*) * be->world), "exchange base table") ||
        !cuda_ok(cudaMemcpy(x.base_table, bases.data(), sizeof(float*) * be->world, cudaMemcpyHostToDevice),
                 "exchange base table upload")) {
        release_exchange(be);
        return false;
    }
    // the GEMV scratch slots move into the exchange region (zeroed with it)
    for (int s = 0; s < 2; ++s) {
        if (be->xscratch[s]) cudaFree(be->xscratch[s]);
        be->xscratch[s] = x.local + kXchgFlagBytes + 2 * half_bytes + s * x.slot_bytes;
    }
    be->xscratch_bytes = x.slot_bytes;
    ++be->scratch_gen;
    x.ok = true;
    return true;
}

// A timed-out gather wait leaves its mark in the exchange's error word.
bool exchange_error(Backend* be) {
    if (!be->xg.ok) return false;
    int e = 0;
    if (cudaMemcpy(&e, be->xg.err, sizeof e, cudaMemcpyDeviceToHost) != cudaSuccess) return true;
    if (!e) return false;
    cudaMemset(be->xg.err, 0, sizeof(int));
    return true;
}

Backend* as_backend(void* p) {
    auto* b = static_cast<Backend*>(p);
    return (b && b->magic == kBackendMagic) ? b : nullptr;
}

bool is_device_pointer(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// --------------------------------------------------------- tensor transfers
// A tensor of a claimed quant type is held as nmat matrices of N rows, each in
// the stripe layout.  Transfers walk tile-aligned row chunks of at most one
// staging slot.
struct Chunk {
    int64_t mat, row0, nrows;
    size_t byte0, bytes;  // tensor-relative GGUF byte range of the chunk
};

std::vector<Chunk> chunks_for(const TensorInfo& ti, size_t off, size_t size, size_t slot_bytes) {
    std::vector<Chunk> out;
    const size_t rb = static_cast<size_t>(ti.mat_bytes / std::max<int64_t>(ti.N, 1));
    if (rb == 0 || size == 0) return out;
    // 16-row granularity suits both layouts (stripe tiles of 8, MMA tiles of 16 rows)
    const int64_t tile_rows_per_chunk = std::max<int64_t>(
        MMA_TILE_ROWS, static_cast<int64_t>(slot_bytes / (rb * MMA_TILE_ROWS)) * MMA_TILE_ROWS);
    const size_t end = off + size;
    for (int64_t m = off / ti.mat_bytes; m < ti.nmat && static_cast<size_t>(m) * ti.mat_bytes < end; ++m) {
        const size_t mb = static_cast<size_t>(m) * ti.mat_bytes;
        const size_t lo = std::max(off, mb) - mb, hi = std::min(end, mb + ti.mat_bytes) - mb;
        int64_t r0 = static_cast<int64_t>(lo / rb) / MMA_TILE_ROWS * MMA_TILE_ROWS;
        const int64_t r1 = static_cast<int64_t>((hi + rb - 1) / rb);
        while (r0 < r1) {
            const int64_t n = std::min<int64_t>(tile_rows_per_chunk, ti.N - r0);
            out.push_back({m, r0, n, mb + static_cast<size_t>(r0) * rb, static_cast<size_t>(n) * rb});
            r0 += n;
        }
    }
    return out;
}

bool upload_packed(Staging& st, const TensorInfo& ti, uint8_t* dev_tensor, const uint8_t* host, size_t off,
                   size_t size, const uint8_t* fill /* memset value or null */) {
    for (const Chunk& c : chunks_for(ti, off, size, st.slot_bytes)) {
        const int s = st.acquire();
        uint8_t* raw = static_cast<uint8_t*>(st.devbuf[s]);
        uint8_t* dst = dev_tensor + c.byte0;
        const size_t w0 = std::max(off, c.byte0), w1 = std::min(off + size, c.byte0 + c.bytes);
        const bool full = (w0 == c.byte0 && w1 == c.byte0 + c.bytes);
        if (!full) {  // read-modify-write: bring the chunk back to GGUF layout first
            if (!cuda_ok(unpack_launch(ti.type, dst, raw, ti.N, ti.K, c.row0, c.nrows, st.stream), "unpack"))
                return false;
        }
        if (fill) {
            if (!cuda_ok(cudaMemsetAsync(raw + (w0 - c.byte0), *fill, w1 - w0, st.stream), "memset")) return false;
        } else {
            memcpy(st.pinned[s], host + (w0 - off), w1 - w0);
            if (!cuda_ok(cudaMemcpyAsync(raw + (w0 - c.byte0), st.pinned[s], w1 - w0, cudaMemcpyHostToDevice,
                                         st.stream),
                         "H2D"))
                return false;
        }
        if (!cuda_ok(repack_launch(ti.type, raw, dst, ti.N, ti.K, c.row0, c.nrows, st.stream), "repack"))
            return false;
        cudaEventRecord(st.done[s], st.stream);
    }
    return cuda_ok(cudaStreamSynchronize(st.stream), "staging sync");
}

bool download_packed(Staging& st, const TensorInfo& ti, const uint8_t* dev_tensor, uint8_t* host, size_t off,
                     size_t size) {
    for (const Chunk& c : chunks_for(ti, off, size, st.slot_bytes)) {
        const int s = st.acquire();
        uint8_t* raw = static_cast<uint8_t*>(st.devbuf[s]);
        if (!cuda_ok(unpack_launch(ti.type, dev_tensor + c.byte0, raw, ti.N, ti.K, c.row0, c.nrows, st.stream),
                     "unpack"))
            return false;
        const size_t r0 = std::max(off, c.byte0), r1 = std::min(off + size, c.byte0 + c.bytes);
        if (!cuda_ok(cudaMemcpyAsync(st.pinned[s], raw + (r0 - c.byte0), r1 - r0, cudaMemcpyDeviceToHost, st.stream),
                     "D2H"))
            return false;
        if (!cuda_ok(cudaStreamSynchronize(st.stream), "staging sync")) return false;
        memcpy(host + (r0 - off), st.pinned[s], r1 - r0);
        cudaEventRecord(st.done[s], st.stream);
    }
    return true;
}

bool copy_plain(Staging& st, void* dev, const void* host_src, void* host_dst, size_t size) {
    for (size_t o = 0; o < size; o += st.slot_bytes) {
        const size_t n = std::min(st.slot_bytes, size - o);
        const int s = st.acquire();
        if (host_src) {
            memcpy(st.pinned[s], static_cast<const char*>(host_src) + o, n);
            if (!cuda_ok(cudaMemcpyAsync(static_cast<char*>(dev) + o, st.pinned[s], n, cudaMemcpyHostToDevice,
                                         st.stream),
                         "H2D"))
                return false;
            cudaEventRecord(st.done[s], st.stream);
        } else {
            if (!cuda_ok(cudaMemcpyAsync(st.pinned[s], static_cast<char*>(dev) + o, n, cudaMemcpyDeviceToHost,
                                         st.stream),
                         "D2H"))
                return false;
            if (!cuda_ok(cudaStreamSynchronize(st.stream), "staging sync")) return false;
            memcpy(static_cast<char*>(host_dst) + o, st.pinned[s], n);
            cudaEventRecord(st.done[s], st.stream);
        }
    }
    return cuda_ok(cudaStreamSynchronize(st.stream), "staging sync");
}

// Describe (and validate) a tensor written into a device buffer.
bool tensor_info_for(const ggml_tensor_xdna* t, TensorInfo* ti) {
    ti->type = t->type;
    ti->K = t->ne[0];
    ti->N = t->ne[1] > 0 ? t->ne[1] : 1;
    ti->nmat = (t->ne[2] > 0 ? t->ne[2] : 1) * (t->ne[3] > 0 ? t->ne[3] : 1);
    const FormatInfo f = format_info(t->type);
    const bool contiguous =
        (t->nb[1] == 0 || t->nb[1] == static_cast<size_t>(ti->K / std::max(f.block_vals, 1)) * f.block_bytes);
    ti->packed = f.block_vals != 0 && ti->K > 0 && ti->K % f.block_vals == 0 && contiguous;
    ti->mat_bytes = ti->packed ? static_cast<size_t>(ti->N) * static_cast<size_t>(ti->K / f.block_vals) * f.block_bytes
                               : 0;
    return true;
}

// ------------------------------------------------------------- supports_op
bool row_bytes_for(int type, int64_t K, size_t* rb) {
    const FormatInfo f = format_info(type);
    if (!f.block_vals || K % f.block_vals) return false;
    *rb = static_cast<size_t>(K / f.block_vals) * f.block_bytes;
    return true;
}

bool resident_weights(const void* data);

// Same predicate as the reference's supports_op_impl (src/ggml-xdna.cpp:95-147):
// MUL_MAT, F32 src1, N >= 32, N % 4 == 0, K a block multiple, packed rows, and
// M == 1 -- except for weights that already live in this backend's device
// buffers, which the reference's ggml path also claims for any M
// (is_tensor_loader_probe, :81-93, :109-111): a host cannot run those rows
// itself, and the executor loops over the M activation rows.
bool supports_mul_mat(const ggml_tensor_xdna* op) {
    if (!op || op->op != GGML_OP_MUL_MAT) return false;
    const ggml_tensor_xdna* src0 = op->src[0];
    const ggml_tensor_xdna* src1 = op->src[1];
    if (!src0 || !src1) return false;
    if (src1->type != GGML_TYPE_F32) return false;
    const int64_t K = src0->ne[0], N = src0->ne[1], M = src1->ne[1];
    if (N < 32 || N % 4 != 0) return false;
    if (M != 1 && !(M > 1 && resident_weights(src0->data))) return false;
    size_t rb = 0;
    if (!type_supported(src0->type) || !row_bytes_for(src0->type, K, &rb)) return false;
    return src0->nb[1] == 0 || src0->nb[1] == rb;
}

// ------------------------------------------------------------- execution
struct Job {
    int type;
    const void* w;  // device, stripe layout
    const float* x; // device, 16-byte aligned
    float* y;       // device
    int64_t N, K;
};

bool ranges_overlap(const void* a, size_t an, const void* b, size_t bn) {
    const char* pa = static_cast<const char*>(a);
    const char* pb = static_cast<const char*>(b);
    return pa < pb + bn && pb < pa + an;
}

bool flush(Backend* be) {
    if (!cuda_ok(cudaStreamSynchronize(be->stream), "compute sync")) {
        be->pending.clear();
        be->dev_arena.used = be->host_arena.used = be->wt_arena.used = 0;
        return false;
    }
    if (exchange_error(be)) {
        set_error("row-sharded exchange: a peer's rows did not arrive within the wait limit");
        be->pending.clear();
        be->dev_arena.used = be->host_arena.used = be->wt_arena.used = 0;
        return false;
    }
    for (const auto& p : be->pending) memcpy(p.dst, p.src, p.bytes);
    be->pending.clear();
    be->dev_arena.used = be->host_arena.used = be->wt_arena.used = 0;
    return true;
}

bool overlaps_pending(Backend* be, const void* p, size_t n) {
    for (const auto& o : be->pending)
        if (ranges_overlap(o.dst, o.bytes, p, n)) return true;
    return false;
}

// device copy of a host range (through the pinned arena), 256-byte aligned
const void* stage_in(Backend* be, const void* host, size_t bytes) {
    if (overlaps_pending(be, host, bytes) && !flush(be)) return nullptr;
    void* h = be->host_arena.take(bytes);
    void* d = be->dev_arena.take(bytes);
    if (!h || !d) {
        if (!flush(be)) return nullptr;
        if (!be->host_arena.reserve(std::max(bytes, be->host_arena.cap * 2)) ||
            !be->dev_arena.reserve(std::max(bytes, be->dev_arena.cap * 2)))
            return nullptr;
        h = be->host_arena.take(bytes);
        d = be->dev_arena.take(bytes);
        if (!h || !d) return nullptr;
    }
    memcpy(h, host, bytes);
    if (!cuda_ok(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, be->stream), "H2D activations")) return nullptr;
    return d;
}

// device output slot for a host destination, written back at flush time
float* stage_out(Backend* be, void* host, size_t bytes, void** pinned_out) {
    void* h = be->host_arena.take(bytes);
    void* d = be->dev_arena.take(bytes);
    if (!h || !d) {
        if (!flush(be)) return nullptr;
        if (!be->host_arena.reserve(std::max(bytes, be->host_arena.cap * 2)) ||
            !be->dev_arena.reserve(std::max(bytes, be->dev_arena.cap * 2)))
            return nullptr;
        h = be->host_arena.take(bytes);
        d = be->dev_arena.take(bytes);
        if (!h || !d) return nullptr;
    }
    *pinned_out = h;
    (void)host;
    return static_cast<float*>(d);
}

// Host-resident weights: uploaded and repacked for this call into the weight
// arena (there is no residency cache keyed by host pointer: a caller may
// rewrite the same host memory between calls).  Device-resident weights
// belong in a buffer of ggml_backend_xdna_buffer_type().
const void* stage_weights(Backend* be, int type, const uint8_t* host, int64_t N, int64_t K, size_t rb) {
    const size_t bytes = static_cast<size_t>(N) * rb;
    if (overlaps_pending(be, host, bytes) && !flush(be)) return nullptr;
    void* d = be->wt_arena.take(bytes);
    if (!d) {
        if (!flush(be)) return nullptr;
        if (!be->wt_arena.reserve(std::max(bytes, be->wt_arena.cap * 2))) return nullptr;
        d = be->wt_arena.take(bytes);
        if (!d) return nullptr;
    }
    Staging& st = staging_for(be->dev);
    std::lock_guard<std::mutex> lk(st.mtx);
    if (!st.init(be->dev)) return nullptr;
    TensorInfo ti;
    ti.type = type;
    ti.K = K;
    ti.N = N;
    ti.nmat = 1;
    ti.mat_bytes = bytes;
    ti.packed = true;
    // the staging stream must not overwrite d while an earlier kernel of this
    // call still reads the arena region: make the staging stream wait.
    cudaEvent_t ev;
    cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    cudaEventRecord(ev, be->stream);
    cudaStreamWaitEvent(st.stream, ev, 0);
    cudaEventDestroy(ev);
    if (!upload_packed(st, ti, static_cast<uint8_t*>(d), host, 0, bytes, nullptr)) return nullptr;
    return d;
}

// ------------------------------------------------------------------ NCCL
double nccl_timeout_s() {
    const char* v = getenv("XDNA_B200_NCCL_TIMEOUT_S");
    const double t = v ? atof(v) : 0.0;
    return t > 0 ? t : 120.0;
}

// Poll a non-blocking communicator until its pending operation completes,
// with a host-side time limit; on timeout the communicator is aborted so
// that no rank waits forever for a peer that never arrives.
bool nccl_wait(ncclComm_t comm, ncclResult_t r, const char* what) {
    const NcclApi& api = nccl_api();
    const auto t0 = std::chrono::steady_clock::now();
    // enqueueing a collective on a non-blocking communicator finishes within
    // microseconds: spin (yielding) first, sleep only if it takes longer
    while (r == ncclInProgress) {
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > nccl_timeout_s()) {
            api.CommAbort(comm);
            set_error("%s: timed out after %.0f s (communicator aborted)", what, nccl_timeout_s());
            return false;
        }
        if (el < 2e-3)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        if (api.CommGetAsyncError(comm, &r) != ncclSuccess) break;
    }
    if (r != ncclSuccess) {
        set_error("%s: %s", what, api.GetErrorString(r));
        return false;
    }
    return true;
}

bool all_gather_rows(Backend* be, float* y_full, int64_t n_local) {
    const NcclApi& api = nccl_api();
    const ncclResult_t r = api.AllGather(y_full + be->rank * n_local, y_full, static_cast<size_t>(n_local), ncclFloat32,
                                         be->comm, be->stream);
    return nccl_wait(be->comm, r, "ncclAllGather");
}

// One MUL_MAT node -> jobs (reference process_mul_mat_node, :149-308).
// A planned MMA launch (compute_graph): its scratch slot, and whether it
// prepares the next launch's x (feed) or runs on x prepared by the previous one.
struct MmaPlan {
    void* scratch = nullptr;
    const MmaFeed* feed = nullptr;
    bool x_ready = false;
    // sharded chain: the feed goes to every rank (no gather kernel after this
    // launch), and this launch assembles the previous launch's outputs
    bool feed_peers = false;
    int nprev = 0;
    GatherSeg prev[MMA_MAX_SEGMENTS];
};

bool run_node(Backend* be, ggml_tensor_xdna* node, const MmaPlan* plan = nullptr) {
    ggml_tensor_xdna* src0 = node->src[0];
    ggml_tensor_xdna* src1 = node->src[1];
    const char* name = node->name;
    if (!src0 || !src1) {
        set_error("node '%s' missing src0/src1", name);
        return false;
    }
    if (src1->type != GGML_TYPE_F32) {
        set_error("node '%s' src1 type %d != F32", name, src1->type);
        return false;
    }
    if (!node->data || !src0->data || !src1->data) {
        set_error("node '%s' null data ptrs: node->data=%p src0->data=%p src1->data=%p", name, node->data,
                  src0->data, src1->data);
        return false;
    }
    const int64_t K = src0->ne[0], N = src0->ne[1], M = src1->ne[1];
    if (M == 0 || N == 0) return true;
    if (M < 0 || N < 0 || K < 0) {
        set_error("node '%s' negative dim: M=%ld N=%ld K=%ld", name, long(M), long(N), long(K));
        return false;
    }
    const FormatInfo f = format_info(src0->type);
    if (!f.block_vals) {
        set_error("node '%s' unsupported src0 type=%d", name, src0->type);
        return false;
    }
    if (K % f.block_vals != 0) {
        set_error("node '%s' K=%ld not div by %d", name, long(K), f.block_vals);
        return false;
    }
    const size_t rb = static_cast<size_t>(K / f.block_vals) * f.block_bytes;
    if (src0->nb[1] != 0 && src0->nb[1] != rb) {
        set_error("node '%s' src0 nb1 mismatch: %zu != %zu", name, src0->nb[1], rb);
        return false;
    }
    const size_t total_weight_bytes = static_cast<size_t>(N) * rb;
    const int64_t ne2 = node->ne[2] > 0 ? node->ne[2] : 1;
    const int64_t ne3 = node->ne[3] > 0 ? node->ne[3] : 1;
    // Row-sharded node: src0 holds this rank's N rows of a weight with
    // N * world rows, dst is the full output; each rank computes its slice
    // and the slices are all-gathered over NCCL.
    const bool sharded = be->world > 1 && node->ne[0] == N * be->world;
    const int64_t n_out = sharded ? N * be->world : N;
    const size_t dst_stride1 = node->nb[1] > 0 ? node->nb[1] : static_cast<size_t>(n_out) * sizeof(float);
    const size_t dst_stride2 = node->nb[2] > 0 ? node->nb[2] : dst_stride1 * M;
    const size_t dst_stride3 = node->nb[3] > 0 ? node->nb[3] : dst_stride2 * ne2;
    const size_t src1_stride1 = src1->nb[1] > 0 ? src1->nb[1] : static_cast<size_t>(K) * sizeof(float);
    const size_t src1_stride2 = src1->ne[2] > 1 ? (src1->nb[2] > 0 ? src1->nb[2] : src1_stride1 * M) : 0;
    const size_t src1_stride3 = src1->ne[3] > 1 ? (src1->nb[3] > 0 ? src1->nb[3] : src1_stride2 * ne2) : 0;
    const size_t src0_stride2 = src0->ne[2] > 1 ? (src0->nb[2] > 0 ? src0->nb[2] : total_weight_bytes) : 0;
    const size_t src0_stride3 = src0->ne[3] > 1 ? (src0->nb[3] > 0 ? src0->nb[3] : src0_stride2 * ne2) : 0;

    // where the weights live
    Buffer* wbuf = registry().find(src0->data);
    const TensorInfo* wti = nullptr;
    if (wbuf && !wbuf->buft->host) {
        std::lock_guard<std::mutex> lk(wbuf->mtx);
        auto it = wbuf->tensors.find(reinterpret_cast<uintptr_t>(src0->data));
        if (it == wbuf->tensors.end() || !it->second.packed) {
            set_error("node '%s': weights in a B200 buffer were not written with "
                      "ggml_backend_xdna_buffer_set_tensor as a claimed quant type",
                      name);
            return false;
        }
        wti = &it->second;
        if (wbuf->buft->dev != be->dev) {
            set_error("node '%s': weights live on device %d, backend is on device %d", name, wbuf->buft->dev, be->dev);
            return false;
        }
    }
    const bool w_device = wbuf != nullptr && !wbuf->buft->host;
    const bool x_device = is_device_pointer(src1->data);
    const bool y_device = is_device_pointer(node->data);

    const uint8_t* base_w = static_cast<const uint8_t*>(src0->data);
    const char* base_x = static_cast<const char*>(src1->data);
    char* base_y = static_cast<char*>(node->data);

    for (int64_t i3 = 0; i3 < ne3; ++i3) {
        for (int64_t i2 = 0; i2 < ne2; ++i2) {
            const uint8_t* w_host = base_w + i3 * src0_stride3 + i2 * src0_stride2;
            const void* w_dev = nullptr;
            if (w_device) {
                const size_t rel = static_cast<size_t>(w_host - base_w);
                if (wti->mat_bytes == 0 || rel % wti->mat_bytes != 0 || wti->K != K || wti->N != N) {
                    set_error("node '%s': weight slice does not match the packed tensor geometry", name);
                    return false;
                }
                w_dev = w_host;
            } else {
                w_dev = stage_weights(be, src0->type, w_host, N, K, rb);
                if (!w_dev) {
                    set_error("node '%s': weight upload failed: %s", name, g_last_error.c_str());
                    return false;
                }
            }
            for (int64_t m = 0; m < M; ++m) {
                const char* a_m = base_x + i3 * src1_stride3 + i2 * src1_stride2 + m * src1_stride1;
                char* o_m = base_y + i3 * dst_stride3 + i2 * dst_stride2 + m * dst_stride1;
                const float* xd;
                if (x_device && (reinterpret_cast<uintptr_t>(a_m) & 15u) == 0) {
                    xd = reinterpret_cast<const float*>(a_m);
                } else if (x_device) {
                    void* d = be->dev_arena.take(static_cast<size_t>(K) * 4);
                    if (!d) {
                        if (!flush(be) || !be->dev_arena.reserve(std::max<size_t>(K * 4, be->dev_arena.cap * 2)))
                            return false;
                        d = be->dev_arena.take(static_cast<size_t>(K) * 4);
                    }
                    if (!cuda_ok(cudaMemcpyAsync(d, a_m, static_cast<size_t>(K) * 4, cudaMemcpyDeviceToDevice,
                                                 be->stream),
                                 "align activations"))
                        return false;
                    xd = static_cast<const float*>(d);
                } else {
                    xd = static_cast<const float*>(stage_in(be, a_m, static_cast<size_t>(K) * 4));
                    if (!xd) return false;
                }
                float* yd;
                void* pinned = nullptr;
                const size_t out_bytes = static_cast<size_t>(n_out) * 4;
                if (y_device) {
                    yd = reinterpret_cast<float*>(o_m);
                } else {
                    yd = stage_out(be, o_m, out_bytes, &pinned);
                    if (!yd) return false;
                }
                LaunchOpts lo;
                lo.pdl = true;  // kernels wait (griddepcontrol) before touching what earlier work writes
                if (layout_kind(src0->type, N, K) == 1) {
                    lo.scratch = plan && plan->scratch ? plan->scratch : backend_xscratch(be, N, K);
                    if (!lo.scratch) return false;
                    if (plan) {
                        lo.feed = plan->feed;
                        lo.x_ready = plan->x_ready;
                    }
                }
                float* y_local = sharded ? yd + be->rank * N : yd;
                if (!cuda_ok(gemv_launch(src0->type, w_dev, xd, y_local, N, K, be->stream, lo), "gemv launch"))
                    return false;
                if (sharded && !all_gather_rows(be, yd, N)) return false;
                if (!y_device) {
                    if (!cuda_ok(cudaMemcpyAsync(pinned, yd, out_bytes, cudaMemcpyDeviceToHost, be->stream),
                                 "D2H outputs"))
                        return false;
                    be->pending.push_back({o_m, pinned, out_bytes});
                }
            }
        }
    }
    return true;
}

// ------------------------------------------------------------- node fusion
// Consecutive MUL_MAT nodes that multiply the same device-resident x by
// MMA-layout weights (q / k / v, or gate / up, of a transformer block) run as
// one launch: one x preparation, one GEMV grid over all their row tiles.
struct FusableNode {
    int type;
    int64_t K;
    const float* x;
    MmaSegment seg;   // W, this rank's output rows, local N
    float* y_full;    // the node's output (all ranks' rows when sharded)
    int64_t n_out;    // rows of y_full
    bool sharded;
};

bool fusable(Backend* be, const ggml_tensor_xdna* node, FusableNode* out) {
    if (!node || node->op != GGML_OP_MUL_MAT) return false;
    const ggml_tensor_xdna* src0 = node->src[0];
    const ggml_tensor_xdna* src1 = node->src[1];
    if (!src0 || !src1 || src1->type != GGML_TYPE_F32 || !node->data || !src0->data || !src1->data) return false;
    const int64_t K = src0->ne[0], N = src0->ne[1];
    if (src1->ne[1] != 1 || src1->ne[0] != K || layout_kind(src0->type, N, K) != 1) return false;
    for (int d = 2; d < 4; ++d)
        if (node->ne[d] > 1 || src0->ne[d] > 1 || src1->ne[d] > 1) return false;
    const size_t rb = static_cast<size_t>(K / 256) * mma_row_group_bytes(src0->type);
    if (src0->nb[1] != 0 && src0->nb[1] != rb) return false;
    if ((reinterpret_cast<uintptr_t>(src1->data) & 15u) || !is_device_pointer(src1->data) ||
        !is_device_pointer(node->data))
        return false;
    Buffer* wbuf = registry().find(src0->data);
    if (!wbuf || wbuf->buft->host || wbuf->buft->dev != be->dev) return false;
    {
        std::lock_guard<std::mutex> lk(wbuf->mtx);
        auto it = wbuf->tensors.find(reinterpret_cast<uintptr_t>(src0->data));
        if (it == wbuf->tensors.end() || !it->second.packed || it->second.N != N || it->second.K != K) return false;
    }
    const bool sharded = be->world > 1 && node->ne[0] == N * be->world;
    if (!sharded && node->ne[0] != N) return false;
    out->type = src0->type;
    out->K = K;
    out->x = static_cast<const float*>(src1->data);
    out->y_full = static_cast<float*>(node->data);
    out->n_out = sharded ? N * be->world : N;
    out->seg = MmaSegment{src0->data, out->y_full + (sharded ? be->rank * N : 0), N};
    out->sharded = sharded;
    return true;
}

// Nodes [i, i + count) of `nodes` that fuse with node i (count >= 1 when node i is fusable).
size_t fused_run_length(Backend* be, ggml_tensor_xdna** nodes, size_t i, size_t n_nodes, FusableNode* f) {
    if (!fusable(be, nodes[i], &f[0])) return 0;
    const char* x0 = reinterpret_cast<const char*>(f[0].x);
    const size_t xbytes = static_cast<size_t>(f[0].K) * sizeof(float);
    auto overlaps = [](const void* a, size_t an, const void* b, size_t bn) {
        return static_cast<const char*>(a) < static_cast<const char*>(b) + bn &&
               static_cast<const char*>(b) < static_cast<const char*>(a) + an;
    };
    if (overlaps(f[0].y_full, f[0].n_out * 4, x0, xbytes)) return 1;
    size_t n = 1;
    while (n < static_cast<size_t>(MMA_MAX_SEGMENTS) && i + n < n_nodes) {
        FusableNode c;
        if (!fusable(be, nodes[i + n], &c) || c.type != f[0].type || c.K != f[0].K || c.x != f[0].x) break;
        bool clash = overlaps(c.y_full, c.n_out * 4, x0, xbytes);
        for (size_t k = 0; k < n && !clash; ++k) clash = overlaps(c.y_full, c.n_out * 4, f[k].y_full, f[k].n_out * 4);
        if (clash) break;
        f[n++] = c;
    }
    return n;
}

bool run_fused(Backend* be, const FusableNode* f, size_t n, const MmaPlan* plan = nullptr) {
    MmaSegment segs[MMA_MAX_SEGMENTS];
    int64_t rows = 0;
    for (size_t k = 0; k < n; ++k) {
        segs[k] = f[k].seg;
        rows += f[k].seg.N;
    }
    void* scratch = plan && plan->scratch ? plan->scratch : backend_xscratch(be, rows, f[0].K);
    if (!scratch) return false;
    // row-sharded: rows travel to the peers from the GEMV itself when the
    // outputs fit the exchange buffers; NCCL all-gather otherwise
    int64_t full = 0;
    bool all_sharded = true;
    for (size_t k = 0; k < n; ++k) {
        full += f[k].n_out;
        all_sharded = all_sharded && f[k].sharded;
    }
    if (be->xg.ok && all_sharded && static_cast<size_t>(full) <= be->xg.cap_floats) {
        Backend::Exchange& xg = be->xg;
        PeerExchange pe = {};
        pe.world = be->world;
        pe.rank = be->rank;
        pe.half_floats = static_cast<int64_t>(xg.cap_floats);
        pe.epoch = xg.epoch;
        for (int p = 0; p < be->world; ++p) {
            pe.peer_data[p] = reinterpret_cast<float*>(xg.peer[p] + kXchgFlagBytes);
            pe.peer_flags[p] = reinterpret_cast<uint32_t*>(xg.peer[p]);
        }
        pe.err = xg.err;
        GatherSeg gs[MMA_MAX_SEGMENTS];
        int64_t off = 0;
        for (size_t k = 0; k < n; ++k) {
            pe.xo[k] = off;
            gs[k] = GatherSeg{f[k].y_full, f[k].seg.N, off};
            off += f[k].n_out;
        }
        ShardChain sc;
        sc.peer_base = xg.base_table;
        sc.feed_peers = plan && plan->feed_peers;
        sc.nprev = plan ? plan->nprev : 0;
        sc.prev = plan ? plan->prev : nullptr;
        if (!cuda_ok(gemv_mma_multi_launch(f[0].type, segs, static_cast<int>(n), f[0].x, f[0].K, scratch, be->stream,
                                           true, &pe, sc.feed_peers ? plan->feed : nullptr, plan && plan->x_ready,
                                           false, &sc),
                     "sharded gemv launch"))
            return false;
        // the next sharded launch assembles these outputs itself; otherwise a
        // gather (which also prepares a planned feed from the full output)
        if (sc.feed_peers) return true;
        return cuda_ok(xchg_gather_launch(reinterpret_cast<const float*>(xg.local + kXchgFlagBytes),
                                          static_cast<int64_t>(xg.cap_floats),
                                          reinterpret_cast<const uint32_t*>(xg.local), xg.epoch, be->world, be->rank,
                                          gs, static_cast<int>(n), xg.err, be->stream, plan ? plan->feed : nullptr),
                       "exchange gather launch");
    }
    if (!cuda_ok(gemv_mma_multi_launch(f[0].type, segs, static_cast<int>(n), f[0].x, f[0].K, scratch, be->stream, true,
                                       nullptr, plan ? plan->feed : nullptr, plan && plan->x_ready),
                 "fused gemv launch"))
        return false;
    bool any = false;
    for (size_t k = 0; k < n; ++k) any = any || f[k].sharded;
    if (!any) return true;
    // one NCCL group: the slices of every fused node travel in one launch
    const NcclApi& api = nccl_api();
    ncclResult_t r = api.GroupStart();
    for (size_t k = 0; k < n && r == ncclSuccess; ++k)
        if (f[k].sharded)
            r = api.AllGather(f[k].y_full + be->rank * f[k].seg.N, f[k].y_full, static_cast<size_t>(f[k].seg.N),
                              ncclFloat32, be->comm, be->stream);
    const ncclResult_t e = api.GroupEnd();
    if (r == ncclSuccess || r == ncclInProgress) r = e;
    return nccl_wait(be->comm, r, "grouped ncclAllGather");
}

// ------------------------------------------------------------- graph replay
// The MUL_MAT fields that determine the launches of a node list.
void graph_signature(ggml_tensor_xdna** nodes, size_t n, std::vector<uint64_t>* sig) {
    sig->clear();
    for (size_t i = 0; i < n; ++i) {
        const ggml_tensor_xdna* t = nodes[i];
        if (!t || t->op != GGML_OP_MUL_MAT) continue;
        const ggml_tensor_xdna* a = t->src[0];
        const ggml_tensor_xdna* b = t->src[1];
        if (!a || !b) {
            sig->push_back(~0ull);
            continue;
        }
        const uint64_t v[] = {reinterpret_cast<uintptr_t>(a->data), uint64_t(a->type), uint64_t(a->ne[0]),
                              uint64_t(a->ne[1]), uint64_t(a->ne[2]), uint64_t(a->ne[3]), a->nb[1],
                              reinterpret_cast<uintptr_t>(b->data), uint64_t(b->type), uint64_t(b->ne[0]),
                              uint64_t(b->ne[1]), uint64_t(b->ne[2]), b->nb[1], reinterpret_cast<uintptr_t>(t->data),
                              uint64_t(t->ne[0]), uint64_t(t->ne[1]), t->nb[1]};
        sig->insert(sig->end(), v, v + sizeof v / sizeof v[0]);
    }
}

// Every MUL_MAT node runs on this device without host staging: resident
// weights, device x and y, one activation row.
bool device_only_nodes(Backend* be, ggml_tensor_xdna** nodes, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        const ggml_tensor_xdna* t = nodes[i];
        if (!t || t->op != GGML_OP_MUL_MAT) continue;
        const ggml_tensor_xdna* a = t->src[0];
        const ggml_tensor_xdna* b = t->src[1];
        if (!a || !b || b->ne[1] != 1 || b->ne[2] > 1 || b->ne[3] > 1 || a->ne[2] > 1 || a->ne[3] > 1) return false;
        if (!resident_weights(a->data) || registry().find(a->data)->buft->dev != be->dev) return false;
        if (!b->data || (reinterpret_cast<uintptr_t>(b->data) & 15u) || !is_device_pointer(b->data)) return false;
        if (!t->data || !is_device_pointer(t->data)) return false;
    }
    return true;
}

void drop_graph(Backend* be) {
    if (be->graph_exec) cudaGraphExecDestroy(be->graph_exec);
    be->graph_exec = nullptr;
}

bool is_pinned_host(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// A node list whose MUL_MAT inputs or outputs are single F32 rows in
// page-locked host memory (a decode step's token input and logits, say) is
// run on a copy of the list in which those operands are device buffers: the
// inputs are copied in at the start of the call and the outputs out at its
// end.  The copy then plans, fuses, chains and replays as a CUDA graph like a
// device-resident list, instead of staging every such node through the
// host (page-locked copies are stream operations that a graph can hold).
// Not used when a host range is both written and read by the list, or when
// an operand is not one contiguous row.
struct ShadowPlan {
    std::vector<ggml_tensor_xdna> nodes, srcs;
    std::vector<ggml_tensor_xdna*> ptrs;
    std::vector<size_t> in, out;  // indices into Backend::shadows
};
constexpr size_t kMaxShadows = 64;

bool shadow_host_operands(Backend* be, ggml_tensor_xdna** nodes, size_t n, const std::vector<uint64_t>& sig,
                          bool may_alloc, ShadowPlan* sp) {
    struct Use {
        void* host;
        size_t bytes;
        bool out;
    };
    if (sig != be->pin_sig) {
        be->pin_ops.clear();
        for (size_t i = 0; i < n; ++i) {
            const ggml_tensor_xdna* t = nodes[i];
            if (!t || t->op != GGML_OP_MUL_MAT || !t->src[0] || !t->src[1]) continue;
            const unsigned m = (t->src[1]->data && is_pinned_host(t->src[1]->data) ? 1u : 0u) |
                               (t->data && is_pinned_host(t->data) ? 2u : 0u);
            if (m) be->pin_ops.push_back({i, m, t->src[1]->data, t->data});
        }
        be->pin_sig = sig;
    }
    if (be->pin_ops.empty()) return false;
    std::vector<Use> uses;
    for (const Backend::PinnedOp& op : be->pin_ops) {
        // the same signature with the MUL_MATs at other node indices: classify again next call
        const ggml_tensor_xdna* t = op.node < n ? nodes[op.node] : nullptr;
        if (!t || t->op != GGML_OP_MUL_MAT || !t->src[0] || !t->src[1] || t->src[1]->data != op.x ||
            t->data != op.y) {
            be->pin_sig.clear();
            return false;
        }
        const ggml_tensor_xdna* b = t->src[1];
        const bool xh = (op.mask & 1u) != 0, yh = (op.mask & 2u) != 0;
        if (b->type != GGML_TYPE_F32 || b->ne[1] != 1 || b->ne[2] != 1 || b->ne[3] != 1 || t->ne[1] != 1 ||
            t->ne[2] != 1 || t->ne[3] != 1)
            return false;
        if (xh) uses.push_back({b->data, static_cast<size_t>(b->ne[0]) * 4, false});
        if (yh) uses.push_back({t->data, static_cast<size_t>(t->ne[0]) * 4, true});
    }
    if (uses.empty()) return false;
    for (const Use& u : uses)
        for (const Use& v : uses)
            if ((u.out || v.out) && &u != &v && ranges_overlap(u.host, u.bytes, v.host, v.bytes) &&
                !(u.host == v.host && !u.out && !v.out))
                return false;
    // one shadow per host range
    std::vector<size_t> idx(uses.size());
    for (size_t k = 0; k < uses.size(); ++k) {
        size_t j = be->shadows.size();
        for (size_t q = 0; q < be->shadows.size(); ++q)
            if (be->shadows[q].host == uses[k].host && be->shadows[q].bytes >= uses[k].bytes) j = q;
        if (j == be->shadows.size()) {
            if (!may_alloc || be->shadows.size() >= kMaxShadows) return false;
            void* d = nullptr;
            if (cudaMalloc(&d, uses[k].bytes) != cudaSuccess) {
                cudaGetLastError();
                return false;
            }
            be->shadows.push_back({uses[k].host, uses[k].bytes, d});
            ++be->scratch_gen;  // a graph holding other device copies is out of date
        }
        idx[k] = j;
    }
    sp->in.clear();
    sp->out.clear();
    for (size_t k = 0; k < uses.size(); ++k) {
        std::vector<size_t>& v = uses[k].out ? sp->out : sp->in;
        if (std::find(v.begin(), v.end(), idx[k]) == v.end()) v.push_back(idx[k]);
    }
    auto shadow_of = [&](const void* host) -> void* {
        for (size_t k = 0; k < uses.size(); ++k)
            if (uses[k].host == host) return be->shadows[idx[k]].dev;
        return nullptr;
    };
    sp->nodes.clear();
    sp->srcs.clear();
    sp->nodes.reserve(n);
    sp->srcs.reserve(n);
    sp->ptrs.assign(nodes, nodes + n);
    for (size_t i = 0; i < n; ++i) {
        ggml_tensor_xdna* t = nodes[i];
        if (!t || t->op != GGML_OP_MUL_MAT || !t->src[0] || !t->src[1]) continue;
        void* xd = shadow_of(t->src[1]->data);
        void* yd = shadow_of(t->data);
        if (!xd && !yd) continue;
        sp->nodes.push_back(*t);
        ggml_tensor_xdna& c = sp->nodes.back();
        if (xd) {
            sp->srcs.push_back(*t->src[1]);
            sp->srcs.back().data = xd;
            c.src[1] = &sp->srcs.back();
        }
        if (yd) c.data = yd;
        sp->ptrs[i] = &c;
    }
    return true;
}


}  // namespace
}  // namespace xb

using namespace xb;

// ====================================================================== C ABI
extern "C" {

const char* ggml_backend_xdna_last_error(void) { return g_last_error.c_str(); }

size_t ggml_backend_xdna_get_device_count(void) { return static_cast<size_t>(device_count()); }

void ggml_backend_xdna_get_device_memory(size_t dev_num, size_t* free_bytes, size_t* total_bytes) {
    size_t f = 0, t = 0;
    if (static_cast<int>(dev_num) < device_count()) {
        DeviceGuard g(static_cast<int>(dev_num));
        if (cudaMemGetInfo(&f, &t) != cudaSuccess) cudaGetLastError();
    }
    if (free_bytes) *free_bytes = f;
    if (total_bytes) *total_bytes = t;
}

ggml_backend_reg_t ggml_backend_xdna_reg(void) {
    static uint32_t reg_token = 0x58524547;  // "XREG": opaque registry handle of the compat ABI
    return &reg_token;
}

ggml_backend_t ggml_backend_xdna_init(size_t dev_num) {
    if (static_cast<int>(dev_num) >= device_count()) {
        set_error("ggml_backend_xdna_init: CUDA device %zu not available (%d device(s))", dev_num, device_count());
        return nullptr;
    }
    auto be = std::make_unique<Backend>();
    be->dev = static_cast<int>(dev_num);
    DeviceGuard g(be->dev);
    if (!cuda_ok(cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking), "backend stream")) return nullptr;
    return be.release();
}

int ggml_backend_xdna_nccl_unique_id(uint8_t out[128]) {
    const NcclApi& api = nccl_api();
    if (!api.ok) {
        set_error("NCCL (libnccl.so.2) could not be loaded");
        return -1;
    }
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    ncclUniqueId id;
    const ncclResult_t r = api.GetUniqueId(&id);
    if (r != ncclSuccess) {
        set_error("ncclGetUniqueId: %s", api.GetErrorString(r));
        return -2;
    }
    memcpy(out, &id, sizeof id);
    return 0;
}

ggml_backend_t ggml_backend_xdna_init_sharded(size_t dev_num, int world, int rank, const uint8_t id[128]) {
    if (world < 1 || rank < 0 || rank >= world || !id) {
        set_error("init_sharded: bad world %d / rank %d", world, rank);
        return nullptr;
    }
    Backend* be = static_cast<Backend*>(ggml_backend_xdna_init(dev_num));
    if (!be) return nullptr;
    be->rank = rank;
    be->world = world;
    if (world == 1) return be;
    const NcclApi& api = nccl_api();
    if (!api.ok) {
        set_error("init_sharded: NCCL (libnccl.so.2) could not be loaded");
        ggml_backend_xdna_free(be);
        return nullptr;
    }
    DeviceGuard g(be->dev);
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // initialisation polled below with a time limit
    const ncclResult_t r = api.CommInitRankConfig(&be->comm, world, uid, rank, &cfg);
    if ((r != ncclSuccess && r != ncclInProgress) || !nccl_wait(be->comm, r, "ncclCommInitRankConfig")) {
        if (r != ncclSuccess && r != ncclInProgress) set_error("ncclCommInitRankConfig: %s", api.GetErrorString(r));
        if (be->comm && r == ncclSuccess) api.CommDestroy(be->comm);
        be->comm = nullptr;
        ggml_backend_xdna_free(be);
        return nullptr;
    }
    setup_exchange(be);  // on failure the sharded nodes use NCCL all-gathers
    return be;
}

int ggml_backend_xdna_shard_rows(int64_t n, int world, int rank, int64_t* row0, int64_t* nrows) {
    if (world < 1 || rank < 0 || rank >= world || n < 0 || n % world != 0) {
        set_error("shard_rows: N=%ld is not divisible by world %d", long(n), world);
        return -1;
    }
    if (row0) *row0 = (n / world) * rank;
    if (nrows) *nrows = n / world;
    return 0;
}

bool ggml_backend_is_xdna(ggml_backend_t backend) { return as_backend(backend) != nullptr; }

void ggml_backend_xdna_free(ggml_backend_t backend) {
    Backend* be = as_backend(backend);
    if (!be) return;
    {
        DeviceGuard g(be->dev);
        std::lock_guard<std::mutex> lk(be->mtx);
        cudaStreamSynchronize(be->stream);
        be->dev_arena.release();
        be->host_arena.release();
        be->wt_arena.release();
        if (!be->xg.ok)
            for (void* p : be->xscratch)
                if (p) cudaFree(p);
        for (const Backend::HostShadow& h : be->shadows) cudaFree(h.dev);
        release_exchange(be);
        drop_graph(be);
        if (be->comm) nccl_api().CommDestroy(be->comm);
        cudaStreamDestroy(be->stream);
        be->magic = 0;
    }
    delete be;
}

void* ggml_backend_xdna_get_stream(ggml_backend_t backend) {
    Backend* be = as_backend(backend);
    return be ? static_cast<void*>(be->stream) : nullptr;
}

void ggml_backend_xdna_synchronize(ggml_backend_t backend) {
    Backend* be = as_backend(backend);
    if (!be) return;
    DeviceGuard g(be->dev);
    cudaStreamSynchronize(be->stream);
}

ggml_backend_buffer_type_t ggml_backend_xdna_buffer_type(size_t dev_num) {
    return buft_instance(static_cast<int>(dev_num), false);
}

ggml_backend_buffer_type_t ggml_backend_xdna_host_buffer_type(void) { return buft_instance(0, true); }

bool ggml_backend_xdna_supports_op(ggml_backend_t backend, const struct ggml_tensor_xdna* op) {
    (void)backend;
    return supports_mul_mat(op);
}

static bool run_nodes(Backend* be, ggml_tensor_xdna** nodes, size_t n_nodes) {
    static const bool trace = getenv("XDNA_TRACE_NODES") != nullptr;
    static const bool no_fuse = getenv("XDNA_NO_FUSE") != nullptr;
    // Plan the launches first.  Device-resident MMA launches (one fused run
    // or one node) get their scratch slots in order, alternating; where a
    // launch's x is, in full, one output segment of the launch before it, that
    // launch's epilogue prepares the x (MmaFeed) and the x-preparation kernel
    // is left out.
    struct Run {
        size_t i, count, nf;
        int64_t rows;  // of all the launch's segments
        bool fused, planned;
        FusableNode f[MMA_MAX_SEGMENTS];
        MmaPlan plan;
        MmaFeed feed;
    };
    static thread_local std::vector<Run> runs;  // reused: no allocation per call
    runs.clear();
    size_t need = 0;
    for (size_t i = 0; i < n_nodes;) {
        ggml_tensor_xdna* node = nodes[i];
        if (!node || node->op != GGML_OP_MUL_MAT) {
            ++i;
            continue;
        }
        Run r;
        r.i = i;
        r.nf = no_fuse ? (fusable(be, node, &r.f[0]) ? 1 : 0) : fused_run_length(be, nodes, i, n_nodes, r.f);
        r.count = !no_fuse && r.nf > 1 ? r.nf : 1;
        r.fused = !no_fuse && (r.nf > 1 || (r.nf == 1 && r.f[0].sharded && be->xg.ok));
        // planned: a device-resident MMA launch that is either local or
        // sharded over the peer exchange (whose gather holds the full output)
        r.planned = r.nf > 0;
        const size_t nseg = r.fused ? r.nf : 1;
        int64_t rows = 0, full = 0;
        size_t nsharded = 0;
        for (size_t j = 0; j < nseg && r.planned; ++j) {
            nsharded += r.f[j].sharded ? 1 : 0;
            rows += r.f[j].seg.N;
            full += r.f[j].n_out;
        }
        if (nsharded > 0)
            r.planned = r.planned && r.fused && nsharded == nseg && be->xg.ok &&
                        static_cast<size_t>(full) <= be->xg.cap_floats;
        r.rows = rows;
        if (r.planned) need = std::max(need, gemv_scratch_bytes(rows, r.f[0].K));
        runs.push_back(r);
        i += r.count;
    }
    if (need > 0 && !backend_xscratch_reserve(be, need)) return false;
    for (Run& r : runs)
        if (r.planned) {
            r.plan.scratch = be->xscratch[be->xscratch_next];
            be->xscratch_next ^= 1;
        }
    for (size_t k = 0; k + 1 < runs.size(); ++k) {
        Run &r = runs[k], &q = runs[k + 1];
        if (!r.planned || !q.planned || r.plan.scratch == q.plan.scratch) continue;
        const size_t nseg = r.fused ? r.nf : 1;
        for (size_t j = 0; j < nseg; ++j)
            if (r.f[j].y_full == q.f[0].x && r.f[j].n_out == q.f[0].K) {
                r.feed.next_scratch = q.plan.scratch;
                r.feed.next_rows = q.rows;
                r.feed.seg = static_cast<int>(j);
                r.feed.bl = mma_blk16(q.f[0].type) ? 16 : 32;
                r.plan.feed = &r.feed;
                q.plan.x_ready = true;
                // both sharded over the exchange: this launch's rows of the
                // next x go to every rank, and the next launch (after waiting
                // for the peers) completes this launch's outputs
                if (r.f[0].sharded && q.f[0].sharded && r.f[j].seg.N % 32 == 0) {
                    r.plan.feed_peers = true;
                    q.plan.nprev = static_cast<int>(nseg);
                    int64_t off = 0;
                    for (size_t s2 = 0; s2 < nseg; ++s2) {
                        q.plan.prev[s2] = GatherSeg{r.f[s2].y_full, r.f[s2].seg.N, off};
                        off += r.f[s2].n_out;
                    }
                }
                break;
            }
    }
    bool ok = true;
    for (size_t k = 0; k < runs.size() && ok; ++k) {
        const Run& r = runs[k];
        const MmaPlan* mp = r.planned ? &r.plan : nullptr;
        ok = r.fused ? run_fused(be, r.f, r.nf, mp) : run_node(be, nodes[r.i], mp);
        for (size_t j = r.i; trace && ok && j < r.i + r.count; ++j)
            fprintf(stderr, "[b200 trace] node %3zu: %-30s | type=%2d | N=%6ld K=%5ld | queued%s%s%s\n", j,
                    nodes[j]->name[0] ? nodes[j]->name : "unnamed", nodes[j]->src[0]->type,
                    long(nodes[j]->src[0]->ne[1]), long(nodes[j]->src[0]->ne[0]), r.count > 1 ? " (fused)" : "",
                    r.plan.x_ready ? " (x from the previous launch)" : "", r.plan.feed ? " (prepares the next x)" : "");
    }
    return ok;
}

// The call on a shadowed list: host inputs in, the list, outputs out.
static bool run_shadowed(Backend* be, const ShadowPlan& sp, size_t n) {
    for (size_t j : sp.in) {
        const Backend::HostShadow& h = be->shadows[j];
        if (!cuda_ok(cudaMemcpyAsync(h.dev, h.host, h.bytes, cudaMemcpyHostToDevice, be->stream), "H2D inputs"))
            return false;
    }
    if (!run_nodes(be, const_cast<ggml_tensor_xdna**>(sp.ptrs.data()), n)) return false;
    for (size_t j : sp.out) {
        const Backend::HostShadow& h = be->shadows[j];
        if (!cuda_ok(cudaMemcpyAsync(h.host, h.dev, h.bytes, cudaMemcpyDeviceToHost, be->stream), "D2H outputs"))
            return false;
    }
    return true;
}

// A node list that comes back unchanged (a decode step) is captured into a
// CUDA graph on its second call and replayed from then on, when every operand
// lives on this device, or is a single F32 row in page-locked host memory
// (run through a device copy, see shadow_host_operands).  The first call
// runs eagerly, so the x scratch and device copies the capture bakes in
// already have their final size.
bool ggml_backend_xdna_compute_graph(ggml_backend_t backend, struct ggml_tensor_xdna** nodes, size_t n_nodes) {
    if (!backend || !nodes || n_nodes == 0) return false;
    Backend* be = as_backend(backend);
    if (!be) return false;
    std::lock_guard<std::mutex> lk(be->mtx);
    DeviceGuard g(be->dev);
    static const bool no_graph = getenv("XDNA_B200_NO_GRAPH") != nullptr || getenv("XDNA_TRACE_NODES") != nullptr;
    // page-locked host operands: run a copy of the list on device copies of them
    std::vector<uint64_t> sig;
    graph_signature(nodes, n_nodes, &sig);
    static thread_local ShadowPlan sp;
    const bool shadowed = shadow_host_operands(be, nodes, n_nodes, sig, true, &sp);
    ggml_tensor_xdna** list = shadowed ? sp.ptrs.data() : nodes;
    auto run_all = [&]() { return shadowed ? run_shadowed(be, sp, n_nodes) : run_nodes(be, nodes, n_nodes); };
    if (!no_graph) {
        if (sig == be->graph_sig && be->graph_ok_sig) {
            if (be->graph_exec && be->graph_gen != be->scratch_gen) drop_graph(be);
            if (!be->graph_exec) {
                cudaGraph_t graph = nullptr;
                bool cap = cudaStreamBeginCapture(be->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
                const bool ran = cap && run_all();
                cap = cudaStreamEndCapture(be->stream, &graph) == cudaSuccess && cap;
                if (ran && cap && graph && cudaGraphInstantiate(&be->graph_exec, graph, 0) == cudaSuccess) {
                    be->graph_gen = be->scratch_gen;
                } else {
                    be->graph_exec = nullptr;
                    be->graph_ok_sig = false;  // run this list eagerly from now on
                }
                if (graph) cudaGraphDestroy(graph);
                cudaGetLastError();
            }
            if (be->graph_exec) {
                const bool ok = cuda_ok(cudaGraphLaunch(be->graph_exec, be->stream), "graph launch");
                return flush(be) && ok;
            }
        } else if (sig != be->graph_sig) {
            drop_graph(be);
            be->graph_sig.swap(sig);
            be->graph_ok_sig = device_only_nodes(be, list, n_nodes);
        }
    }
    const bool ok = run_all();
    const bool flushed = flush(be);
    return ok && flushed;
}

// ---------------------------------------------------------------- buffers
const char* ggml_backend_xdna_buft_name(ggml_backend_buffer_type_t buft) {
    BufferType* t = as_buft(buft);
    return !t ? "" : (t->host ? "B200_Host" : "B200");
}

size_t ggml_backend_xdna_buft_get_alignment(ggml_backend_buffer_type_t buft) {
    (void)buft;
    return kAlignment;
}

size_t ggml_backend_xdna_buft_get_alloc_size(ggml_backend_buffer_type_t buft, const struct ggml_tensor_xdna* tensor) {
    (void)buft;
    return tensor ? tensor_nbytes(tensor) : 0;
}

bool ggml_backend_xdna_buft_is_host(ggml_backend_buffer_type_t buft) {
    BufferType* t = as_buft(buft);
    return t && t->host;
}

ggml_backend_buffer_t ggml_backend_xdna_buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size) {
    BufferType* t = as_buft(buft);
    if (!t) {
        set_error("alloc_buffer: not a B200 buffer type");
        return nullptr;
    }
    if (!t->host && t->dev >= device_count()) {
        set_error("alloc_buffer: CUDA device %d not available", t->dev);
        return nullptr;
    }
    auto b = std::make_unique<Buffer>();
    b->buft = t;
    b->size = size;
    const size_t alloc = size == 0 ? kAlignment : size;
    DeviceGuard g(t->host ? 0 : t->dev);
    const cudaError_t e =
        t->host ? cudaHostAlloc(&b->base, alloc, cudaHostAllocPortable) : cudaMalloc(&b->base, alloc);
    if (e != cudaSuccess) {
        set_error("alloc_buffer(%zu bytes): %s", size, cudaGetErrorString(e));
        cudaGetLastError();
        return nullptr;
    }
    registry().add(b.get());
    return b.release();
}

void ggml_backend_xdna_buffer_free(ggml_backend_buffer_t buffer) {
    Buffer* b = as_buffer(buffer);
    if (!b) return;
    registry().remove(b);
    if (b->owned && b->base) {
        DeviceGuard g(b->buft->host ? 0 : b->buft->dev);
        b->buft->host ? cudaFreeHost(b->base) : cudaFree(b->base);
    }
    b->magic = 0;
    delete b;
}

void* ggml_backend_xdna_buffer_get_base(ggml_backend_buffer_t buffer) {
    Buffer* b = as_buffer(buffer);
    return b ? b->base : nullptr;
}

size_t ggml_backend_xdna_buffer_get_size(ggml_backend_buffer_t buffer) {
    Buffer* b = as_buffer(buffer);
    return b ? b->size : 0;
}

static bool check_tensor_range(Buffer* b, const ggml_tensor_xdna* t, size_t offset, size_t size, const char* what) {
    if (!b || !t || !t->data) {
        set_error("%s: null buffer/tensor", what);
        return false;
    }
    const char* base = static_cast<const char*>(b->base);
    const char* d = static_cast<const char*>(t->data);
    const size_t nbytes = tensor_nbytes(t);
    if (d < base || d + nbytes > base + b->size) {
        set_error("%s: tensor '%s' [%p, +%zu) is not inside the buffer", what, t->name, t->data, nbytes);
        return false;
    }
    if (offset > nbytes || size > nbytes - offset) {
        set_error("%s: range [%zu, +%zu) exceeds tensor '%s' size %zu", what, offset, size, t->name, nbytes);
        return false;
    }
    return true;
}

bool ggml_backend_xdna_buffer_set_tensor(ggml_backend_buffer_t buffer, struct ggml_tensor_xdna* tensor,
                                         const void* data, size_t offset, size_t size) {
    Buffer* b = as_buffer(buffer);
    if (!check_tensor_range(b, tensor, offset, size, "set_tensor")) return false;
    if (size == 0) return true;
    if (!data) {
        set_error("set_tensor: null data");
        return false;
    }
    if (b->buft->host) {
        memcpy(static_cast<char*>(tensor->data) + offset, data, size);
        return true;
    }
    TensorInfo ti;
    tensor_info_for(tensor, &ti);
    {
        std::lock_guard<std::mutex> lk(b->mtx);
        b->tensors[reinterpret_cast<uintptr_t>(tensor->data)] = ti;
    }
    Staging& st = staging_for(b->buft->dev);
    std::lock_guard<std::mutex> lk(st.mtx);
    if (!st.init(b->buft->dev)) return false;
    DeviceGuard g(b->buft->dev);
    if (ti.packed)
        return upload_packed(st, ti, static_cast<uint8_t*>(tensor->data), static_cast<const uint8_t*>(data), offset,
                             size, nullptr);
    return copy_plain(st, static_cast<char*>(tensor->data) + offset, data, nullptr, size);
}

bool ggml_backend_xdna_buffer_set_tensor_device(ggml_backend_buffer_t buffer, struct ggml_tensor_xdna* tensor,
                                                const void* dev_data, size_t offset, size_t size) {
    Buffer* b = as_buffer(buffer);
    if (!check_tensor_range(b, tensor, offset, size, "set_tensor_device")) return false;
    if (size == 0) return true;
    if (!dev_data || b->buft->host) {
        set_error("set_tensor_device: needs device source data and a device buffer");
        return false;
    }
    TensorInfo ti;
    tensor_info_for(tensor, &ti);
    {
        std::lock_guard<std::mutex> lk(b->mtx);
        b->tensors[reinterpret_cast<uintptr_t>(tensor->data)] = ti;
    }
    Staging& st = staging_for(b->buft->dev);
    std::lock_guard<std::mutex> lk(st.mtx);
    if (!st.init(b->buft->dev)) return false;
    DeviceGuard g(b->buft->dev);
    uint8_t* dst = static_cast<uint8_t*>(tensor->data);
    const uint8_t* src = static_cast<const uint8_t*>(dev_data);
    if (!ti.packed) {
        if (!cuda_ok(cudaMemcpyAsync(dst + offset, src, size, cudaMemcpyDeviceToDevice, st.stream), "D2D")) return false;
        return cuda_ok(cudaStreamSynchronize(st.stream), "D2D sync");
    }
    for (const Chunk& c : chunks_for(ti, offset, size, st.slot_bytes)) {
        const size_t w0 = std::max(offset, c.byte0), w1 = std::min(offset + size, c.byte0 + c.bytes);
        if (w0 == c.byte0 && w1 == c.byte0 + c.bytes) {  // whole chunk: repack straight from the source
            if (!cuda_ok(repack_launch(ti.type, src + (w0 - offset), dst + c.byte0, ti.N, ti.K, c.row0, c.nrows,
                                       st.stream),
                         "repack"))
                return false;
            continue;
        }
        const int s = st.acquire();
        uint8_t* raw = static_cast<uint8_t*>(st.devbuf[s]);
        if (!cuda_ok(unpack_launch(ti.type, dst + c.byte0, raw, ti.N, ti.K, c.row0, c.nrows, st.stream), "unpack") ||
            !cuda_ok(cudaMemcpyAsync(raw + (w0 - c.byte0), src + (w0 - offset), w1 - w0, cudaMemcpyDeviceToDevice,
                                     st.stream),
                     "D2D") ||
            !cuda_ok(repack_launch(ti.type, raw, dst + c.byte0, ti.N, ti.K, c.row0, c.nrows, st.stream), "repack"))
            return false;
        cudaEventRecord(st.done[s], st.stream);
    }
    return cuda_ok(cudaStreamSynchronize(st.stream), "set_tensor_device sync");
}

bool ggml_backend_xdna_buffer_cpy_tensor(const struct ggml_tensor_xdna* src, struct ggml_tensor_xdna* dst) {
    if (!src || !dst || !src->data || !dst->data) {
        set_error("cpy_tensor: null tensor");
        return false;
    }
    Buffer* bs = registry().find(src->data);
    Buffer* bd = registry().find(dst->data);
    if (!bs || !bd || bs->buft->host || bd->buft->host || bs->buft->dev != bd->buft->dev) {
        set_error("cpy_tensor: both tensors must live in B200 device buffers of one GPU");
        return false;
    }
    const size_t n = tensor_nbytes(src);
    if (src->type != dst->type || n != tensor_nbytes(dst) || src->ne[0] != dst->ne[0] || src->ne[1] != dst->ne[1]) {
        set_error("cpy_tensor: '%s' and '%s' differ in type or shape", src->name, dst->name);
        return false;
    }
    if (!check_tensor_range(bd, dst, 0, n, "cpy_tensor")) return false;
    TensorInfo ti;
    {
        std::lock_guard<std::mutex> lk(bs->mtx);
        auto it = bs->tensors.find(reinterpret_cast<uintptr_t>(src->data));
        if (it == bs->tensors.end()) {
            set_error("cpy_tensor: source '%s' was never written", src->name);
            return false;
        }
        ti = it->second;
    }
    {
        std::lock_guard<std::mutex> lk(bd->mtx);
        bd->tensors[reinterpret_cast<uintptr_t>(dst->data)] = ti;
    }
    DeviceGuard g(bd->buft->dev);
    // both tensors share the stripe layout, so the copy is byte for byte
    return cuda_ok(cudaMemcpy(dst->data, src->data, n, cudaMemcpyDeviceToDevice), "cpy_tensor");
}

bool ggml_backend_xdna_buffer_get_tensor(ggml_backend_buffer_t buffer, const struct ggml_tensor_xdna* tensor,
                                         void* data, size_t offset, size_t size) {
    Buffer* b = as_buffer(buffer);
    if (!check_tensor_range(b, tensor, offset, size, "get_tensor")) return false;
    if (size == 0) return true;
    if (!data) {
        set_error("get_tensor: null data");
        return false;
    }
    if (b->buft->host) {
        memcpy(data, static_cast<const char*>(tensor->data) + offset, size);
        return true;
    }
    TensorInfo ti;
    bool known = false;
    {
        std::lock_guard<std::mutex> lk(b->mtx);
        auto it = b->tensors.find(reinterpret_cast<uintptr_t>(tensor->data));
        if (it != b->tensors.end()) {
            ti = it->second;
            known = true;
        }
    }
    Staging& st = staging_for(b->buft->dev);
    std::lock_guard<std::mutex> lk(st.mtx);
    if (!st.init(b->buft->dev)) return false;
    DeviceGuard g(b->buft->dev);
    if (known && ti.packed)
        return download_packed(st, ti, static_cast<const uint8_t*>(tensor->data), static_cast<uint8_t*>(data), offset,
                               size);
    return copy_plain(st, static_cast<char*>(tensor->data) + offset, nullptr, data, size);
}

bool ggml_backend_xdna_buffer_memset_tensor(ggml_backend_buffer_t buffer, struct ggml_tensor_xdna* tensor,
                                            uint8_t value, size_t offset, size_t size) {
    Buffer* b = as_buffer(buffer);
    if (!check_tensor_range(b, tensor, offset, size, "memset_tensor")) return false;
    if (size == 0) return true;
    if (b->buft->host) {
        memset(static_cast<char*>(tensor->data) + offset, value, size);
        return true;
    }
    TensorInfo ti;
    tensor_info_for(tensor, &ti);
    {
        std::lock_guard<std::mutex> lk(b->mtx);
        b->tensors[reinterpret_cast<uintptr_t>(tensor->data)] = ti;
    }
    Staging& st = staging_for(b->buft->dev);
    std::lock_guard<std::mutex> lk(st.mtx);
    if (!st.init(b->buft->dev)) return false;
    DeviceGuard g(b->buft->dev);
    if (ti.packed)
        return upload_packed(st, ti, static_cast<uint8_t*>(tensor->data), nullptr, offset, size, &value);
    if (!cuda_ok(cudaMemsetAsync(static_cast<char*>(tensor->data) + offset, value, size, st.stream), "memset"))
        return false;
    return cuda_ok(cudaStreamSynchronize(st.stream), "memset sync");
}

bool ggml_backend_xdna_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value) {
    Buffer* b = as_buffer(buffer);
    if (!b) return false;
    if (b->buft->host) {
        if (b->size) memset(b->base, value, b->size);
        return true;
    }
    DeviceGuard g(b->buft->dev);
    if (b->size && !cuda_ok(cudaMemset(b->base, value, b->size), "clear")) return false;
    // Every byte of the GGUF view is now `value`.  Every kernel layout is a
    // permutation of the GGUF bits, so 0x00 and 0xFF read back unchanged; any
    // other value reads back permuted (nibbles re-paired, bit planes
    // transposed), so packed tensors are rewritten through the repack.
    if (value == 0x00 || value == 0xFF) return true;
    std::vector<std::pair<uintptr_t, TensorInfo>> fix;
    {
        std::lock_guard<std::mutex> lk(b->mtx);
        for (auto& kv : b->tensors)
            if (kv.second.packed) fix.push_back(kv);
    }
    if (fix.empty()) return true;
    Staging& st = staging_for(b->buft->dev);
    std::lock_guard<std::mutex> lk(st.mtx);
    if (!st.init(b->buft->dev)) return false;
    for (auto& kv : fix)
        if (!upload_packed(st, kv.second, reinterpret_cast<uint8_t*>(kv.first), nullptr, 0,
                           kv.second.mat_bytes * kv.second.nmat, &value))
            return false;
    return true;
}

// ---------------------------------------------------------------- launcher
static int launch_rc(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 0;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return -static_cast<int>(e);
}

int b200_gemv(int type, const void* w_packed, const float* x, float* y, int64_t n, int64_t k, void* stream,
              int pdl) {
    const FormatInfo f = format_info(type);
    if (!f.block_vals || k < 0 || k % f.block_vals || n < 0) {
        set_error("b200_gemv: bad type %d / shape N=%ld K=%ld", type, long(n), long(k));
        return -1;
    }
    if (n > 0 && (!w_packed || !x || !y)) {
        set_error("b200_gemv: null pointer");
        return -1;
    }
    if (reinterpret_cast<uintptr_t>(x) & 15u) {
        set_error("b200_gemv: x must be 16-byte aligned");
        return -1;
    }
    LaunchOpts lo;
    lo.pdl = pdl != 0;
    return launch_rc(gemv_launch(type, w_packed, x, y, n, k, static_cast<cudaStream_t>(stream), lo), "b200_gemv");
}

int b200_gemv_multi(int type, const void* const* w_packed, float* const* y, const int64_t* n, int nseg, const float* x,
                    int64_t k, void* stream, int pdl) {
    if (nseg < 1 || nseg > MMA_MAX_SEGMENTS || !w_packed || !y || !n || !x) {
        set_error("b200_gemv_multi: bad segment list (1..%d matrices)", MMA_MAX_SEGMENTS);
        return -1;
    }
    if (reinterpret_cast<uintptr_t>(x) & 15u) {
        set_error("b200_gemv_multi: x must be 16-byte aligned");
        return -1;
    }
    MmaSegment segs[MMA_MAX_SEGMENTS];
    int64_t rows = 0;
    for (int s = 0; s < nseg; ++s) {
        if (!w_packed[s] || !y[s] || layout_kind(type, n[s], k) != 1) {
            set_error("b200_gemv_multi: matrix %d (type %d, N=%ld, K=%ld) is not in the 16-row MMA layout "
                      "(N %% 16 == 0 and K %% 256 == 0)",
                      s, type, long(n[s]), long(k));
            return -1;
        }
        segs[s] = MmaSegment{w_packed[s], y[s], n[s]};
        rows += n[s];
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* scratch = launcher_scratch(st, rows, k);
    if (!scratch) return launch_rc(cudaErrorMemoryAllocation, "b200_gemv_multi scratch");
    return launch_rc(gemv_mma_multi_launch(type, segs, nseg, x, k, scratch, st, pdl != 0), "b200_gemv_multi");
}

// b200_gemv without device allocation (see the declaration): the MMA path
// gets the static-array scratch instead of launcher_scratch's buffers.
int b200_gemv_noalloc(int type, const void* w_packed, const float* x, float* y, int64_t n, int64_t k, void* stream) {
    const FormatInfo f = format_info(type);
    if (!f.block_vals || k < 0 || k % f.block_vals || n < 0) {
        set_error("b200_gemv_noalloc: bad type %d / shape N=%ld K=%ld", type, long(n), long(k));
        return -1;
    }
    if (n > 0 && (!w_packed || !x || !y)) {
        set_error("b200_gemv_noalloc: null pointer");
        return -1;
    }
    if (reinterpret_cast<uintptr_t>(x) & 15u) {
        set_error("b200_gemv_noalloc: x must be 16-byte aligned");
        return -1;
    }
    LaunchOpts lo;
    if (n > 0 && layout_kind(type, n, k) == 1) {
        const size_t need = xprep_bytes(n, k);
        if (need > static_scratch_bytes()) {
            set_error("b200_gemv_noalloc: N=%ld K=%ld needs %zu bytes of scratch, more than its fixed %zu-byte "
                      "area (fits N <= 131072 with K <= 32768); use b200_gemv",
                      long(n), long(k), need, static_scratch_bytes());
            return -1;
        }
        void* s = nullptr;
        const cudaError_t e = static_scratch(&s);
        if (e != cudaSuccess) return launch_rc(e, "b200_gemv_noalloc: cudaGetSymbolAddress");
        lo.scratch = s;
        lo.classic = true;  // the fixed area is sized for the classic kernel's scratch
    }
    return launch_rc(gemv_launch(type, w_packed, x, y, n, k, static_cast<cudaStream_t>(stream), lo),
                     "b200_gemv_noalloc");
}

int b200_gemv_error(int* status) {
    if (!status) {
        set_error("b200_gemv_error: null status pointer");
        return -1;
    }
    return launch_rc(gemv_error_status(status), "b200_gemv_error");
}

int b200_repack(int type, const void* raw, void* packed, int64_t n, int64_t k, void* stream) {
    return launch_rc(repack_launch(type, raw, packed, n, k, 0, n, static_cast<cudaStream_t>(stream)), "b200_repack");
}

int b200_unpack(int type, const void* packed, void* raw, int64_t n, int64_t k, void* stream) {
    return launch_rc(unpack_launch(type, packed, raw, n, k, 0, n, static_cast<cudaStream_t>(stream)), "b200_unpack");
}

int b200_bf16_to_f32(const uint16_t* src, float* dst, int64_t n, void* stream) {
    return launch_rc(bf16_to_f32_launch(src, dst, n, static_cast<cudaStream_t>(stream)), "b200_bf16_to_f32");
}

// F32 copy of a BF16 activation row, one growing buffer per (device, stream);
// the conversion kernel and the GEMV that reads it are ordered on the stream.
static float* bf16_staging(cudaStream_t stream, int64_t k) {
    static std::mutex m;
    static std::map<std::pair<int, cudaStream_t>, std::pair<float*, int64_t>> bufs;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(m);
    auto& b = bufs[{dev, stream}];
    if (b.second < k) {
        if (b.first) {
            cudaStreamSynchronize(stream);
            cudaFree(b.first);
        }
        b = {nullptr, 0};
        const int64_t cap = std::max<int64_t>(k, 16384);
        if (cudaMalloc(&b.first, static_cast<size_t>(cap) * sizeof(float)) != cudaSuccess) return nullptr;
        b.second = cap;
    }
    return b.first;
}

int b200_gemv_bf16(int type, const void* w_packed, const uint16_t* x_bf16, float* y, int64_t n, int64_t k, void* stream,
                   int pdl) {
    const FormatInfo f = format_info(type);
    if (!f.block_vals || k < 0 || k % f.block_vals || n < 0) {
        set_error("b200_gemv_bf16: bad type %d / shape N=%ld K=%ld", type, long(n), long(k));
        return -1;
    }
    if (n > 0 && (!w_packed || !x_bf16 || !y)) {
        set_error("b200_gemv_bf16: null pointer");
        return -1;
    }
    if (n == 0) return 0;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* xf = bf16_staging(st, k);
    if (!xf) return launch_rc(cudaErrorMemoryAllocation, "b200_gemv_bf16 staging");
    const int rc = launch_rc(bf16_to_f32_launch(x_bf16, xf, k, st), "b200_gemv_bf16 convert");
    if (rc) return rc;
    LaunchOpts lo;
    lo.pdl = pdl != 0;
    return launch_rc(gemv_launch(type, w_packed, xf, y, n, k, st, lo), "b200_gemv_bf16");
}

int b200_fill_normal(float* out, int64_t n, uint64_t seed, float sigma, void* stream) {
    return launch_rc(fill_normal_launch(out, n, seed, sigma, static_cast<cudaStream_t>(stream)), "b200_fill_normal");
}

int b200_quantize(int type, const float* src, void* dst, int64_t n, int64_t k, void* stream) {
    return launch_rc(quantize_launch(type, src, dst, n, k, static_cast<cudaStream_t>(stream)), "b200_quantize");
}

static int host_repack(int type, const void* src, void* dst, int64_t n, int64_t k, bool pack) {
    const FormatInfo f = format_info(type);
    if (!f.block_vals || k < 0 || k % f.block_vals || n < 0 || (n > 0 && (!src || !dst))) {
        set_error("b200_%s_host: bad arguments", pack ? "repack" : "unpack");
        return -1;
    }
    if (layout_kind(type, n, k) == 1) {
        const size_t rb = static_cast<size_t>(k / 256) * mma_row_group_bytes(type);
        const size_t gb = static_cast<size_t>(mma_group_bytes(type));
        for (int64_t t = 0; t < n / MMA_TILE_ROWS; ++t)
            for (int64_t gi = 0; gi < k / 256; ++gi) {
                const size_t tb = static_cast<size_t>(t) * MMA_TILE_ROWS * rb;
                if (pack)
                    mma_pack_group(type, static_cast<const uint8_t*>(src) + tb, rb, gi,
                                   static_cast<uint8_t*>(dst) + tb + gi * gb);
                else
                    mma_unpack_group(type, static_cast<const uint8_t*>(src) + tb + gi * gb, rb, gi,
                                     static_cast<uint8_t*>(dst) + tb);
            }
        return 0;
    }
    const Geometry g = make_geometry(type, n, k);
    for (int64_t t = 0; t < g.ntiles; ++t) {
        const int tr = static_cast<int>(std::min<int64_t>(TILE_ROWS, n - t * TILE_ROWS));
        const size_t base = static_cast<size_t>(t) * TILE_ROWS * g.row_bytes;
        for (int r = 0; r < tr; ++r)
            for (int64_t b = 0; b < g.nb; ++b) {
                if (pack)
                    repack_one(g, tr, r, b, static_cast<const uint8_t*>(src) + base, static_cast<uint8_t*>(dst) + base);
                else
                    unrepack_one(g, tr, r, b, static_cast<const uint8_t*>(src) + base, static_cast<uint8_t*>(dst) + base);
            }
    }
    return 0;
}

int b200_repack_host(int type, const void* raw, void* packed, int64_t n, int64_t k) {
    return host_repack(type, raw, packed, n, k, true);
}

int b200_unpack_host(int type, const void* packed, void* raw, int64_t n, int64_t k) {
    return host_repack(type, packed, raw, n, k, false);
}

size_t b200_row_bytes(int type, int64_t k) {
    size_t rb = 0;
    return (k >= 0 && row_bytes_for(type, k, &rb)) ? rb : 0;
}

size_t b200_gemv_smem_bytes(int type, int64_t k) { return gemv_smem_bytes(type, k); }

}  // extern "C"
