// ggml backend plugin over the B200 compat ABI: libggml-b200-ggml.so.
//
// Pointing GGML_BACKEND_PATH at this library makes each CUDA GPU an
// ordinary ggml device ("B200<n>") that claims the reference's MUL_MAT set
// and runs it through libggml-b200.so.  It is the counterpart of the
// reference's ggml plugin surface (src/ggml-xdna.cpp:316-730 and the API v3
// entry points at :719-823):
//
//   ggml_backend_init / ggml_backend_score   dynamic-load entry (reference :721-730)
//   registry    one device per CUDA GPU (the reference exposes one NPU)
//   device      name, memory (cudaMemGetInfo through the engine), type ACCEL,
//               props, init_backend, buffer types, supports_op / supports_buft
//   buffer type HBM buffers of the engine (is_host false: weights live on the
//               GPU and are repacked on upload), plus its pinned host type
//   buffer      free / get_base / init_tensor / memset / set / get / cpy / clear
//               forwarded to ggml_backend_xdna_buffer_* with the tensor's
//               compat record
//   backend     get_name / free / synchronize / graph_compute; graph_compute
//               converts the graph's MUL_MAT nodes (ggml-b200-convert.h) and
//               calls ggml_backend_xdna_compute_graph
//
// Built only against a ggml tree (XDNA_LLAMA_CPP_DIR; see build.py), as the
// reference builds its plugin only when ggml headers are found
// (CMakeLists.txt:293-311).  The interface tables are filled field by field,
// by name, so the source does not depend on the order of the fields in a
// given ggml version.
#include "ggml-backend-impl.h"
#include "ggml-backend.h"
#include "ggml.h"

// The engine's C ABI declares its own ggml-free handle typedefs and enums;
// scoped in a namespace they do not meet ggml's (the functions keep their C
// names).
namespace b200 {
#include "ggml-b200.h"
}
#include "ggml-b200-convert.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace {

using XT = b200::ggml_tensor_xdna;

struct DeviceCtx {
    int index = 0;
    std::string name, description;
    ggml_backend_buffer_type buft;       // HBM buffers of this GPU
    ggml_backend_buffer_type host_buft;  // pinned host buffers
};

struct BackendCtx {
    b200::ggml_backend_t engine = nullptr;
    b200_convert::NodeBatch<XT> batch;
    std::mutex mtx;
};

// The registry and its devices, built on first use.
struct Registry {
    ggml_backend_reg reg;
    std::vector<DeviceCtx> ctxs;
    std::vector<ggml_backend_device> devs;
};

const ggml_guid* b200_guid() {
    static ggml_guid guid = {0x42, 0x32, 0x30, 0x30, 0x67, 0x67, 0x6d, 0x6c,
                             0x2d, 0x61, 0x64, 0x61, 0x70, 0x74, 0x65, 0x72};  // "B200ggml-adapter"
    return &guid;
}

Registry& registry();

// ------------------------------------------------------------------ buffers
XT record(const ggml_tensor* t) {
    XT x;
    b200_convert::copy_tensor(*t, x);
    return x;
}

b200::ggml_backend_buffer_t engine_buffer(ggml_backend_buffer_t buffer) {
    return static_cast<b200::ggml_backend_buffer_t>(buffer->context);
}

void buf_free(ggml_backend_buffer_t buffer) { b200::ggml_backend_xdna_buffer_free(engine_buffer(buffer)); }

void* buf_get_base(ggml_backend_buffer_t buffer) { return b200::ggml_backend_xdna_buffer_get_base(engine_buffer(buffer)); }

ggml_status buf_init_tensor(ggml_backend_buffer_t, ggml_tensor*) { return GGML_STATUS_SUCCESS; }

void buf_memset_tensor(ggml_backend_buffer_t buffer, ggml_tensor* tensor, uint8_t value, size_t offset, size_t size) {
    XT x = record(tensor);
    if (!b200::ggml_backend_xdna_buffer_memset_tensor(engine_buffer(buffer), &x, value, offset, size))
        GGML_ABORT("b200: memset_tensor failed: %s", b200::ggml_backend_xdna_last_error());
}

void buf_set_tensor(ggml_backend_buffer_t buffer, ggml_tensor* tensor, const void* data, size_t offset, size_t size) {
    XT x = record(tensor);
    if (!b200::ggml_backend_xdna_buffer_set_tensor(engine_buffer(buffer), &x, data, offset, size))
        GGML_ABORT("b200: set_tensor failed: %s", b200::ggml_backend_xdna_last_error());
}

void buf_get_tensor(ggml_backend_buffer_t buffer, const ggml_tensor* tensor, void* data, size_t offset, size_t size) {
    XT x = record(tensor);
    if (!b200::ggml_backend_xdna_buffer_get_tensor(engine_buffer(buffer), &x, data, offset, size))
        GGML_ABORT("b200: get_tensor failed: %s", b200::ggml_backend_xdna_last_error());
}

bool buf_cpy_tensor(ggml_backend_buffer_t, const ggml_tensor* src, ggml_tensor* dst) {
    // both in B200 buffers of one GPU (the engine checks); ggml copies other
    // pairs through the host
    XT s = record(src), d = record(dst);
    return b200::ggml_backend_xdna_buffer_cpy_tensor(&s, &d);
}

void buf_clear(ggml_backend_buffer_t buffer, uint8_t value) {
    if (!b200::ggml_backend_xdna_buffer_clear(engine_buffer(buffer), value))
        GGML_ABORT("b200: clear failed: %s", b200::ggml_backend_xdna_last_error());
}

const ggml_backend_buffer_i& buffer_iface() {
    static const ggml_backend_buffer_i iface = [] {
        ggml_backend_buffer_i i;
        std::memset(static_cast<void*>(&i), 0, sizeof i);
        i.free_buffer = buf_free;
        i.get_base = buf_get_base;
        i.init_tensor = buf_init_tensor;
        i.memset_tensor = buf_memset_tensor;
        i.set_tensor = buf_set_tensor;
        i.get_tensor = buf_get_tensor;
        i.cpy_tensor = buf_cpy_tensor;
        i.clear = buf_clear;
        return i;
    }();
    return iface;
}

// ------------------------------------------------------------- buffer types
// context: the engine's buffer type handle
b200::ggml_backend_buffer_type_t engine_buft(ggml_backend_buffer_type_t buft) {
    return static_cast<b200::ggml_backend_buffer_type_t>(buft->context);
}

const char* buft_get_name(ggml_backend_buffer_type_t buft) { return b200::ggml_backend_xdna_buft_name(engine_buft(buft)); }

ggml_backend_buffer_t buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size) {
    b200::ggml_backend_buffer_t eb = b200::ggml_backend_xdna_buft_alloc_buffer(engine_buft(buft), size ? size : 1);
    if (!eb) {
        fprintf(stderr, "[b200 error] alloc_buffer(%zu): %s\n", size, b200::ggml_backend_xdna_last_error());
        return nullptr;
    }
    return ggml_backend_buffer_init(buft, buffer_iface(), eb, size);
}

size_t buft_get_alignment(ggml_backend_buffer_type_t buft) {
    return b200::ggml_backend_xdna_buft_get_alignment(engine_buft(buft));
}

size_t buft_get_max_size(ggml_backend_buffer_type_t) { return SIZE_MAX; }

size_t buft_get_alloc_size(ggml_backend_buffer_type_t buft, const ggml_tensor* tensor) {
    XT x = record(tensor);
    return b200::ggml_backend_xdna_buft_get_alloc_size(engine_buft(buft), &x);
}

bool buft_is_host(ggml_backend_buffer_type_t buft) { return b200::ggml_backend_xdna_buft_is_host(engine_buft(buft)); }

const ggml_backend_buffer_type_i& buft_iface() {
    static const ggml_backend_buffer_type_i iface = [] {
        ggml_backend_buffer_type_i i;
        std::memset(static_cast<void*>(&i), 0, sizeof i);
        i.get_name = buft_get_name;
        i.alloc_buffer = buft_alloc_buffer;
        i.get_alignment = buft_get_alignment;
        i.get_max_size = buft_get_max_size;
        i.get_alloc_size = buft_get_alloc_size;
        i.is_host = buft_is_host;
        return i;
    }();
    return iface;
}

bool ours(ggml_backend_buffer_type_t buft) {
    if (!buft) return false;
    for (const DeviceCtx& d : registry().ctxs)
        if (buft == &d.buft || buft == &d.host_buft) return true;
    return false;
}

// ------------------------------------------------------------------ backend
BackendCtx* backend_ctx(ggml_backend_t backend) {
    if (!backend || !backend->guid || std::memcmp(backend->guid, b200_guid(), sizeof(ggml_guid)) != 0) return nullptr;
    return static_cast<BackendCtx*>(backend->context);
}

const char* backend_get_name(ggml_backend_t backend) { return backend->device->iface.get_name(backend->device); }

void backend_free(ggml_backend_t backend) {
    BackendCtx* ctx = backend_ctx(backend);
    if (ctx) {
        b200::ggml_backend_xdna_free(ctx->engine);
        delete ctx;
    }
    delete backend;
}

void backend_synchronize(ggml_backend_t backend) {
    BackendCtx* ctx = backend_ctx(backend);
    if (ctx) b200::ggml_backend_xdna_synchronize(ctx->engine);
}

// The graph's MUL_MAT nodes, as the compat ABI's records, in one
// compute_graph call (the engine fuses, chains and replays them); the other
// nodes belong to the backends ggml's scheduler gave them to.
ggml_status backend_graph_compute(ggml_backend_t backend, ggml_cgraph* cgraph) {
    BackendCtx* ctx = backend_ctx(backend);
    if (!ctx || !cgraph) return GGML_STATUS_FAILED;
    std::lock_guard<std::mutex> lk(ctx->mtx);
    const int n = ggml_graph_n_nodes(cgraph);
    const size_t m = ctx->batch.convert<ggml_tensor>(n, [&](int i) { return ggml_graph_node(cgraph, i); },
                                                     GGML_OP_MUL_MAT);
    if (m == 0) return GGML_STATUS_SUCCESS;
    if (!b200::ggml_backend_xdna_compute_graph(ctx->engine, ctx->batch.nodes(), m)) {
        fprintf(stderr, "[b200 error] graph_compute: %s\n", b200::ggml_backend_xdna_last_error());
        return GGML_STATUS_FAILED;
    }
    return GGML_STATUS_SUCCESS;
}

const ggml_backend_i& backend_iface() {
    static const ggml_backend_i iface = [] {
        ggml_backend_i i;
        std::memset(static_cast<void*>(&i), 0, sizeof i);
        i.get_name = backend_get_name;
        i.free = backend_free;
        i.synchronize = backend_synchronize;
        i.graph_compute = backend_graph_compute;
        return i;
    }();
    return iface;
}

// ------------------------------------------------------------------ devices
DeviceCtx& dev_ctx(ggml_backend_dev_t dev) { return *static_cast<DeviceCtx*>(dev->context); }

const char* dev_get_name(ggml_backend_dev_t dev) { return dev_ctx(dev).name.c_str(); }

const char* dev_get_description(ggml_backend_dev_t dev) { return dev_ctx(dev).description.c_str(); }

void dev_get_memory(ggml_backend_dev_t dev, size_t* free_bytes, size_t* total_bytes) {
    b200::ggml_backend_xdna_get_device_memory(static_cast<size_t>(dev_ctx(dev).index), free_bytes, total_bytes);
}

ggml_backend_dev_type dev_get_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_ACCEL; }

void dev_get_props(ggml_backend_dev_t dev, ggml_backend_dev_props* props) {
    props->name = dev_get_name(dev);
    props->description = dev_get_description(dev);
    props->type = dev_get_type(dev);
    dev_get_memory(dev, &props->memory_free, &props->memory_total);
    props->caps.async = false;                 // graph_compute returns with its outputs complete
    props->caps.host_buffer = true;            // pinned staging buffers
    props->caps.buffer_from_host_ptr = false;  // weights are repacked into HBM on upload
    props->caps.events = false;
}

ggml_backend_t dev_init_backend(ggml_backend_dev_t dev, const char*) {
    b200::ggml_backend_t engine = b200::ggml_backend_xdna_init(static_cast<size_t>(dev_ctx(dev).index));
    if (!engine) {
        fprintf(stderr, "[b200 error] init_backend: %s\n", b200::ggml_backend_xdna_last_error());
        return nullptr;
    }
    auto* ctx = new BackendCtx();
    ctx->engine = engine;
    auto* be = new ggml_backend();
    be->guid = const_cast<ggml_guid_t>(b200_guid());
    be->iface = backend_iface();
    be->device = dev;
    be->context = ctx;
    return be;
}

ggml_backend_buffer_type_t dev_get_buffer_type(ggml_backend_dev_t dev) { return &dev_ctx(dev).buft; }

ggml_backend_buffer_type_t dev_get_host_buffer_type(ggml_backend_dev_t dev) { return &dev_ctx(dev).host_buft; }

// The reference's claim predicate (src/ggml-xdna.cpp:95-147) through the
// engine; a node whose weights live in this plugin's HBM buffers is claimed
// for any row count, as the reference claims rows for its own buffers.
bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor* op) {
    XT x, srcs[2];
    if (!op || op->op != GGML_OP_MUL_MAT) return false;
    const bool resident = op->src[0] && op->src[0]->buffer && ours(op->src[0]->buffer->buft) &&
                          !ggml_backend_buffer_is_host(op->src[0]->buffer);
    if (!b200_convert::convert_op(*op, GGML_OP_MUL_MAT, x, srcs, resident)) return false;
    return b200::ggml_backend_xdna_supports_op(nullptr, &x);
}

bool dev_supports_buft(ggml_backend_dev_t, ggml_backend_buffer_type_t buft) {
    // this plugin's buffers, and host memory for activations (staged by the engine)
    return ours(buft) || ggml_backend_buft_is_host(buft);
}

bool dev_offload_op(ggml_backend_dev_t, const ggml_tensor*) {
    return false;  // weights belong in HBM buffers; nothing is worth a per-call upload
}

const ggml_backend_device_i& device_iface() {
    static const ggml_backend_device_i iface = [] {
        ggml_backend_device_i i;
        std::memset(static_cast<void*>(&i), 0, sizeof i);
        i.get_name = dev_get_name;
        i.get_description = dev_get_description;
        i.get_memory = dev_get_memory;
        i.get_type = dev_get_type;
        i.get_props = dev_get_props;
        i.init_backend = dev_init_backend;
        i.get_buffer_type = dev_get_buffer_type;
        i.get_host_buffer_type = dev_get_host_buffer_type;
        i.supports_op = dev_supports_op;
        i.supports_buft = dev_supports_buft;
        i.offload_op = dev_offload_op;
        return i;
    }();
    return iface;
}

// ----------------------------------------------------------------- registry
const char* reg_get_name(ggml_backend_reg_t) { return "B200"; }

size_t reg_get_device_count(ggml_backend_reg_t) { return registry().devs.size(); }

ggml_backend_dev_t reg_get_device(ggml_backend_reg_t, size_t index) {
    Registry& r = registry();
    return index < r.devs.size() ? &r.devs[index] : nullptr;
}

// The compat entry points, by name, as the reference's registry exposes its
// own (src/ggml-xdna.cpp:645-660).
void* reg_get_proc_address(ggml_backend_reg_t, const char* name) {
    if (!name) return nullptr;
    struct Entry {
        const char* name;
        void* fn;
    };
    static const Entry entries[] = {
        {"ggml_backend_xdna_init", reinterpret_cast<void*>(b200::ggml_backend_xdna_init)},
        {"ggml_backend_is_xdna", reinterpret_cast<void*>(b200::ggml_backend_is_xdna)},
        {"ggml_backend_xdna_free", reinterpret_cast<void*>(b200::ggml_backend_xdna_free)},
        {"ggml_backend_xdna_compute_graph", reinterpret_cast<void*>(b200::ggml_backend_xdna_compute_graph)},
        {"ggml_backend_xdna_supports_op", reinterpret_cast<void*>(b200::ggml_backend_xdna_supports_op)},
    };
    for (const Entry& e : entries)
        if (!std::strcmp(name, e.name)) return e.fn;
    return nullptr;
}

Registry& registry() {
    static Registry* r = [] {
        auto* reg = new Registry();
        reg->reg.api_version = GGML_BACKEND_API_VERSION;
        std::memset(static_cast<void*>(&reg->reg.iface), 0, sizeof reg->reg.iface);
        reg->reg.iface.get_name = reg_get_name;
        reg->reg.iface.get_device_count = reg_get_device_count;
        reg->reg.iface.get_device = reg_get_device;
        reg->reg.iface.get_proc_address = reg_get_proc_address;
        reg->reg.context = nullptr;
        const size_t n = b200::ggml_backend_xdna_get_device_count();
        reg->ctxs.resize(n);
        reg->devs.resize(n);
        for (size_t k = 0; k < n; ++k) {
            DeviceCtx& d = reg->ctxs[k];
            d.index = static_cast<int>(k);
            d.name = "B200" + std::to_string(k);
            d.description = "NVIDIA B200 (decode GEMV, CUDA device " + std::to_string(k) + ")";
            d.buft.iface = buft_iface();
            d.buft.device = &reg->devs[k];
            d.buft.context = b200::ggml_backend_xdna_buffer_type(k);
            d.host_buft.iface = buft_iface();
            d.host_buft.device = &reg->devs[k];
            d.host_buft.context = b200::ggml_backend_xdna_host_buffer_type();
            reg->devs[k].iface = device_iface();
            reg->devs[k].reg = &reg->reg;
            reg->devs[k].context = &d;
        }
        return reg;
    }();
    return *r;
}

}  // namespace

extern "C" {

// Dynamic-load entry points of a ggml backend library (reference
// include/xdna/ggml-xdna.h:147-148, src/ggml-xdna.cpp:721-730).
GGML_BACKEND_API ggml_backend_reg_t ggml_backend_init(void) { return &registry().reg; }

// Preferred over the CPU backend when a GPU is present.
GGML_BACKEND_API int ggml_backend_score(void) { return registry().devs.empty() ? 0 : 100; }

// The ggml-API graph entry of the reference's header (ggml-xdna.h:151),
// for callers that hold a ggml backend of this plugin.
GGML_BACKEND_API enum ggml_status ggml_backend_b200_graph_compute(ggml_backend_t backend, struct ggml_cgraph* cgraph) {
    return backend_graph_compute(backend, cgraph);
}

}  // extern "C"
