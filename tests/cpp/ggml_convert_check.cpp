// CPU check of include/ggml-b200-convert.h, the ggml -> compat-record
// conversion of the ggml adapter, with a stand-in tensor type that has the
// field names the helpers read.  Converted MUL_MAT nodes go through the
// library's claim predicate (ggml_backend_xdna_supports_op, no GPU needed).
#include <cassert>
#include <cstdio>
#include <cstring>

#include "ggml-b200-convert.h"
#include "ggml-b200.h"

namespace {

// A graph node as a ggml-like front end holds it: ggml's own op numbering
// (MUL_MAT is not 18 there), type ids as in ggml.h.
constexpr int kHostMulMat = 29, kHostAdd = 2, kHostNorm = 7;

struct HostTensor {
    int type;
    long long ne[4];
    unsigned long nb[4];
    int op;
    HostTensor* src[10];
    void* data;
    char name[64];
};

HostTensor tensor(int type, long long ne0, long long ne1, long long ne2, long long ne3, size_t ts, size_t blk,
                  void* data, const char* name) {
    HostTensor t;
    std::memset(&t, 0, sizeof t);
    t.type = type;
    t.ne[0] = ne0;
    t.ne[1] = ne1;
    t.ne[2] = ne2;
    t.ne[3] = ne3;
    t.nb[0] = ts;
    t.nb[1] = ts * (ne0 / blk);
    t.nb[2] = t.nb[1] * ne1;
    t.nb[3] = t.nb[2] * ne2;
    t.data = data;
    std::snprintf(t.name, sizeof t.name, "%s", name);
    return t;
}

int fails = 0;
#define CHECK(c)                                                       \
    do {                                                               \
        if (!(c)) {                                                    \
            std::fprintf(stderr, "FAIL %s:%d %s\n", __FILE__, __LINE__, #c); \
            ++fails;                                                   \
        }                                                              \
    } while (0)

void same_tensor(const ggml_tensor_xdna& x, const HostTensor& h) {
    CHECK(static_cast<int>(x.type) == h.type);
    for (int d = 0; d < 4; ++d) {
        CHECK(x.ne[d] == h.ne[d]);
        CHECK(x.nb[d] == h.nb[d]);
    }
    CHECK(x.data == h.data);
    CHECK(std::strcmp(x.name, h.name) == 0);
}

}  // namespace

int main() {
    static char wbuf[1], xbuf[1], ybuf[1];
    // q-projection of a 4096-wide model: Q4_K weights [K, N], F32 x [K, 1], F32 y [N, 1]
    HostTensor wq = tensor(GGML_TYPE_Q4_K, 4096, 4096, 1, 1, 144, 256, wbuf, "blk.0.attn_q.weight");
    HostTensor xq = tensor(GGML_TYPE_F32, 4096, 1, 1, 1, 4, 1, xbuf, "attn_norm-0");
    HostTensor yq = tensor(GGML_TYPE_F32, 4096, 1, 1, 1, 4, 1, ybuf, "Qcur-0");
    yq.op = kHostMulMat;
    yq.src[0] = &wq;
    yq.src[1] = &xq;
    // a 4-D MUL_MAT (ne2 = ne3 = 2, Q4_0) and nodes of other ops
    HostTensor w4 = tensor(GGML_TYPE_Q4_0, 256, 64, 2, 2, 18, 32, wbuf, "w4");
    HostTensor x4 = tensor(GGML_TYPE_F32, 256, 1, 2, 2, 4, 1, xbuf, "x4");
    HostTensor y4 = tensor(GGML_TYPE_F32, 64, 1, 2, 2, 4, 1, ybuf, "y4");
    y4.op = kHostMulMat;
    y4.src[0] = &w4;
    y4.src[1] = &x4;
    HostTensor norm = tensor(GGML_TYPE_F32, 4096, 1, 1, 1, 4, 1, xbuf, "norm");
    norm.op = kHostNorm;
    norm.src[0] = &xq;
    HostTensor add = tensor(GGML_TYPE_F32, 4096, 1, 1, 1, 4, 1, ybuf, "add");
    add.op = kHostAdd;
    add.src[0] = &yq;
    add.src[1] = &xq;
    // a node numbered 18 by the host (its own op 18 is not MUL_MAT): left alone
    HostTensor other = yq;
    other.op = static_cast<int>(b200_convert::kCompatMulMat);
    HostTensor* graph[] = {&norm, &yq, &add, nullptr, &y4, &other};
    const int n = sizeof graph / sizeof graph[0];

    b200_convert::NodeBatch<ggml_tensor_xdna> batch;
    const size_t m = batch.convert<HostTensor>(n, [&](int i) { return graph[i]; }, kHostMulMat);
    CHECK(m == 2 && batch.size() == 2);
    ggml_tensor_xdna** nodes = batch.nodes();
    CHECK(nodes[0]->op == GGML_OP_MUL_MAT && nodes[1]->op == GGML_OP_MUL_MAT);
    same_tensor(*nodes[0], yq);
    same_tensor(*nodes[0]->src[0], wq);
    same_tensor(*nodes[0]->src[1], xq);
    same_tensor(*nodes[1], y4);
    same_tensor(*nodes[1]->src[0], w4);
    same_tensor(*nodes[1]->src[1], x4);
    CHECK(nodes[0]->src[2] == nullptr && nodes[0]->src[0]->op == GGML_OP_NONE);
    // the library's claim predicate on the converted records (reference supports_op_impl)
    CHECK(ggml_backend_xdna_supports_op(nullptr, nodes[0]));
    CHECK(ggml_backend_xdna_supports_op(nullptr, nodes[1]));

    // a second conversion replaces the first (records stay valid until then)
    HostTensor* g2[] = {&y4};
    CHECK(batch.convert<HostTensor>(1, [&](int i) { return g2[i]; }, kHostMulMat) == 1);
    same_tensor(*batch.nodes()[0], y4);

    // claim of one op: a prefill batch (M = 8) is claimed only as rows of
    // weights resident in the plugin's buffers
    HostTensor xp = tensor(GGML_TYPE_F32, 4096, 8, 1, 1, 4, 1, xbuf, "x-prefill");
    HostTensor yp = tensor(GGML_TYPE_F32, 4096, 8, 1, 1, 4, 1, ybuf, "y-prefill");
    yp.op = kHostMulMat;
    yp.src[0] = &wq;
    yp.src[1] = &xp;
    ggml_tensor_xdna x, srcs[2];
    CHECK(b200_convert::convert_op(yp, kHostMulMat, x, srcs, false));
    CHECK(srcs[1].ne[1] == 8 && !ggml_backend_xdna_supports_op(nullptr, &x));
    CHECK(b200_convert::convert_op(yp, kHostMulMat, x, srcs, true));
    CHECK(srcs[1].ne[1] == 1 && ggml_backend_xdna_supports_op(nullptr, &x));
    CHECK(!b200_convert::convert_op(norm, kHostMulMat, x, srcs));
    // a long name is cut and terminated
    HostTensor lw = wq;
    std::memset(lw.name, 'a', sizeof lw.name);
    lw.name[63] = 'b';
    ggml_tensor_xdna lx;
    b200_convert::copy_tensor(lw, lx);
    CHECK(std::strlen(lx.name) == 63);

    if (fails) return 1;
    std::printf("ggml_convert_check: ok\n");
    return 0;
}
