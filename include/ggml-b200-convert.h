/*
 * ggml-b200-convert.h -- ggml tensors -> the compat ABI's ggml_tensor_xdna.
 *
 * Header-only C++ helpers used by the ggml adapter (xdna.cpp_b200/ggml/
 * ggml-b200-adapter.cpp) to hand a ggml graph to
 * ggml_backend_xdna_compute_graph.  They are templates over both tensor
 * types, so this header includes nothing from ggml: the adapter instantiates
 * them with ggml's `struct ggml_tensor`, the CPU tests with a stand-in that
 * has the same field names.  The compat struct's fields are the ones the
 * reference's process_mul_mat_node reads (src/ggml-xdna.cpp:149-308): type,
 * ne, nb, op, src[0..1], data and name.
 *
 * Op ids differ: ggml numbers GGML_OP_MUL_MAT by its own (changing)
 * enumeration, the compat ABI by the reference's standalone one (18,
 * include/xdna/ggml-xdna.h:50-92).  The caller passes ggml's value.
 */
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

namespace b200_convert {

// The compat ABI's id of MUL_MAT (reference include/xdna/ggml-xdna.h:50-92).
constexpr uint32_t kCompatMulMat = 18;

// Shape, strides, type, data and name of a tensor (op left NONE, no sources).
template <class XT, class GT>
void copy_tensor(const GT& g, XT& x) {
    std::memset(static_cast<void*>(&x), 0, sizeof x);
    x.type = static_cast<decltype(x.type)>(static_cast<int>(g.type));
    for (int d = 0; d < 4; ++d) {
        x.ne[d] = static_cast<int64_t>(g.ne[d]);
        x.nb[d] = static_cast<size_t>(g.nb[d]);
    }
    x.data = g.data;
    std::strncpy(x.name, g.name, sizeof x.name - 1);
    x.name[sizeof x.name - 1] = '\0';
}

// A graph's MUL_MAT nodes as compat tensors: three records per node (the
// node and its two sources), kept alive until the next convert().
template <class XT>
class NodeBatch {
   public:
    template <class GT, class NodeAt>
    size_t convert(int n_nodes, NodeAt node_at, int ggml_mul_mat) {
        recs_.clear();
        ptrs_.clear();
        recs_.reserve(3 * static_cast<size_t>(n_nodes > 0 ? n_nodes : 0));
        for (int i = 0; i < n_nodes; ++i) {
            const GT* g = node_at(i);
            if (!g || static_cast<int>(g->op) != ggml_mul_mat || !g->src[0] || !g->src[1]) continue;
            recs_.emplace_back();
            copy_tensor(*g->src[0], recs_.back());
            recs_.emplace_back();
            copy_tensor(*g->src[1], recs_.back());
            recs_.emplace_back();
            XT& x = recs_.back();
            copy_tensor(*g, x);
            x.op = kCompatMulMat;
            x.src[0] = &recs_[recs_.size() - 3];
            x.src[1] = &recs_[recs_.size() - 2];
        }
        for (size_t k = 2; k < recs_.size(); k += 3) ptrs_.push_back(&recs_[k]);
        return ptrs_.size();
    }
    XT** nodes() { return ptrs_.data(); }
    size_t size() const { return ptrs_.size(); }

   private:
    std::vector<XT> recs_;
    std::vector<XT*> ptrs_;
};

// One tensor (a MUL_MAT node, for the claim predicate) as a compat record
// with its sources in `srcs`; rows_one = true gives the activation one row,
// for weights resident in this backend's buffers, which the reference claims
// for any row count (src/ggml-xdna.cpp:81-93, 109-111).
template <class XT, class GT>
bool convert_op(const GT& g, int ggml_mul_mat, XT& x, XT (&srcs)[2], bool rows_one = false) {
    if (static_cast<int>(g.op) != ggml_mul_mat || !g.src[0] || !g.src[1]) return false;
    copy_tensor(*g.src[0], srcs[0]);
    copy_tensor(*g.src[1], srcs[1]);
    if (rows_one) srcs[1].ne[1] = 1;
    copy_tensor(g, x);
    x.op = kCompatMulMat;
    x.src[0] = &srcs[0];
    x.src[1] = &srcs[1];
    return true;
}

}  // namespace b200_convert
