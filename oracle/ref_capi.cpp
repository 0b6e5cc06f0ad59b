// extern "C" wrapper around the reference's own CPU code for the decode-GEMV
// path, compiled from the reference sources in place by oracle/Makefile into
// oracle/_ref/libxdna_ref.so.  TEST INFRASTRUCTURE ONLY: it pins the C
// restatement in quant_oracle.c and is the timed CPU baseline in bench.py.
//
// Wrapped entry points:
//   xdna::q4_0::{dequantize_row, gemv_f32, gemv_bf16}  src/xdna-q4-0-reference.cpp:200-300
//   xdna::dequantize_row_*_ref, xdna::gemv_*_ref       include/xdna/kquants.h:290-577
//   xdna::XdnaGemvEngine::{run, run_bf16, run_quant}    src/xdna-gemv-engine.cpp:1817-2009
//   xdna::XdnaGemvEngine::evaluate                      src/xdna-gemv-engine.cpp:2053-2095
//   xdna::TilePartition                                 include/xdna/xdna_gemv_engine.h:18-82
//   xdna::Q4Prepacker                                   src/xdna-q4-prepack.cpp:39-114
#include "xdna/kquants.h"
#include "xdna/q4_0_reference.h"
#include "xdna/q4_prepack.h"
#include "xdna/xdna_gemv_engine.h"

#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>

namespace {

thread_local std::string g_last_error;

bool to_quant_type(int ggml_type, xdna::QuantType* out) {
    switch (ggml_type) {
        case 2:  *out = xdna::QuantType::Q4_0; return true;
        case 11: *out = xdna::QuantType::Q3_K; return true;
        case 12: *out = xdna::QuantType::Q4_K; return true;
        case 13: *out = xdna::QuantType::Q5_K; return true;
        case 14: *out = xdna::QuantType::Q6_K; return true;
        case 18: *out = xdna::QuantType::IQ3_XXS; return true;
        case 21: *out = xdna::QuantType::IQ3_S; return true;
        case 22: *out = xdna::QuantType::IQ2_S; return true;
        case 23: *out = xdna::QuantType::IQ4_XS; return true;
        default: return false;
    }
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_last_error = e.what();
        return -1;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return -2;
    } catch (...) {
        g_last_error = "unknown exception";
        return -3;
    }
}

}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_last_error.c_str(); }

int ref_q4_0_dequantize_row(const uint8_t* row, size_t nbytes, size_t K, float* out) {
    return guarded([&] { xdna::q4_0::dequantize_row(row, nbytes, K, out); });
}

int ref_q4_0_gemv_f32(const uint8_t* w, size_t nbytes, size_t N, size_t K, const float* x, float* y) {
    return guarded([&] { xdna::q4_0::gemv_f32(w, nbytes, N, K, x, K, y, N); });
}

int ref_q4_0_gemv_bf16(const uint8_t* w, size_t nbytes, size_t N, size_t K, const uint16_t* x, float* y) {
    static_assert(sizeof(xdna::q4_0::Bf16) == sizeof(uint16_t), "bf16 layout");
    return guarded([&] {
        xdna::q4_0::gemv_bf16(w, nbytes, N, K, reinterpret_cast<const xdna::q4_0::Bf16*>(x), K, y, N);
    });
}

float ref_fp16_to_f32(uint16_t h) { return xdna::q4_0::fp16_to_float(h); }

int ref_kquant_dequantize_row(int type, const uint8_t* row, int64_t K, float* out) {
    return guarded([&] {
        switch (type) {
            case 12: xdna::dequantize_row_q4_K_ref(reinterpret_cast<const xdna::block_q4_K*>(row), out, K); break;
            case 13: xdna::dequantize_row_q5_K_ref(reinterpret_cast<const xdna::block_q5_K*>(row), out, K); break;
            case 11: xdna::dequantize_row_q3_K_ref(reinterpret_cast<const xdna::block_q3_K*>(row), out, K); break;
            case 14: xdna::dequantize_row_q6_K_ref(reinterpret_cast<const xdna::block_q6_K*>(row), out, K); break;
            case 23: xdna::dequantize_row_iq4_xs_ref(reinterpret_cast<const xdna::block_iq4_xs*>(row), out, K); break;
            case 21: xdna::dequantize_row_iq3_s_ref(reinterpret_cast<const xdna::block_iq3_s*>(row), out, K); break;
            default: throw std::invalid_argument("no in-repo reference dequantizer for this type");
        }
    });
}

int ref_kquant_gemv(int type, const uint8_t* w, size_t N, size_t K, const float* x, float* y) {
    return guarded([&] {
        switch (type) {
            case 12: xdna::gemv_q4_K_ref(w, N, K, x, y); break;
            case 13: xdna::gemv_q5_K_ref(w, N, K, x, y); break;
            case 11: xdna::gemv_q3_K_ref(w, N, K, x, y); break;
            case 14: xdna::gemv_q6_K_ref(w, N, K, x, y); break;
            case 23: xdna::gemv_iq4_xs_ref(w, N, K, x, y); break;
            case 21: xdna::gemv_iq3_s_ref(w, N, K, x, y); break;
            default: throw std::invalid_argument("no in-repo reference GEMV for this type");
        }
    });
}

void ref_iq3s_grid(uint32_t* out512) { std::memcpy(out512, xdna::iq3s_grid, sizeof(xdna::iq3s_grid)); }
void ref_kvalues_iq4nl(int8_t* out16) { std::memcpy(out16, xdna::kvalues_iq4nl, sizeof(xdna::kvalues_iq4nl)); }

size_t ref_bytes_per_row(int type, size_t K) {
    xdna::QuantType qt;
    if (!to_quant_type(type, &qt)) return 0;
    return xdna::bytes_per_row_for_quant(qt, K);
}

// ---- the reference's CPU GEMV engine (the timed baseline) -----------------
void* ref_engine_create(size_t crossover_n) {
    try {
        return new xdna::XdnaGemvEngine(0, 4, crossover_n);
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return nullptr;
    }
}

void ref_engine_destroy(void* h) { delete static_cast<xdna::XdnaGemvEngine*>(h); }

int ref_engine_hardware_ready(void* h) {
    return static_cast<xdna::XdnaGemvEngine*>(h)->is_hardware_ready() ? 1 : 0;
}

int ref_engine_run(void* h, int type, const uint8_t* w, size_t nbytes, size_t N, size_t K,
                   const float* x, float* y) {
    xdna::QuantType qt;
    if (!to_quant_type(type, &qt)) {
        g_last_error = "unsupported type";
        return -1;
    }
    auto* e = static_cast<xdna::XdnaGemvEngine*>(h);
    return guarded([&] { e->run_quant(qt, w, nbytes, N, K, x, y); });
}

int ref_engine_run_bf16(void* h, int type, const uint8_t* w, size_t nbytes, size_t N, size_t K,
                        const uint16_t* x, float* y) {
    xdna::QuantType qt;
    if (!to_quant_type(type, &qt)) {
        g_last_error = "unsupported type";
        return -1;
    }
    auto* e = static_cast<xdna::XdnaGemvEngine*>(h);
    return guarded([&] {
        e->run_quant_bf16(qt, w, nbytes, N, K, reinterpret_cast<const xdna::q4_0::Bf16*>(x), y);
    });
}

// XdnaGemvEngine::evaluate: out[0]=cos, out[1]=maxabs, out[2]=GB/s, out[3]=passed
void ref_evaluate(const float* actual, const float* reference, size_t count, size_t weight_bytes,
                  double duration_us, double* out4) {
    auto m = xdna::XdnaGemvEngine::evaluate(actual, reference, count, weight_bytes, duration_us, false);
    out4[0] = m.cosine_similarity;
    out4[1] = m.max_abs_error;
    out4[2] = m.effective_bandwidth_gb_s;
    out4[3] = m.passed ? 1.0 : 0.0;
}

// TilePartition::create(N, K, cols).tile_row_range for all tiles -> ranges[2*16]
int ref_tile_partition(size_t N, size_t K, size_t cols, size_t* rows_per_col, size_t* rows_per_tile,
                       size_t* ranges, size_t max_tiles) {
    return guarded([&] {
        auto p = xdna::TilePartition::create(N, K, cols);
        *rows_per_col = p.rows_per_col;
        *rows_per_tile = p.rows_per_tile;
        size_t t = 0;
        for (size_t c = 0; c < p.num_columns; ++c)
            for (size_t i = 0; i < p.tiles_per_col && t < max_tiles; ++i, ++t) {
                auto r = p.tile_row_range(c, i);
                ranges[2 * t] = r.first;
                ranges[2 * t + 1] = r.second;
            }
    });
}

int ref_q4_prepack_dequantize(const uint8_t* q4_0, size_t M, size_t K, size_t cols, float* out) {
    return guarded([&] {
        auto layout = xdna::Q4Prepacker::compute_layout(M, K, cols);
        std::string packed(layout.total_packed_bytes, '\0');
        xdna::Q4Prepacker::pack(q4_0, M, K, reinterpret_cast<uint8_t*>(&packed[0]), cols);
        xdna::Q4Prepacker::dequantize_packed(reinterpret_cast<const uint8_t*>(packed.data()), M, K, out, cols);
    });
}

}  // extern "C"
