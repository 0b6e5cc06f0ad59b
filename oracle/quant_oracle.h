/*
 * CPU oracle for the decode-GEMV hot path (M = 1 GGML_OP_MUL_MAT).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the GPU kernels are
 * compared against; it is loaded by tests/, by __graft_entry__.smoke() and by
 * bench.py's CPU-baseline leg, never by the product library.
 *
 * It restates, in plain C, the reference's scalar arithmetic for the nine
 * weight formats the plugin claims:
 *   Q4_0            src/xdna-q4-0-reference.cpp:63-97 (dot order) and :101-136
 *                   (fp16 bit recipe); gemv_f32/gemv_bf16 :246-300
 *   Q4_K Q5_K Q3_K  include/xdna/kquants.h:290-423 (dequant) and :495-577 (gemv)
 *   Q6_K IQ4_XS     include/xdna/kquants.h:394-445
 *   IQ3_S           include/xdna/kquants.h:447-490
 *   IQ3_XXS IQ2_S   third party: the reference has no in-repo code for these
 *                   (src/xdna-gemv-engine.cpp:1340-1341 returns 0); the
 *                   algorithm restated is gguf 0.19.0 gguf/quants.py:901-1056.
 *
 * Type ids are ggml's (ggml.h enum ggml_type; reference include/xdna/ggml-xdna.h:19-48).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    OR_Q4_0 = 2, OR_Q3_K = 11, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14,
    OR_IQ3_XXS = 18, OR_IQ3_S = 21, OR_IQ2_S = 22, OR_IQ4_XS = 23,
};

/* 0 on success, negative on a bad argument. */
int    oracle_block_values(int type);          /* 32 or 256, 0 if unknown */
int    oracle_block_bytes(int type);           /* bytes per block, 0 if unknown */
size_t oracle_row_bytes(int type, int64_t K);  /* 0 if K is not a block multiple */

float    oracle_fp16_to_f32(uint16_t h);
uint16_t oracle_f32_to_fp16(float f);           /* round to nearest even */
float    oracle_bf16_to_f32(uint16_t b);
uint16_t oracle_f32_to_bf16(float f);           /* reference float_to_bf16 */

int oracle_dequantize_row(int type, const uint8_t *row, int64_t K, float *out);

/* y[N] = W[N,K] x[K] with the reference's exact float operation order. */
int oracle_gemv(int type, const uint8_t *W, int64_t N, int64_t K,
                const float *x, float *y, int nthreads);
/* Q4_0 with BF16 activations (reference gemv_bf16). */
int oracle_gemv_q4_0_bf16(const uint8_t *W, int64_t N, int64_t K,
                          const uint16_t *x_bf16, float *y, int nthreads);

/* Seeded synthetic-weight quantisers (row of K values -> row_bytes bytes).
 * Q4_0 follows ggml's quantize_row_q4_0_ref; the others are this build's own
 * simple quantisers written from the format definitions (ggml's are absent
 * here).  Parity does not depend on them: oracle and GPU consume the same bytes. */
int oracle_quantize_row(int type, const float *x, int64_t K, uint8_t *out);
int oracle_quantize(int type, const float *x, int64_t N, int64_t K,
                    uint8_t *out, int nthreads);

#ifdef __cplusplus
}
#endif
