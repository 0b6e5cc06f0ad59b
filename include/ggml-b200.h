/*
 * ggml-b200 -- B200 decode-GEMV backend, public C ABI.
 *
 * The library claims single-row (M = 1) GGML_OP_MUL_MAT with Q4_0, Q3_K, Q4_K,
 * Q5_K, Q6_K, IQ2_S, IQ3_S, IQ3_XXS or IQ4_XS weights and F32 activations and
 * runs it as hand-written sm_100a kernels: an integer tensor-core GEMV for
 * every format (matrices of 16-row tiles), an F32 dequantise-and-FMA kernel
 * for the other row counts.
 *
 * Section 1 is the reference's ggml-free "backwards-compatibility" C ABI with
 * the same names, argument meaning and error behaviour
 * (reference include/xdna/ggml-xdna.h:124-165, src/ggml-xdna.cpp:719-844), so
 * code written against libggml-xdna's compat ABI links unchanged.  Section 2
 * exposes the buffer-type / buffer interface of the reference's ggml plugin
 * (src/ggml-xdna.cpp:316-470) as plain C calls, because without ggml the
 * compat ABI has no way to place weights in a device buffer.  Section 3 is the
 * thin launcher layer over the CUDA kernels (device pointers, explicit stream).
 * Section 4 is the N-row sharded multi-GPU path.
 *
 * Error behaviour: bool-returning calls return false and print
 * "[b200 error] ..." to stderr, as the reference does; int-returning calls
 * return 0 on success and a negative code otherwise.  The last message is
 * also kept per thread (ggml_backend_xdna_last_error).
 */
#pragma once

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (values as in ggml.h; reference include/xdna/ggml-xdna.h:19-48). */
typedef enum {
    GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6, GGML_TYPE_Q5_1 = 7, GGML_TYPE_Q8_0 = 8, GGML_TYPE_Q8_1 = 9,
    GGML_TYPE_Q2_K = 10, GGML_TYPE_Q3_K = 11, GGML_TYPE_Q4_K = 12, GGML_TYPE_Q5_K = 13,
    GGML_TYPE_Q6_K = 14, GGML_TYPE_Q8_K = 15, GGML_TYPE_IQ2_XXS = 16, GGML_TYPE_IQ2_XS = 17,
    GGML_TYPE_IQ3_XXS = 18, GGML_TYPE_IQ1_S = 19, GGML_TYPE_IQ4_NL = 20, GGML_TYPE_IQ3_S = 21,
    GGML_TYPE_IQ2_S = 22, GGML_TYPE_IQ4_XS = 23, GGML_TYPE_I8 = 24, GGML_TYPE_I16 = 25,
    GGML_TYPE_I32 = 26, GGML_TYPE_I64 = 27, GGML_TYPE_F64 = 28, GGML_TYPE_IQ1_M = 29,
    GGML_TYPE_BF16 = 30, GGML_TYPE_COUNT
} ggml_type_xdna;

/* Op ids of the compat ABI: the reference's standalone enumeration
 * (include/xdna/ggml-xdna.h:50-92), in which GGML_OP_MUL_MAT is 18. */
typedef enum {
    GGML_OP_NONE = 0, GGML_OP_DUP, GGML_OP_ADD, GGML_OP_ADD1, GGML_OP_ACC, GGML_OP_SUB,
    GGML_OP_MUL, GGML_OP_DIV, GGML_OP_SQR, GGML_OP_SQRT, GGML_OP_LOG, GGML_OP_SIN,
    GGML_OP_COS, GGML_OP_CLAMP, GGML_OP_NORM, GGML_OP_RMS_NORM, GGML_OP_RMS_NORM_BACK,
    GGML_OP_GROUP_NORM, GGML_OP_MUL_MAT, GGML_OP_MUL_MAT_ID, GGML_OP_OUT_PROD, GGML_OP_SCALE,
    GGML_OP_SET, GGML_OP_CPY, GGML_OP_CONT, GGML_OP_RESHAPE, GGML_OP_VIEW, GGML_OP_PERMUTE,
    GGML_OP_TRANSPOSE, GGML_OP_GET_ROWS, GGML_OP_GET_ROWS_BACK, GGML_OP_DIAG,
    GGML_OP_DIAG_MASK_INF, GGML_OP_DIAG_MASK_ZERO, GGML_OP_SOFT_MAX, GGML_OP_SOFT_MAX_BACK,
    GGML_OP_ROPE, GGML_OP_ROPE_BACK, GGML_OP_ALIBI, GGML_OP_SILU, GGML_OP_COUNT
} ggml_op_xdna;

typedef void *ggml_backend_t;
typedef void *ggml_backend_buffer_t;
typedef void *ggml_backend_buffer_type_t;
typedef void *ggml_backend_reg_t;
typedef void *ggml_backend_dev_t;

enum ggml_status {
    GGML_STATUS_ALLOC_FAILED = -2,
    GGML_STATUS_FAILED = -1,
    GGML_STATUS_SUCCESS = 0,
    GGML_STATUS_ABORTED = 1,
};

/* Tensor record of the compat ABI (reference include/xdna/ggml-xdna.h:131-142).
 * For MUL_MAT: src[0] weights [K = ne[0], N = ne[1], ne2, ne3], src[1] F32
 * activations [K, M, ne2, ne3], the node itself the F32 output [N, M, ne2, ne3].
 * `data` may point to host memory or into a B200 buffer (section 2). */
struct ggml_tensor_xdna {
    ggml_type_xdna type;
    int64_t ne[4];
    size_t nb[4];
    uint32_t op;
    int32_t op_params[16];
    int32_t flags;
    struct ggml_tensor_xdna *src[10];
    void *data;
    char name[64];
    void *extra;
};

/* ======================= 1. compat C ABI (reference names) ======================= */

/* Backend on CUDA device dev_num (reference :736-748).  NULL on failure
 * (no such device, CUDA error). */
ggml_backend_t ggml_backend_xdna_init(size_t dev_num);
/* Reference :750-752. */
bool ggml_backend_is_xdna(ggml_backend_t backend);
/* Reference :754-767. */
void ggml_backend_xdna_free(ggml_backend_t backend);
/* HBM-resident weight buffer type of device dev_num (reference :769-772). */
ggml_backend_buffer_type_t ggml_backend_xdna_buffer_type(size_t dev_num);
/* Pinned host buffer type (reference :774-776). */
ggml_backend_buffer_type_t ggml_backend_xdna_host_buffer_type(void);
/* Claim predicate (reference supports_op_impl :95-147, compat entry :778-781). */
bool ggml_backend_xdna_supports_op(ggml_backend_t backend, const struct ggml_tensor_xdna *op);
/* Runs every MUL_MAT node, skips others (reference :825-844).  Synchronous:
 * outputs are complete when it returns. */
bool ggml_backend_xdna_compute_graph(ggml_backend_t backend, struct ggml_tensor_xdna **nodes, size_t n_nodes);
/* Registry handle (reference :732-734); device count = number of CUDA devices. */
ggml_backend_reg_t ggml_backend_xdna_reg(void);

/* Last error message of the calling thread ("" if none).  No reference counterpart. */
const char *ggml_backend_xdna_last_error(void);

/* ================= 2. buffer type / buffer (reference ggml iface, as C) ================= */

/* buft name, "B200" or "B200_Host" (reference buft_get_name :382-385). */
const char *ggml_backend_xdna_buft_name(ggml_backend_buffer_type_t buft);
/* Allocate a buffer (reference buft_alloc_buffer :387-405): cudaMalloc for the
 * device type, cudaHostAlloc for the host type.  NULL on failure. */
ggml_backend_buffer_t ggml_backend_xdna_buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size);
/* Alignment of tensor data offsets inside a buffer: 4096 (reference :407-410). */
size_t ggml_backend_xdna_buft_get_alignment(ggml_backend_buffer_type_t buft);
/* Bytes a tensor occupies: ggml_nbytes; both device layouts have the same span (reference :417-454). */
size_t ggml_backend_xdna_buft_get_alloc_size(ggml_backend_buffer_type_t buft, const struct ggml_tensor_xdna *tensor);
/* false for the device type, true for the host type (reference :456-459 returns true). */
bool ggml_backend_xdna_buft_is_host(ggml_backend_buffer_type_t buft);
/* Reference buf_free_buffer / buf_get_base (:316-327). */
void ggml_backend_xdna_buffer_free(ggml_backend_buffer_t buffer);
void *ggml_backend_xdna_buffer_get_base(ggml_backend_buffer_t buffer);
size_t ggml_backend_xdna_buffer_get_size(ggml_backend_buffer_t buffer);
/* Host -> tensor bytes [offset, offset + size) in GGUF layout (reference
 * buf_set_tensor :341-345).  Quantised weight tensors are uploaded through a
 * bounded pinned staging ring and repacked on the GPU into the device layout
 * (MMA tiles or stripe tiles, as b200_gemv describes). */
bool ggml_backend_xdna_buffer_set_tensor(ggml_backend_buffer_t buffer, struct ggml_tensor_xdna *tensor,
                                         const void *data, size_t offset, size_t size);
/* Tensor -> host, GGUF layout (reference buf_get_tensor :347-351). */
bool ggml_backend_xdna_buffer_get_tensor(ggml_backend_buffer_t buffer, const struct ggml_tensor_xdna *tensor,
                                         void *data, size_t offset, size_t size);
/* Reference buf_memset_tensor :335-339 and buf_clear :353-359. */
bool ggml_backend_xdna_buffer_memset_tensor(ggml_backend_buffer_t buffer, struct ggml_tensor_xdna *tensor,
                                            uint8_t value, size_t offset, size_t size);
bool ggml_backend_xdna_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value);
/* Like set_tensor, with the GGUF bytes already in device memory of the same
 * GPU (e.g. produced by a device quantiser): device-to-device, repacked in
 * place.  No reference counterpart (its buffers are host memory). */
bool ggml_backend_xdna_buffer_set_tensor_device(ggml_backend_buffer_t buffer, struct ggml_tensor_xdna *tensor,
                                                const void *dev_data, size_t offset, size_t size);
/* Copy tensor src to dst, both in B200 buffers of one GPU, same type and shape
 * (ggml buffer iface cpy_tensor; the reference leaves that slot empty, :370). */
bool ggml_backend_xdna_buffer_cpy_tensor(const struct ggml_tensor_xdna *src, struct ggml_tensor_xdna *dst);
/* The cudaStream_t the backend computes on (for event timing / interop). */
void *ggml_backend_xdna_get_stream(ggml_backend_t backend);
/* Wait for all work queued on the backend's stream (reference synchronize :692-694). */
void ggml_backend_xdna_synchronize(ggml_backend_t backend);
/* Device memory (reference dev_get_memory :505-509, which hard-codes 16 GiB). */
void ggml_backend_xdna_get_device_memory(size_t dev_num, size_t *free_bytes, size_t *total_bytes);
size_t ggml_backend_xdna_get_device_count(void);

/* ===================== 3. launcher layer (device pointers) ===================== */

/* y[N] = W[N,K] x[K] on `stream` (a cudaStream_t, NULL = legacy default).  W is
 * in the device layout b200_repack writes: 16-row MMA tiles for every format
 * when N % 16 == 0 and K % 256 == 0, stripe tiles otherwise.  x must be
 * 16-byte aligned.  pdl != 0
 * launches with programmatic dependent launch.  Replaces the reference's
 * XdnaGemvEngine::run / run_quant (src/xdna-gemv-engine.cpp:1817-1992). */
int b200_gemv(int type, const void *w_packed, const float *x, float *y, int64_t n, int64_t k,
              void *stream, int pdl);
/* y_s = W_s x for up to 4 matrices that share x (q / k / v or gate / up of a
 * transformer block) in one x preparation and one GEMV launch.  Every W_s must
 * be in the 16-row MMA layout (any of the nine formats, N_s % 16 == 0,
 * K % 256 == 0).  No
 * reference counterpart; ggml_backend_xdna_compute_graph applies the same
 * fusion to consecutive nodes that qualify. */
int b200_gemv_multi(int type, const void *const *w_packed, float *const *y, const int64_t *n, int nseg,
                    const float *x, int64_t k, void *stream, int pdl);
/* b200_gemv that allocates no device memory.  No reference counterpart (the
 * reference's CPU path needs no device scratch).  It is for callers that
 * cannot allocate device memory at call time: a host that has handed all
 * device memory to its own pools, or a decode loop that cannot take the
 * device-wide synchronisation of cudaMalloc / cudaFree in the middle of a
 * token.  The MMA path, which every format takes when N % 16 == 0 and
 * K % 256 == 0, then uses a fixed 1 MiB static device array for its scratch
 * instead of the per-stream buffers b200_gemv grows on demand; shapes needing
 * more (above N = 131072 with K = 32768) fail with an error naming the limit.
 * Matrices in the stripe layout (N % 16 != 0) need no scratch and run as in
 * b200_gemv.  The array's device address is
 * looked up (cudaGetSymbolAddress) by the first call on each device, so make
 * that first call before capturing a stream.  The array is shared by every
 * stream of the device: calls whose executions overlap in time race. */
int b200_gemv_noalloc(int type, const void *w_packed, const float *x, float *y, int64_t n, int64_t k,
                      void *stream);
/* Status of the GEMV kernels' bounded waits on the current CUDA device:
 * *status = 1 if a wait inside a shared-memory GEMV variant (XDNA_B200_GEMV =
 * ring / bulk / bulkx) ran out since the last call, else 0; the word is
 * cleared.  Returns 0, or a negative code on a CUDA error.  No reference
 * counterpart (its engine has no device waits). */
int b200_gemv_error(int *status);
/* GGUF rows -> device layout (MMA tiles or stripe tiles, as b200_gemv
 * describes; out of place), the GPU replacement of the
 * reference's Q4Prepacker::pack (src/xdna-q4-prepack.cpp:39-114). */
int b200_repack(int type, const void *raw, void *packed, int64_t n, int64_t k, void *stream);
/* Inverse of b200_repack (Q4Prepacker::dequantize_packed's role, exact). */
int b200_unpack(int type, const void *packed, void *raw, int64_t n, int64_t k, void *stream);
/* BF16 activations -> F32 on the device (reference run_bf16 conversion :1894-1908). */
int b200_bf16_to_f32(const uint16_t *src, float *dst, int64_t n, void *stream);
/* y = W x for BF16 x: exact conversion to F32 (into a per-stream device buffer
 * that grows on demand) followed by b200_gemv.  Replaces
 * XdnaGemvEngine::run_bf16 / run_quant_bf16 (src/xdna-gemv-engine.cpp:1894-1908,
 * 1994-2009). */
int b200_gemv_bf16(int type, const void *w_packed, const uint16_t *x_bf16, float *y, int64_t n, int64_t k,
                   void *stream, int pdl);
/* Synthetic N(0, sigma) F32 values and device quantisers (Q4_0, Q4_K). */
int b200_fill_normal(float *out, int64_t n, uint64_t seed, float sigma, void *stream);
int b200_quantize(int type, const float *src, void *dst, int64_t n, int64_t k, void *stream);
/* Host-side stripe repack of one whole matrix (CPU, no GPU needed). */
int b200_repack_host(int type, const void *raw, void *packed, int64_t n, int64_t k);
int b200_unpack_host(int type, const void *packed, void *raw, int64_t n, int64_t k);
/* Bytes per GGUF row, 0 if the type is not claimed or k is not a block multiple. */
size_t b200_row_bytes(int type, int64_t k);
/* Dynamic shared memory one GEMV CTA uses for row length k. */
size_t b200_gemv_smem_bytes(int type, int64_t k);

/* ============== 4. row-sharded multi-GPU execution (one process per GPU) ==============
 * No reference counterpart: the reference drives one device.  Each rank owns
 * rows [row0, row0 + N/world) of every weight (ggml_backend_xdna_shard_rows);
 * a MUL_MAT node whose src0 holds the local rows and whose dst has
 * ne[0] = N_local * world is computed locally and completed with an NCCL
 * all-gather of the F32 slices, so every rank ends with the full output.
 * Every rank must submit the same node sequence. */

/* A fresh NCCL unique id (rank 0 creates it and distributes the 128 bytes). */
int ggml_backend_xdna_nccl_unique_id(uint8_t out[128]);
/* Backend of `rank` in a group of `world` ranks on device dev_num.  NCCL
 * initialisation is bounded by XDNA_B200_NCCL_TIMEOUT_S (default 120 s);
 * NULL on failure or timeout. */
ggml_backend_t ggml_backend_xdna_init_sharded(size_t dev_num, int world, int rank, const uint8_t id[128]);
/* Rows of an N-row weight owned by `rank`; N must be divisible by world. */
int ggml_backend_xdna_shard_rows(int64_t n, int world, int rank, int64_t *row0, int64_t *nrows);

#ifdef __cplusplus
}
#endif
