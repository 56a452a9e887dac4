/*
 * jkb200.h -- C ABI of the B200 (sm_100a) quantized-matmul hot path of jero-kernels-rvv.
 *
 * Every entry point below replaces one public Rust function of the jero-kernels-rvv crate
 * (path:line inside that crate is cited beside it) and keeps its argument meaning, validation
 * order and error kinds. The differences are the ones a GPU boundary forces:
 *   - slices become (pointer, element count) pairs; activation, output and scratch pointers are
 *     device pointers unless a comment says otherwise;
 *   - `&TensorView` weights become a `jkb_weight*` handle, created once at load time (validate,
 *     upload, relayout), the analogue of RepackedWeight::from_tensor (repack.rs:2288);
 *   - `Result<_, K3Error>` becomes an int status (jkb_status) plus a thread-local error record
 *     with the K3Error::TensorBoundsError fields (tensor_name, offset, byte_len, buffer_len,
 *     reason);
 *   - every call takes a CUDA stream (`void*` holding a cudaStream_t, NULL = legacy default
 *     stream) and is asynchronous on it; nothing is launched when validation fails, and no call
 *     allocates device memory (all buffers live in handles created at load time).
 *
 * All structs are plain C, little-endian, with the same layout as the reference #[repr(C)]
 * block structs.
 */
#ifndef JKB200_H
#define JKB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define JKB_ABI_VERSION 1

/* ---- status codes: K3Error variants plus device-side failures ---- */
typedef enum {
    JKB_OK = 0,
    JKB_E_BOUNDS = 1,     /* K3Error::TensorBoundsError */
    JKB_E_CAPABILITY = 2, /* K3Error::CapabilityMismatch (unsupported_tensor_quant) */
    JKB_E_CUDA = 3,       /* CUDA runtime / launch failure */
    JKB_E_NCCL = 4,       /* collective failure (sharded calls) */
    JKB_E_TIMEOUT = 5,    /* a bounded wait expired (sharded calls) */
    JKB_E_INVALID = 6     /* null pointer or destroyed handle */
} jkb_status;

/* QuantType codes (GGML type ids; I2_S is BitNet.cpp's 36). Q4_K_M is the crate's name for
 * GGML Q4_K (lib.rs:129-132). */
typedef enum {
    JKB_F32 = 0,
    JKB_F16 = 1,
    JKB_Q4_0 = 2,
    JKB_Q4_1 = 3, /* RepackedWeight and compact nibble matrices */
    JKB_Q5_0 = 6,
    JKB_Q5_1 = 7, /* RepackedWeight only */
    JKB_Q8_0 = 8,
    JKB_Q2_K = 10, /* RepackedWeight only */
    JKB_Q3_K = 11, /* RepackedWeight only */
    JKB_Q4_K_M = 12,
    JKB_Q5_K = 13,
    JKB_Q6_K = 14,
    JKB_IQ4_NL = 20, /* RepackedWeight and compact nibble matrices */
    JKB_BF16 = 30,
    JKB_TQ1_0 = 34,
    JKB_TQ2_0 = 35,
    JKB_I2_S = 36
} jkb_quant;

/* BlockQ8_0 (quant_q8.rs:37-44): 36 bytes. */
typedef struct {
    float d;
    int8_t qs[32];
} jkb_block_q8_0;

/* BlockQ8K (quant_q8.rs:62-71): 292 bytes. */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} jkb_block_q8_k;

/* jero_core::TensorView: name, quant, shape ([rows, cols], GGUF [cols, rows] or 1-D), offset
 * of the tensor in its file (reported in errors only), and the raw GGUF block bytes. `data`
 * may be host or device memory (data_on_device). */
typedef struct {
    const char *name;
    int32_t quant;
    uint32_t ndim;
    size_t shape[4];
    size_t offset;
    const void *data;
    size_t byte_len;
    int32_t data_on_device;
} jkb_tensor_view;

/* K3Error::TensorBoundsError fields of the last failure on this thread. */
typedef struct {
    int32_t status;
    char tensor_name[64];
    size_t offset;
    size_t byte_len;
    size_t buffer_len;
    char reason[256];
} jkb_error_info;

typedef struct jkb_weight jkb_weight;                   /* GEMV / BitLinear weight */
typedef struct jkb_repacked_weight jkb_repacked_weight; /* RepackedWeight (GEMM)    */
typedef struct jkb_act_q8 jkb_act_q8;                   /* QuantizedActQ8           */

/* ---- library / errors ---- */
int jkb_abi_version(void);
const char *jkb_last_error(void);
int jkb_last_error_info(jkb_error_info *out);
void jkb_clear_error(void);
/* No reference counterpart: the device error word of the kernels with bounded waits (bit 0: a
 * wait in the tensor-core GEMM expired, so that call's output is not valid; bit 1: a peer-group
 * wait expired). Synchronizes `stream`, copies the word to *flags, clears it, and returns
 * JKB_E_TIMEOUT when it was non-zero, JKB_OK otherwise. */
int jkb_device_status(int32_t *flags, void *stream);
/* No reference counterpart: the f32 epilogue of the tensor-core repacked GEMM (scale groups
 * of 32 or 16 elements, batches of at least 16 tokens; Q2_K from 32). 0 (the default): acc = fma((f32)c, xs * ws, acc)
 * per group, within one rounding per group of the reference and far inside its 1e-5 relative
 * tolerance; the integer group sums c are exact either way. 1: the reference's separately
 * rounded product and sum (accumulate_scaled_tile_scalar, repack.rs:3045-3093), bit-identical
 * outputs at about two thirds of the speed. Process-wide; takes effect at the next launch. */
int jkb_gemm_set_exact(int exact);
int jkb_gemm_get_exact(void);

/* ---- activation quantizers ---- */
/* quant_q8.rs:395 quantize_row_q8_0 (alias of quantize_row_q8_0_f32, :370). */
int jkb_quantize_row_q8_0(const float *x, size_t x_len, jkb_block_q8_0 *out, size_t out_len,
                          void *stream);
/* quant_q8.rs:370 quantize_row_q8_0_f32 */
int jkb_quantize_row_q8_0_f32(const float *x, size_t x_len, jkb_block_q8_0 *out, size_t out_len,
                              void *stream);
/* quant_q8.rs:576 quantize_row_q8_k */
int jkb_quantize_row_q8_k(const float *x, size_t x_len, jkb_block_q8_k *out, size_t out_len,
                          void *stream);
/* M rows of quantize_row_q8_0 / _q8_k in one launch (x is [m][k], out is [m][k/32] or
 * [m][k/256]); each row is exactly one reference call. */
int jkb_quantize_rows_q8_0(const float *x, size_t m, size_t k, jkb_block_q8_0 *out,
                           size_t out_len, void *stream);
int jkb_quantize_rows_q8_k(const float *x, size_t m, size_t k, jkb_block_q8_k *out,
                           size_t out_len, void *stream);
/* lib.rs:1042 subln_quantize_absmax_i8; the returned scale is written to *scale_out (device). */
int jkb_subln_quantize_absmax_i8(int8_t *out_i8, size_t out_len, const float *input,
                                 size_t in_len, const float *norm_weight, size_t w_len, float eps,
                                 float *scale_out, void *stream);
/* M independent rows of subln_quantize_absmax_i8 (input [m][len], out [m][len], scales [m]). */
int jkb_subln_quantize_absmax_i8_rows(int8_t *out_i8, const float *input,
                                      const float *norm_weight, size_t m, size_t len, float eps,
                                      float *scales_out, void *stream);
/* lib.rs:1111 relu_squared_gate_f32: out[i] = max(0, gate[i])^2 * up[i] (device buffers). */
int jkb_relu_squared_gate_f32(float *out, size_t out_len, const float *gate, size_t gate_len,
                              const float *up, size_t up_len, void *stream);
/* relu_squared_gate_f32 followed by subln_quantize_absmax_i8 on the result, m rows of len in
 * one kernel (gate, up [m][len]; out_i8 [m][len]; scales_out [m]). relu_out ([m][len], may be
 * NULL) receives the gated activation. Each row equals the two reference calls in sequence. */
int jkb_relu_squared_subln_quantize_i8_rows(int8_t *out_i8, float *relu_out, const float *gate,
                                            const float *up, const float *norm_weight, size_t m,
                                            size_t len, float eps, float *scales_out,
                                            void *stream);

/* ---- QuantizedActQ8 (repack.rs:461-724) ---- */
/* Allocates device buffers for up to m_capacity rows of k elements (load time). */
int jkb_act_q8_create(size_t m_capacity, size_t k, jkb_act_q8 **out);
int jkb_act_q8_destroy(jkb_act_q8 *act);
/* repack.rs:522 QuantizedActQ8::quantize / :542 quantize_into: act is [m][k] f32 (device). */
int jkb_act_q8_quantize(jkb_act_q8 *act, const float *input, size_t in_len, size_t m, size_t k,
                        void *stream);
/* Device views of the quantized batch (row-major): q [m][k_pad] i8, x_scales and x_sums
 * [m][k_pad/32], x_sums_16 [m][k_pad/16], super_scales [m][ceil(k/256)]. Any out-pointer may
 * be NULL. */
int jkb_act_q8_buffers(const jkb_act_q8 *act, size_t *m, size_t *k, size_t *k_padded,
                       int8_t **q, float **x_scales, float **x_sums, float **x_sums_16,
                       float **super_scales);

/* repack.rs:441 quantize_row_f32_to_q8_32 (scalar :376-400): per 32 elements of the device
 * f32 input (the tail zero-padded, non-finite values read as 0) the i8 quants, the absmax / 127
 * scale and the sequential f32 sum (quantize_block32_scalar, repack.rs:175-204). Device outputs
 * of at least round_up(in_len, 32) quants and in_len / 32 rounded up scales and sums. */
int jkb_quantize_row_f32_to_q8_32(const float *input, size_t in_len, int8_t *out_quants,
                                  size_t q_len, float *out_scales, size_t scales_len,
                                  float *out_sums, size_t sums_len, void *stream);

/* ---- scratch arenas (jero_core ScratchWorkspace / ScratchScope) and QuantizedActQ8View ----
 * A jkb_scratch is a bump arena over one device region: created with its own device memory
 * (jkb_scratch_create, at set-up) or over caller-owned device memory (jkb_scratch_wrap, which
 * allocates nothing on the device). Every carve starts at a JKB_SCRATCH_ALIGNMENT boundary;
 * reset rewinds to 0; a scope is a saved cursor (jkb_scratch_scope_begin) that
 * jkb_scratch_scope_end rewinds to, as dropping a ScratchScope does. The _in_scratch and
 * _in_scope calls below carve from the arena's cursor (the two names exist for drop-in parity;
 * they behave the same) and leave it untouched when they fail. Carved memory is overwritten by
 * later carves after a reset or scope end, so results must be consumed (in stream order) before
 * then. Not thread-safe: one arena per caller thread. */
#define JKB_SCRATCH_ALIGNMENT 128
typedef struct jkb_scratch jkb_scratch;
int jkb_scratch_create(size_t bytes, jkb_scratch **out);
int jkb_scratch_wrap(void *device_base, size_t bytes, jkb_scratch **out);
int jkb_scratch_destroy(jkb_scratch *ws);
int jkb_scratch_reset(jkb_scratch *ws);
int jkb_scratch_used_bytes(const jkb_scratch *ws, size_t *used);
int jkb_scratch_remaining_bytes(const jkb_scratch *ws, size_t *remaining);
int jkb_scratch_alloc(jkb_scratch *ws, size_t bytes, void **out);
int jkb_scratch_scope_begin(const jkb_scratch *ws, size_t *mark);
int jkb_scratch_scope_end(jkb_scratch *ws, size_t mark);
/* quant_q8.rs:405 quantize_row_q8_0_in_scratch / :429 _in_scope: x_len / 32 BlockQ8_0 carved
 * from the arena and filled from device x; *out is their device address. */
int jkb_quantize_row_q8_0_in_scratch(const float *x, size_t x_len, jkb_scratch *ws,
                                     jkb_block_q8_0 **out, void *stream);
int jkb_quantize_row_q8_0_in_scope(const float *x, size_t x_len, jkb_scratch *ws,
                                   jkb_block_q8_0 **out, void *stream);
/* quant_q8.rs:602 quantize_row_q8_k_in_scratch / :626 _in_scope (x_len / 256 BlockQ8K) */
int jkb_quantize_row_q8_k_in_scratch(const float *x, size_t x_len, jkb_scratch *ws,
                                     jkb_block_q8_k **out, void *stream);
int jkb_quantize_row_q8_k_in_scope(const float *x, size_t x_len, jkb_scratch *ws,
                                   jkb_block_q8_k **out, void *stream);

/* QuantizedActQ8View (repack.rs:806-1090): a borrowed view of quantized activations in device
 * memory the library does not own (an arena's planes, or a jkb_act_q8's). Rows are row-major:
 * q [m][k_padded] i8, x_scales and x_sums [m][k_padded / 32], x_sums_16 [m][k_padded / 16],
 * super_scales [m][ceil(k / 256)]. (The reference's view also carries sanitized f32 rows for
 * dense F32 / F16 / BF16 weights, which the GPU path does not build.) */
typedef struct {
    size_t m, k, k_padded;
    int8_t *q;
    float *x_scales;
    float *x_sums;
    float *x_sums_16;
    float *super_scales;
} jkb_act_q8_view;
/* repack.rs:827 QuantizedActQ8View::scratch_bytes_for_row: arena bytes one row of k needs,
 * alignment padding included (0 for k == 0). */
size_t jkb_act_q8_view_scratch_bytes_for_row(size_t k);
/* repack.rs:870 quantize_row_in_scratch / :969 quantize_row_in_scope: quantizes one device f32
 * row of k elements into planes carved from the arena (the QuantizedActQ8 quantizer, bit-exact)
 * and fills *out (m = 1). */
int jkb_act_q8_view_quantize_row_in_scratch(const float *act, size_t k, jkb_scratch *ws,
                                            jkb_act_q8_view *out, void *stream);
int jkb_act_q8_view_quantize_row_in_scope(const float *act, size_t k, jkb_scratch *ws,
                                          jkb_act_q8_view *out, void *stream);
/* repack.rs:708 QuantizedActQ8::as_view: the handle's current batch as a view. */
int jkb_act_q8_as_view(const jkb_act_q8 *act, jkb_act_q8_view *out);

/* ---- weights (GEMV / BitLinear layout) ---- */
/* Validates the view like the reference validators, uploads and relayouts into the GPU layout
 * for an explicit [rows, cols] interpretation (RepackedWeight::from_tensor, repack.rs:2288). */
int jkb_weight_upload(const jkb_tensor_view *view, size_t rows, size_t cols, void *stream,
                      jkb_weight **out);
/* Infers (rows, cols) from a 2-D shape the way RepackedWeight::repack does (repack.rs:2255). */
int jkb_weight_upload_infer(const jkb_tensor_view *view, void *stream, jkb_weight **out);
int jkb_weight_destroy(jkb_weight *w);
int jkb_weight_info(const jkb_weight *w, size_t *rows, size_t *cols, int32_t *quant,
                    size_t *device_bytes, size_t *gguf_bytes);
/* ---- direct-integer single-row block dots (raw GGUF row bytes on the device) ---- */
/* quant_q8.rs:1463 vec_dot_q4_0_q8_0 -> *result (device f32) */
int jkb_vec_dot_q4_0_q8_0(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_0 *x,
                          size_t x_len, float *result, void *stream);
/* quant_q8.rs:1493 vec_dot_q8_0_q8_0 */
int jkb_vec_dot_q8_0_q8_0(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_0 *x,
                          size_t x_len, float *result, void *stream);
/* quant_q8.rs:3019 vec_dot_q4_k_q8_k */
int jkb_vec_dot_q4_k_q8_k(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_k *x,
                          size_t x_len, float *result, void *stream);
/* quant_q8.rs:3056 vec_dot_q6_k_q8_k */
int jkb_vec_dot_q6_k_q8_k(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_k *x,
                          size_t x_len, float *result, void *stream);
/* quant_q8.rs:1478 vec_dot_q5_0_q8_0_blocks / :3041 vec_dot_q5_k_q8_k */
int jkb_vec_dot_q5_0_q8_0_blocks(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_0 *x,
                                 size_t x_len, float *result, void *stream);
int jkb_vec_dot_q5_k_q8_k(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_k *x,
                          size_t x_len, float *result, void *stream);
/* quant_q8.rs:3071 vec_dot_tq1_0_q8_k */
int jkb_vec_dot_tq1_0_q8_k(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_k *x,
                           size_t x_len, float *result, void *stream);
/* quant_q8.rs:3086 vec_dot_tq2_0_q8_k */
int jkb_vec_dot_tq2_0_q8_k(const uint8_t *w_blocks, size_t w_len, const jkb_block_q8_k *x,
                           size_t x_len, float *result, void *stream);

/* ---- M = 1 decode GEMV over pre-quantized activations (output fully overwritten) ---- */
/* quant_q8.rs:1586 gemv_q4_0_q8_0 (and :1612 gemv_q4_0_q8_0_4x) */
int jkb_gemv_q4_0_q8_0(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_0 *x,
                       size_t x_len, void *stream);
int jkb_gemv_q4_0_q8_0_4x(float *out, size_t out_len, const jkb_weight *w,
                          const jkb_block_q8_0 *x, size_t x_len, void *stream);
/* quant_q8.rs:1670 gemv_q8_0_q8_0 (and :1696 gemv_q8_0_q8_0_4x) */
int jkb_gemv_q8_0_q8_0(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_0 *x,
                       size_t x_len, void *stream);
int jkb_gemv_q8_0_q8_0_4x(float *out, size_t out_len, const jkb_weight *w,
                          const jkb_block_q8_0 *x, size_t x_len, void *stream);
/* quant_q8.rs:3101 gemv_q4_k_q8_k */
int jkb_gemv_q4_k_q8_k(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_k *x,
                       size_t x_len, void *stream);
/* quant_q8.rs:3189 gemv_q6_k_q8_k */
int jkb_gemv_q6_k_q8_k(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_k *x,
                       size_t x_len, void *stream);
/* quant_q8.rs:1628 gemv_q5_0_q8_0 (and :1657 the _4x alias), :3160 gemv_q5_k_q8_k */
int jkb_gemv_q5_0_q8_0(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_0 *x,
                       size_t x_len, void *stream);
int jkb_gemv_q5_0_q8_0_4x(float *out, size_t out_len, const jkb_weight *w,
                          const jkb_block_q8_0 *x, size_t x_len, void *stream);
int jkb_gemv_q5_k_q8_k(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_k *x,
                       size_t x_len, void *stream);
/* quant_q8.rs:3221 gemv_tq1_0_q8_k */
int jkb_gemv_tq1_0_q8_k(float *out, size_t out_len, const jkb_weight *w,
                        const jkb_block_q8_k *x, size_t x_len, void *stream);
/* quant_q8.rs:3250 gemv_tq2_0_q8_k */
int jkb_gemv_tq2_0_q8_k(float *out, size_t out_len, const jkb_weight *w,
                        const jkb_block_q8_k *x, size_t x_len, void *stream);
/* Row-sliced form of the gemv_* calls above (the analogue of gemv_repacked_rows,
 * repack.rs:4014): writes out[0 .. row_end - row_begin] for weight rows [row_begin, row_end).
 * x points at BlockQ8_0 (Q4_0, Q5_0, Q8_0 weights) or BlockQ8K (Q4_K_M, Q5_K, Q6_K, TQ1_0,
 * TQ2_0). */
int jkb_gemv_rows(float *out, size_t out_len, const jkb_weight *w, const void *x, size_t x_len,
                  size_t row_begin, size_t row_end, void *stream);
/* M tokens of the gemv_* calls above in one launch (no reference counterpart; the reference
 * calls gemv once per token): x is m rows of BlockQ8_0 (Q4_0, Q8_0 weights) or BlockQ8K (Q4_K_M,
 * Q6_K, TQ1_0, TQ2_0) blocks, m * blocks_per_row in all; out is [m][rows]. Each token's output
 * is exactly its single call's. */
int jkb_gemv_batch(float *out, size_t out_len, const jkb_weight *w, const void *x, size_t x_len,
                   size_t m, void *stream);
/* Diagnostic with no reference counterpart: the per-(row, block) integer sums (sumi and, for
 * Q4_K_M, summins) and the f32 block values the GEMV kernels form before summing a row.
 * Arrays are [rows][blocks_per_row]; summins may be NULL. */
int jkb_gemv_block_dots(const jkb_weight *w, const void *x, size_t x_len, int32_t *sumi,
                        int32_t *summins, float *block_values, void *stream);

/* ---- f32-activation VectorKernel entries (dequantize -> f32 dot, lib.rs:135-199) ---- */
/* lib.rs:157 VectorKernel::vec_dot_q4_k_m (host path vec_dot_q4_k_m_scalar lib.rs:1268) */
int jkb_vec_dot_q4_k_m(float *out, size_t out_len, const jkb_weight *w, const float *input,
                       size_t in_len, void *stream);
/* quant.rs:1069 vec_dot_q8_0 (scalar :899) */
int jkb_vec_dot_q8_0(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream);
/* quant.rs:1089 vec_dot_q6_k (scalar :1012) */
int jkb_vec_dot_q6_k(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream);
/* quant.rs:1458 vec_dot_q4_0 (scalar :1401) */
int jkb_vec_dot_q4_0(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream);
/* quant.rs:2036 vec_dot_q5_0 (host branch: vec_dot_generic_block, :1995-2029) and :1238
 * vec_dot_q5_k / lib.rs:188 VectorKernel::vec_dot_q5_k (host branch: vec_dot_q5_k_scalar,
 * quant.rs:1181-1222): per block the dequantized values' sequential f32 dot, rows summed in
 * block order -- bit-exact. */
int jkb_vec_dot_q5_0(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream);
int jkb_vec_dot_q5_k(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream);
/* quant.rs:2199 vec_dot_i2_s */
int jkb_vec_dot_i2_s(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream);

/* ---- f32-activation integer paths (quantize the input to Q8, then the Q8 GEMV) ---- */
/* The riscv64 entries below validate like the scalar vec_dot_* above, quantize the f32 input
 * to BlockQ8K (Q4_K_M, Q6_K) or BlockQ8_0 (Q8_0, Q4_0) with the bit-exact quantizer and run the
 * integer GEMV (vec_dot_q8_k_chunked_rvv quant_q8.rs:3280, vec_dot_q8_0_chunked_rvv
 * quant_q8.rs:1712). Results equal jkb_quantize_row_q8_k / _q8_0 followed by jkb_gemv_*; the
 * quantization runs inside the GEMV launch (each CTA quantizes the input while staging it). */
/* lib.rs:1313 vec_dot_q4_k_m_rvv */
int jkb_vec_dot_q4_k_m_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                           size_t in_len, void *stream);
/* quant.rs:1056 vec_dot_q6_k_rvv */
int jkb_vec_dot_q6_k_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream);
/* quant.rs:999 vec_dot_q8_0_rvv */
int jkb_vec_dot_q8_0_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream);
/* quant.rs:1445 vec_dot_q4_0_rvv */
int jkb_vec_dot_q4_0_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream);
/* the riscv64 branches of vec_dot_q5_0 (vec_dot_q5_0_4row_rvv) and vec_dot_q5_k
 * (quant.rs:1225 vec_dot_q5_k_rvv): input quantized, then the integer GEMV */
int jkb_vec_dot_q5_0_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream);
int jkb_vec_dot_q5_k_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream);

/* One product of jkb_vec_dot_grouped_rvv: out[0 .. out_len) = w x input. */
typedef struct {
    float *out;
    size_t out_len;
    const jkb_weight *w;
} jkb_vec_dot_item;
/* No reference counterpart: n_items (1..8) vec_dot_*_rvv calls that share one f32 input (the
 * q/k/v or gate/up projections of a decoder layer) in one launch. Every weight must have the
 * quant type of items[0] (Q4_0, Q8_0, Q4_K_M or Q6_K) and in_len columns; each item is
 * validated exactly as its single call and its output equals that call's. Outputs must not
 * overlap. */
int jkb_vec_dot_grouped_rvv(const jkb_vec_dot_item *items, size_t n_items, const float *input,
                            size_t in_len, void *stream);

/* ---- ternary BitLinear (ime.rs) ---- */
/* ime.rs:882 bitlinear_i8_rvv / :1005 bitlinear_i8_ime (bit-identical pair): TQ1_0, TQ2_0,
 * Q8_0 or I2_S weights, i8 activation (device) and its per-tensor scale. */
int jkb_bitlinear_i8(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                     size_t act_len, float act_scale, void *stream);
int jkb_bitlinear_i8_rvv(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                         size_t act_len, float act_scale, void *stream);
int jkb_bitlinear_i8_ime(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                         size_t act_len, float act_scale, void *stream);
/* M tokens of bitlinear_i8 in one launch: act [m][cols] i8, act_scales [m] f32 (device),
 * out [m][rows]; each token is exactly one reference call. */
int jkb_bitlinear_i8_batch(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                           size_t act_len, const float *act_scales, size_t m, void *stream);

/* ---- BitNet b1.58 feed-forward chain ---- */
/* No single reference function: the chain the reference composes in
 * tests/empirical_challenge_m3_bitnet.rs:582-686 for m tokens --
 *   act1, s1 = subln_quantize_absmax_i8(x, norm1, eps)           (lib.rs:1042)
 *   gate = bitlinear_i8(w_gate, act1, s1), up = bitlinear_i8(w_up, act1, s1)   (ime.rs:882)
 *   h = relu_squared_gate_f32(gate, up)                            (lib.rs:1111)
 *   act2, s2 = subln_quantize_absmax_i8(h, norm2, eps)
 *   out = bitlinear_i8(w_down, act2, s2)
 * w_gate / w_up are [intermediate, hidden], w_down [hidden, intermediate] (TQ1_0, TQ2_0, Q8_0 or
 * I2_S, each validated as its bitlinear_i8 call). r_gate / r_up / r_down are NULL or
 * RepackedWeights of the same three tensors: then batches of at least 32 tokens run the
 * projections as jkb_bitlinear_i8_gemm (tensor cores), the others as jkb_bitlinear_i8 /
 * _batch. The handle borrows the weights and the device norm weights (norm1 [hidden], norm2
 * [intermediate]) and owns the intermediates for up to m_capacity tokens, allocated here;
 * forward allocates nothing. x and out are [m][hidden] on the device; the kernels run on
 * `stream`. */
typedef struct jkb_bitnet_ffn jkb_bitnet_ffn;
int jkb_bitnet_ffn_create(const jkb_weight *w_gate, const jkb_weight *w_up,
                          const jkb_weight *w_down, const jkb_repacked_weight *r_gate,
                          const jkb_repacked_weight *r_up, const jkb_repacked_weight *r_down,
                          const float *norm1, size_t norm1_len, const float *norm2,
                          size_t norm2_len, float eps, size_t m_capacity, jkb_bitnet_ffn **out);
int jkb_bitnet_ffn_forward(jkb_bitnet_ffn *ffn, float *out, size_t out_len, const float *x,
                           size_t x_len, size_t m, void *stream);
/* Device views of the last forward's intermediates ([m_capacity] rows each; NULL to skip):
 * act1 i8 [hidden], scale1, gate / up / relu f32 [intermediate], act2 i8 [intermediate],
 * scale2. */
int jkb_bitnet_ffn_buffers(const jkb_bitnet_ffn *ffn, int8_t **act1, float **scale1,
                           float **gate, float **up, float **relu, int8_t **act2,
                           float **scale2);
int jkb_bitnet_ffn_destroy(jkb_bitnet_ffn *ffn);

/* ---- RepackedWeight + GEMM (repack.rs) ---- */
/* repack.rs:2288 RepackedWeight::from_tensor (explicit [rows, cols]) */
int jkb_repacked_weight_from_tensor(const jkb_tensor_view *view, size_t rows, size_t cols,
                                    void *stream, jkb_repacked_weight **out);
/* repack.rs:2255 RepackedWeight::repack (orientation inferred) */
int jkb_repacked_weight_repack(const jkb_tensor_view *view, void *stream,
                               jkb_repacked_weight **out);
int jkb_repacked_weight_destroy(jkb_repacked_weight *w);
/* repack.rs:2529 RepackedWeight::dequantize_row: out[0 .. cols) = scale * q - min per group
 * (device output). */
int jkb_repacked_weight_dequantize_row(const jkb_repacked_weight *w, size_t row, float *out,
                                       size_t out_len, void *stream);
/* ---- parallel load path (repack.rs:1286-1449, :1579-1722, :2366-2440) ----
 * A loader splits a weight's 8-row tiles over worker threads: each fills its tile range of host
 * buffers in the reference's tile layout with jkb_repack_into_tile_range (or
 * jkb_repack_q4_k_m_parallel_slices), then one jkb_repacked_weight_from_tile_buffers call
 * uploads the assembled buffers. The tile layout is the reference's: tiles [n_tiles][k_chunks]
 * of 128 bytes (8 weight rows x 16 K values, row j of a tile at bytes 16j .. 16j + 16), scales
 * and mins [n_tiles][scale_groups][8] f32; rows past `rows` in the last tile are zero. */
typedef struct {
    int32_t quant;
    int32_t has_mins;          /* Q4_K_M, Q5_K, Q4_1, Q5_1, Q2_K */
    size_t rows, cols;
    size_t row_bytes;          /* GGUF bytes per weight row */
    size_t k_padded;           /* cols rounded up to 32 */
    size_t n_tiles;            /* ceil(rows / 8) */
    size_t k_chunks;           /* k_padded / 16 */
    size_t chunks_per_scale;   /* 1 for 16-element scale groups (Q6_K, Q3_K, Q2_K), else 2 */
    size_t scale_groups;       /* k_chunks / chunks_per_scale */
    size_t total_tiles;        /* n_tiles * k_chunks (128-byte tiles) */
    size_t total_scales;       /* n_tiles * scale_groups * 8 */
    size_t total_mins;         /* total_scales when has_mins, else 0 */
} jkb_block_scaled_tile_layout;
/* repack.rs:2372 RepackedWeight::block_scaled_layout (BlockScaledTileLayout::for_tensor,
 * :1308): validates the view like from_tensor and fills *out. Host-only; needs no GPU. */
int jkb_block_scaled_layout(const jkb_tensor_view *view, size_t rows, size_t cols,
                            jkb_block_scaled_tile_layout *out);
/* repack.rs:1579 repack_into_tile_range: tiles [tile_begin, tile_end) into caller buffers of
 * exactly n_out_tiles = tiles * k_chunks 128-byte tiles and n_scales = tiles * scale_groups * 8
 * floats (n_mins the same, for formats with mins; ignored otherwise). The view's bytes must be
 * host memory. Host-only, allocates nothing; disjoint tile ranges may run on parallel threads. */
int jkb_repack_into_tile_range(const jkb_tensor_view *view, size_t rows, size_t cols,
                               size_t tile_begin, size_t tile_end, uint8_t *out_tiles,
                               size_t n_out_tiles, float *out_scales, size_t n_scales,
                               float *out_mins, size_t n_mins);
/* repack.rs:1659 repack_q4_k_m_parallel_slices: the same for Q4_K_M weights (CapabilityMismatch
 * otherwise) with the tiles as raw bytes (tiles_len = tiles * k_chunks * 128) and mandatory
 * mins. */
int jkb_repack_q4_k_m_parallel_slices(const jkb_tensor_view *view, size_t rows, size_t cols,
                                      size_t tile_begin, size_t tile_end, int8_t *out_tiles_i8,
                                      size_t tiles_len, float *out_scales, size_t n_scales,
                                      float *out_mins, size_t n_mins);
/* repack.rs:2386 RepackedWeight::from_tile_buffers: host buffers of the whole layout (n_tiles
 * == total_tiles 128-byte tiles, n_scales == total_scales, mins of total_mins for formats with
 * mins and NULL otherwise) -> a jkb_repacked_weight (device buffers allocated here, the tiles
 * converted to the device layout on `stream`; returns after the upload finished). The layout
 * must be one jkb_block_scaled_layout filled. */
int jkb_repacked_weight_from_tile_buffers(const jkb_block_scaled_tile_layout *layout,
                                          const uint8_t *tiles, size_t n_tiles,
                                          const float *scales, size_t n_scales,
                                          const float *mins, size_t n_mins, void *stream,
                                          jkb_repacked_weight **out);
/* Device views: q [rows][k_pad] i8, scales and mins [rows][scale_groups] f32 (mins NULL
 * unless Q4_K_M). */
int jkb_repacked_weight_buffers(const jkb_repacked_weight *w, size_t *rows, size_t *cols,
                                int32_t *quant, size_t *scale_groups, int8_t **q,
                                float **scales, float **mins);
/* repack.rs:4073 gemm_repacked: out [act.m][rows] */
int jkb_gemm_repacked(float *out, size_t out_len, const jkb_repacked_weight *w,
                      const jkb_act_q8 *act, void *stream);
/* repack.rs:4087 gemm_repacked_rows: out [act.m][row_end - row_begin] */
int jkb_gemm_repacked_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                           const jkb_act_q8 *act, size_t row_begin, size_t row_end,
                           void *stream);
/* repack.rs:3999 gemv_repacked (act.m must be 1) */
int jkb_gemv_repacked(float *out, size_t out_len, const jkb_repacked_weight *w,
                      const jkb_act_q8 *act, void *stream);
/* repack.rs:4014 gemv_repacked_rows */
int jkb_gemv_repacked_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                           const jkb_act_q8 *act, size_t row_begin, size_t row_end,
                           void *stream);
/* repack.rs:4030 gemv_repacked_view / :4045 gemv_repacked_view_rows (and RepackedWeight::
 * gemv_view / gemv_view_rows, :2628 / :2638): the single-token GEMV over a view (act->m must be
 * 1); out [row_end - row_begin]. */
int jkb_gemv_repacked_view(float *out, size_t out_len, const jkb_repacked_weight *w,
                           const jkb_act_q8_view *act, void *stream);
int jkb_gemv_repacked_view_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                                const jkb_act_q8_view *act, size_t row_begin, size_t row_end,
                                void *stream);
/* repack.rs:4101 gemv_repacked_f32 / :4114 gemv_repacked_f32_rows: device f32 input [cols]
 * quantized into the caller's act handle (capacity >= 1 row, k == cols; the reference allocates
 * a QuantizedActQ8 here), then the GEMV of rows [row_begin, row_end). */
int jkb_gemv_repacked_f32(float *out, size_t out_len, const jkb_repacked_weight *w,
                          const float *input, size_t in_len, jkb_act_q8 *scratch, void *stream);
int jkb_gemv_repacked_f32_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                               const float *input, size_t in_len, size_t row_begin,
                               size_t row_end, jkb_act_q8 *scratch, void *stream);
/* repack.rs:4143 gemm_repacked_f32_rows: as jkb_gemm_repacked_f32 for weight rows
 * [row_begin, row_end); out [m][row_end - row_begin]. */
int jkb_gemm_repacked_f32_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                               const float *input, size_t in_len, size_t m, size_t row_begin,
                               size_t row_end, jkb_act_q8 *scratch, void *stream);
/* repack.rs:4129 gemm_repacked_f32: quantizes input [m][cols] into the caller's act handle
 * (the reference allocates a QuantizedActQ8 here; this ABI never allocates), then GEMMs. */
int jkb_gemm_repacked_f32(float *out, size_t out_len, const jkb_repacked_weight *w,
                          const float *input, size_t in_len, size_t m, jkb_act_q8 *scratch,
                          void *stream);
/* bitlinear_i8 (ime.rs:882-938) for m tokens on the tensor cores: a RepackedWeight of TQ1_0,
 * TQ2_0, I2_S or Q8_0 (repacked from the same bytes as the jkb_weight of jkb_bitlinear_i8),
 * act [m][cols] i8 and act_scales [m] f32 (device), out [m][rows]. scratch (capacity >= m, k
 * == cols) receives the activations in the GEMM's layout. From 32 tokens each BitLinear block
 * (256 elements for TQ1_0 / TQ2_0, 128 for I2_S, 32 for Q8_0) is one tensor-core accumulator
 * and its value (f32)c * (d * s) is added in K order: with jkb_gemm_set_exact(1) every output
 * equals the reference's row sum bit for bit, by default within its 1e-5 relative tolerance
 * (one rounding fewer per block). Smaller batches run the repacked GEMM's 32-element groups
 * (within the tolerance). */
int jkb_bitlinear_i8_gemm(float *out, size_t out_len, const jkb_repacked_weight *w,
                          const int8_t *act_i8, size_t act_len, const float *act_scales,
                          size_t m, jkb_act_q8 *scratch, void *stream);
/* No counterpart in the reference. The same computation as jkb_gemm_repacked_f32 for callers
 * that cannot allocate device memory, and so cannot create the jkb_act_q8 scratch handle. Two
 * examples: an engine that reserved all remaining HBM for its KV cache at start-up, and a host
 * whose per-token loop forbids cudaMalloc because it may synchronize the device and stall the
 * pipeline. The quantized activations go to a scratch array built into the library (4.25 MiB
 * of device memory on every GPU that uses it, held until exit). The batch must satisfy
 * m * round_up(cols, 32) <= 2097152 elements (e.g. 512 tokens x 4096); larger batches fail
 * with JKB_E_BOUNDS. Once set up on a device, a call allocates nothing.
 * Set-up: the first call on each device looks up the scratch address (cudaGetSymbolAddress)
 * with that device current. Under CUDA's default lazy module loading that first call is also
 * when the driver loads this part of the library on the device and reserves the 4.25 MiB, so
 * it can fail with out-of-memory if the caller has already claimed all free HBM. Make one call
 * per device at start-up, before reserving HBM and before any stream capture.
 * All calls share the one array, so calls whose executions overlap on the GPU (different
 * streams, or threads sharing a device) race; serialize them. Each call writes every scratch
 * value it reads, so results never depend on an earlier call. Weights with 16-element min
 * groups (Q2_K) run this entry point on the CUDA-core dp4a GEMM (about 7 TOPS against 134 on
 * the tensor cores through jkb_gemm_repacked_f32), because the scratch has no plane for their
 * 16-element activation sums. The address is cached per device ordinal: after cudaDeviceReset
 * every device pointer this library holds for that device, this one included, is invalid. */
int jkb_gemm_repacked_f32_noalloc(float *out, size_t out_len, const jkb_repacked_weight *w,
                                  const float *input, size_t in_len, size_t m, void *stream);

/* ---- PackedNibbleMatrix: compact 4-bit weights and their GEMM (repack.rs:4188-5545) ----
 * Q4_0, Q4_1, IQ4_NL and Q4_K_M weights stay 4-bit on the device: the handle holds each row's
 * GGUF quant bytes and block scales (exactly the GGUF payload size), and the GEMM expands the
 * codes to int8 in shared memory. Results are those of execute_nibble_gemm_rows
 * (repack.rs:5181-5397): per output, 32-element blocks in K order, acc += (f32)c * (xs * ws)
 * [- x_sum * wm]. Batches of at least 32 tokens with cols a multiple of 128 run on the tensor
 * cores (default: fused multiply-add per block, within 1e-5 relative; jkb_gemm_set_exact(1):
 * bit-identical); smaller batches and other shapes run a bit-identical row kernel. */
typedef struct jkb_nibble_matrix jkb_nibble_matrix;
/* repack.rs:4788 PackedNibbleMatrix::from_tensor (explicit [rows, cols]) */
int jkb_packed_nibble_matrix_from_tensor(const jkb_tensor_view *view, size_t rows, size_t cols,
                                         void *stream, jkb_nibble_matrix **out);
/* repack.rs:4654 PackedNibbleMatrix::repack (orientation inferred) */
int jkb_packed_nibble_matrix_repack(const jkb_tensor_view *view, void *stream,
                                    jkb_nibble_matrix **out);
/* repack.rs:4686 PackedNibbleMatrix::from_scale_f16_buffers (Q4_0 / IQ4_NL) and :4743
 * from_q4_k_buffers: host buffers in the reference's tile layout -- nibble_tiles
 * [n_tiles][cols / 32] x 128 bytes (n_tiles = ceil(rows / 8)), scales_f16 [n_tiles][cols / 32][8],
 * headers [n_tiles][cols / 256][8] x 16 bytes; counts are in tiles, scales and headers. */
int jkb_packed_nibble_matrix_from_scale_f16_buffers(int32_t quant, size_t rows, size_t cols,
                                                    const uint8_t *nibble_tiles, size_t n_tiles,
                                                    const uint16_t *scales_f16, size_t n_scales,
                                                    void *stream, jkb_nibble_matrix **out);
int jkb_packed_nibble_matrix_from_q4_k_buffers(size_t rows, size_t cols,
                                               const uint8_t *nibble_tiles, size_t n_tiles,
                                               const uint8_t *headers, size_t n_headers,
                                               void *stream, jkb_nibble_matrix **out);
/* repack.rs:4414 repack_nibble_into_tile_range, on the host: tiles tile_begin..tile_end of the
 * reference's layout (the input of the two constructors above). Output lengths are counts:
 * n_out_tiles = tiles * (cols / 32), n_scales = n_mins = tiles * (cols / 32) * 8 (Q4_0 and
 * IQ4_NL scales; Q4_1 scales and mins), n_headers = tiles * (cols / 256) * 8 (Q4_K_M). Unused
 * outputs may be NULL with count 0. The view's bytes must be host memory. */
int jkb_repack_nibble_into_tile_range(const jkb_tensor_view *view, size_t rows, size_t cols,
                                      size_t tile_begin, size_t tile_end, uint8_t *out_tiles,
                                      size_t n_out_tiles, uint16_t *out_scales_f16,
                                      size_t n_scales, uint16_t *out_mins_f16, size_t n_mins,
                                      uint8_t *out_headers, size_t n_headers);
int jkb_packed_nibble_matrix_destroy(jkb_nibble_matrix *w);
/* rows, cols, quant, n_tiles (rows.div_ceil(8)), k_blocks32, packed_bytes (device bytes of the
 * codes and scales; equal to raw_tensor_bytes), raw_tensor_bytes (GGUF size) */
int jkb_packed_nibble_matrix_info(const jkb_nibble_matrix *w, size_t *rows, size_t *cols,
                                  int32_t *quant, size_t *n_tiles, size_t *k_blocks32,
                                  size_t *packed_bytes, size_t *raw_tensor_bytes);
/* Device views: qs [rows][cols / 2] code bytes, meta [rows][blocks] scale words. */
int jkb_packed_nibble_matrix_buffers(const jkb_nibble_matrix *w, uint8_t **qs, uint8_t **meta);
/* repack.rs:4945 gemm: out [act.m][rows] */
int jkb_packed_nibble_matrix_gemm(float *out, size_t out_len, const jkb_nibble_matrix *w,
                                  const jkb_act_q8 *act, void *stream);
/* repack.rs:4954 gemm_rows: out [act.m][row_end - row_begin] */
int jkb_packed_nibble_matrix_gemm_rows(float *out, size_t out_len, const jkb_nibble_matrix *w,
                                       const jkb_act_q8 *act, size_t row_begin, size_t row_end,
                                       void *stream);
/* repack.rs:4968 gemv (act.m must be 1) */
int jkb_packed_nibble_matrix_gemv(float *out, size_t out_len, const jkb_nibble_matrix *w,
                                  const jkb_act_q8 *act, void *stream);
/* repack.rs:5001 dequantize_row: out [cols] f32 (device) */
int jkb_packed_nibble_matrix_dequantize_row(const jkb_nibble_matrix *w, size_t row, float *out,
                                            size_t out_len, void *stream);
/* repack.rs:5140 gemm_q4_0_ime / :5162 gemm_q4_k_ime: the GEMM, CapabilityMismatch unless the
 * matrix is Q4_0 / Q4_K_M. */
int jkb_gemm_q4_0_ime(float *out, size_t out_len, const jkb_nibble_matrix *w,
                      const jkb_act_q8 *act, void *stream);
int jkb_gemm_q4_k_ime(float *out, size_t out_len, const jkb_nibble_matrix *w,
                      const jkb_act_q8 *act, void *stream);

/* ---- multi-GPU output-row sharding: a one-kernel all-gather over NVLink (no reference
 * counterpart; the reference splits work by row ranges, gemv_repacked_rows repack.rs:4014) ----
 * One process per GPU. Every rank creates a peer group holding a device buffer of `bytes` (the
 * same on every rank: it fixes the all-gather's grid, whose CTAs each signal every peer), the
 * ranks exchange the group handles (JKB_PEER_HANDLE_BYTES each, over any host channel) and
 * open them (CUDA IPC: each rank maps every peer's buffer). Each rank computes its output-row
 * shards into its own buffer at their global offsets (the buffer holds the full output
 * vectors); jkb_peer_group_allgather then pushes this rank's chunks to the same offsets in every
 * peer's buffer with coalesced stores over NVLink, signals each peer, and makes `stream` wait
 * until every peer's push of the same call has arrived -- one kernel launch. Afterwards every
 * rank holds the full vectors. All ranks call it with their own chunks in the same order. The
 * arrival count lives on the device, so a captured CUDA graph replays correctly. Waits are
 * bounded (about 2 s): on expiry bit 1 of the device error word (jkb_device_status) is set and
 * the kernel returns; the group is then out of step and must be recreated. A chunk must not be
 * rewritten before every rank has finished reading it: callers alternate two output slots by
 * step parity (a rank cannot start step s + 2 before every rank has pushed step s + 1, which
 * comes after its reads of step s). */
#define JKB_PEER_HANDLE_BYTES 64
#define JKB_PEER_MAX_RANKS 8
#define JKB_PEER_MAX_CHUNKS 16
typedef struct jkb_peer_group jkb_peer_group;
int jkb_peer_group_create(int world, int rank, size_t bytes, jkb_peer_group **out);
int jkb_peer_group_handle(const jkb_peer_group *pg, void *handle);
/* handles: world * JKB_PEER_HANDLE_BYTES bytes, rank-ordered (this rank's own entry ignored) */
int jkb_peer_group_open(jkb_peer_group *pg, const void *handles);
int jkb_peer_group_buffer(const jkb_peer_group *pg, void **local, size_t *bytes);
/* chunks: n byte ranges [offset[i], offset[i] + len[i]) of the buffer; offsets and lengths
 * must be 4-byte aligned (the 16-byte aligned body of a chunk is copied as 16-byte words, its
 * head and tail as 4-byte words) */
int jkb_peer_group_allgather(jkb_peer_group *pg, const size_t *offset, const size_t *len,
                             size_t n, void *stream);
/* Low-level: make `stream` wait until `arrivals` more peer signals have reached this rank than
 * at its previous wait (each allgather or signal call delivers one from every peer). */
int jkb_peer_group_wait(jkb_peer_group *pg, uint64_t arrivals, void *stream);
/* Pushed outputs: the all-gather fused into the GEMVs. While push is enabled on a group (an
 * opened group; at most 8 groups at a time), every launch of the single-token, grouped and
 * token-batch GEMV entry points (jkb_gemv_q*_q8_*, jkb_gemv_tq*_q8_k, jkb_gemv_rows,
 * jkb_gemv_batch, jkb_vec_dot_<fmt>_rvv, jkb_vec_dot_grouped_rvv, jkb_bitlinear_i8, its _rvv /
 * _ime forms and jkb_bitlinear_i8_batch) whose outputs lie
 * in the group's buffer also stores each output element to the same offset in every peer's
 * buffer, from the kernel that computes it (NVLink stores), and fences those stores at system
 * scope before the kernel ends. jkb_peer_group_signal then completes the exchange: one small
 * kernel signals every peer and makes `stream` wait until every peer's signal of the same call
 * has arrived (bounded like the all-gather). All ranks call it once per step, after their
 * pushing launches; the two-slot rule of the all-gather applies. An output range that crosses
 * the edge of a pushing buffer fails with JKB_E_BOUNDS. The repacked and nibble products
 * (jkb_gemm_repacked*, jkb_gemv_repacked*, jkb_bitlinear_i8_gemm, the PackedNibbleMatrix
 * GEMMs), the scalar block dots jkb_vec_dot_<fmt>_q8_* and the f32 jkb_vec_dot_<fmt> do not
 * push and fail with JKB_E_CAPABILITY on an output in a pushing buffer; other entry points do
 * not push either (their outputs belong outside pushing buffers). With one rank both calls are
 * no-ops. */
int jkb_peer_group_set_push(jkb_peer_group *pg, int enable);
int jkb_peer_group_signal(jkb_peer_group *pg, void *stream);
int jkb_peer_group_destroy(jkb_peer_group *pg);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* JKB200_H */
