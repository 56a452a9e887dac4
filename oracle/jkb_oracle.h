/*
 * jkb_oracle.h -- CPU restatement of the jero-kernels-rvv scalar fallback for the quantized
 * matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA product path and
 * the timed CPU baseline. Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg
 * and the `--impl reference` arm) load it. Nothing in the product library links or calls it.
 *
 * Every function cites the reference file:line (paths inside the jero-kernels-rvv crate) whose
 * arithmetic it restates. Floating-point code is compiled with -ffp-contract=off so that every
 * multiply and add rounds separately, exactly as the Rust scalar fallback does.
 *
 * Layout notes (not arithmetic): the reference `RepackedWeight` / `QuantizedActQ8` store i8
 * values in 8x16 tiles; this oracle keeps the same values row-major ([rows][k_padded] i8 plus
 * [rows][groups] f32 scales), which is also the layout the GPU path uses.
 */
#ifndef JKB_ORACLE_H
#define JKB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* quant_q8.rs:37-44 */
typedef struct {
    float d;
    int8_t qs[32];
} or_block_q8_0;

/* quant_q8.rs:62-71 */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} or_block_q8_k;

enum {
    OR_Q4_0 = 2,
    OR_Q4_1 = 3,
    OR_Q5_0 = 6,
    OR_Q5_1 = 7,
    OR_Q2_K = 10,
    OR_Q3_K = 11,
    OR_Q8_0 = 8,
    OR_Q4_K = 12,
    OR_Q5_K = 13,
    OR_Q6_K = 14,
    OR_IQ4_NL = 20,
    OR_TQ1_0 = 34,
    OR_TQ2_0 = 35,
    OR_I2_S = 36
};

/* ---- f16 decode (lib.rs:676-717) ---- */
float or_f16_to_f32_ieee(uint16_t bits);
float or_f16_to_f32_finite(uint16_t bits);
uint16_t or_f32_to_f16(float x);

/* ---- activation quantizers ---- */
int or_quantize_row_q8_0(const float *x, size_t n, or_block_q8_0 *out, size_t out_len);
int or_quantize_row_q8_k(const float *x, size_t n, or_block_q8_k *out, size_t out_len);
int or_quantize_rows_q8_0(const float *x, size_t m, size_t k, or_block_q8_0 *out);
int or_quantize_rows_q8_k(const float *x, size_t m, size_t k, or_block_q8_k *out);
void or_quantize_block32(const float *src, int8_t *dst, float *scale, float *sum);
int or_act_q8_quantize(const float *act, size_t m, size_t k, int8_t *q, float *x_scales,
                       float *x_sums, float *x_sums_16, float *super_scales);
int or_subln_quantize_absmax_i8(int8_t *out, const float *in, const float *norm_w, size_t len,
                                float eps, float *scale_out);
int or_relu_squared_gate_f32(float *out, const float *gate, const float *up, size_t len);

/* ---- block dots (value as the reference returns it; integer sums through out-params) ---- */
float or_dot_q4_0_q8_0_block(const uint8_t *w, const or_block_q8_0 *x, int32_t *sumi);
float or_dot_q8_0_q8_0_block(const uint8_t *w, const or_block_q8_0 *x, int32_t *sumi);
float or_dot_q4_k_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi,
                             int32_t *summins);
float or_dot_q6_k_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi);
float or_dot_q5_0_q8_0_block(const uint8_t *w, const or_block_q8_0 *x, int32_t *sumi);
float or_dot_q5_k_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi,
                             int32_t *summins);
float or_dot_tq2_0_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi);
float or_dot_tq1_0_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi);

/* Per-(row, block) integer sums and f32 block values of a whole GEMV (diagnostic view of the
 * same block functions). `quant` selects the weight format; `x` points at BlockQ8_0 (Q4_0,
 * Q8_0) or BlockQ8K (K-quants, ternary) activations. summins may be NULL except for Q4_K. */
int or_block_dots(int quant, const uint8_t *w, size_t rows, size_t cols, const void *x,
                  int32_t *sumi, int32_t *summins, float *contrib);

/* ---- M=1 GEMV drivers (run_4row_chunked_gemv semantics, quant_q8.rs:1510-1560) ---- */
int or_gemv(int quant, float *out, const uint8_t *w, size_t rows, size_t cols, const void *x);
int or_gemv_rows_mt(int quant, float *out, const uint8_t *w, size_t rows, size_t cols,
                    const void *x, size_t row_begin, size_t row_end, int nthreads);
float or_vec_dot(int quant, const uint8_t *w_row, const void *x, size_t n_blocks);

/* ---- f32-activation VectorKernel host fallback (dequant + f32 dot) ---- */
void or_dequantize_block(int quant, const uint8_t *blk, float i2s_scale, float *out);
float or_dot_product_f32(const float *a, const float *b, size_t n);
int or_dequantize_rows(int quant, const uint8_t *w, size_t rows, size_t cols, float *out);
int or_vec_dot_f32(int quant, float *out, const uint8_t *w, size_t w_len, size_t rows,
                   size_t cols, const float *input);

/* ---- BitLinear (ime.rs:882-938) ---- */
int or_bitlinear_i8(float *out, int quant, const uint8_t *w, size_t w_len, size_t rows,
                    size_t cols, const int8_t *act, float act_scale);
int or_bitlinear_i8_rows_mt(float *out, int quant, const uint8_t *w, size_t w_len, size_t rows,
                            size_t cols, const int8_t *act, float act_scale, size_t m,
                            const float *act_scales, int nthreads);

/* ---- Repacked block-scaled weights and the scalar GEMM branch (repack.rs) ---- */
size_t or_repack_scale_groups(int quant, size_t cols);
int or_repack_has_mins(int quant);
int or_repack_block_scaled(int quant, const uint8_t *raw, size_t raw_len, size_t rows,
                           size_t cols, int8_t *q, float *scales, float *mins);
int or_gemm_repacked(float *out, int quant, const int8_t *wq, const float *ws, const float *wm,
                     size_t rows, size_t cols, const int8_t *xq, const float *xs,
                     const float *xsum, const float *xsum16, size_t m, size_t row_begin,
                     size_t row_end, int nthreads);

/* ---- Compact 4-bit nibble matrices (PackedNibbleMatrix, repack.rs:4188-5545) ----
 * Q4_0, Q4_1, IQ4_NL, Q4_K_M. The tile layout is the reference's: tiles [n_tiles][k_blocks32]
 * of 128 bytes (8 rows x 32 nibbles), scales_f16 / mins_f16 [n_tiles][k_blocks32][8] f16 bits,
 * headers [n_tiles][cols / 256][8] x 16 bytes (Q4_K_M). */
int or_nibble_supported(int quant);
int or_nibble_pack_tiles(int quant, const uint8_t *raw, size_t raw_len, size_t rows, size_t cols,
                         uint8_t *tiles, uint16_t *scales_f16, uint16_t *mins_f16,
                         uint8_t *headers);
int or_nibble_decode_tiles(int quant, size_t rows, size_t cols, const uint8_t *tiles,
                           const uint16_t *scales_f16, const uint16_t *mins_f16,
                           const uint8_t *headers, int8_t *q, float *ws, float *wm);
int or_nibble_dequantize_row(int quant, const int8_t *q, const float *ws, const float *wm,
                             size_t cols, size_t row, float *out);
int or_gemm_nibble(float *out, int quant, const int8_t *q, const float *ws, const float *wm,
                   size_t rows, size_t cols, const int8_t *xq, const float *xs,
                   const float *xsum, size_t m, size_t row_begin, size_t row_end, int nthreads);

/* ---- seeded synthetic inputs and this project's own weight quantizers ---- */
uint64_t or_splitmix64(uint64_t *state);
void or_fill_normal(float *out, size_t n, uint64_t seed, float sigma);
void or_fill_ternary(int8_t *out, size_t n, uint64_t seed);
int or_quantize_weights(int quant, const float *w, size_t rows, size_t cols, uint8_t *out);
int or_pack_ternary(int quant, const int8_t *t, size_t rows, size_t cols, float scale,
                    uint8_t *out);
size_t or_weight_bytes(int quant, size_t rows, size_t cols);

#ifdef __cplusplus
}
#endif
#endif
