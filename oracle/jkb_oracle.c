/*
 * jkb_oracle.c -- CPU restatement of the jero-kernels-rvv scalar fallback (quantized matmul hot
 * path). TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU baseline.
 * The product library never links this file.
 *
 * Built with -O3 -ffp-contract=off -fno-fast-math: every f32 multiply and add rounds on its
 * own, as in the Rust scalar fallback the functions below restate (file:line in each comment).
 * Rust's `Iterator::sum` over f32 folds from -0.0; the row drivers that use it do the same here.
 */
#include "jkb_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------ */
/* f16 decode                                                                                  */
/* ------------------------------------------------------------------------------------------ */

static inline float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* lib.rs:676-708: exact half -> float, subnormals normalised by a shift loop, NaN payload kept
 * with the quiet bit set. */
float or_f16_to_f32_ieee(uint16_t bits) {
    uint32_t sign = (bits >> 15) & 1u;
    uint32_t exp = (bits >> 10) & 0x1Fu;
    uint32_t mant = bits & 0x3FFu;
    if (exp == 0) {
        if (mant == 0) return bits_f32(sign << 31);
        uint32_t m = mant, e = 127u - 14u;
        while ((m & 0x400u) == 0) {
            m <<= 1;
            e -= 1;
        }
        m &= 0x3FFu;
        return bits_f32((sign << 31) | (e << 23) | (m << 13));
    }
    if (exp == 0x1F) {
        if (mant == 0) return bits_f32((sign << 31) | 0x7F800000u);
        return bits_f32((sign << 31) | 0x7FC00000u | (mant << 13));
    }
    return bits_f32((sign << 31) | ((exp + 112u) << 23) | (mant << 13));
}

/* lib.rs:714-717: non-finite half scales become 0.0. */
float or_f16_to_f32_finite(uint16_t bits) {
    float v = or_f16_to_f32_ieee(bits);
    return isfinite(v) ? v : 0.0f;
}

/* Round-to-nearest-even f32 -> f16 used only by this project's weight quantizers (the reference
 * ships no weight quantizer). */
uint16_t or_f32_to_f16(float x) {
    _Float16 h = (_Float16)x;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------------------------------------ */
/* Activation quantizers                                                                       */
/* ------------------------------------------------------------------------------------------ */

/* quant_q8.rs:102-108 round_scaled_to_i8: RMM rounding of finite values, clamp to +-127;
 * non-finite inputs quantize to 0. */
static inline int8_t round_scaled_to_i8(float v, float inv) {
    if (!isfinite(v)) return 0;
    float r = roundf(v * inv);
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    return (int8_t)r;
}

/* quant_q8.rs:203-219 quantize_block_q8_0_scalar */
static void quantize_block_q8_0(const float *x, or_block_q8_0 *blk) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++)
        if (isfinite(x[i])) amax = fmaxf(amax, fabsf(x[i]));
    if (amax == 0.0f || !isfinite(amax)) {
        memset(blk, 0, sizeof(*blk));
        return;
    }
    float d = amax / 127.0f;
    float inv = 127.0f / amax;
    blk->d = d;
    for (int i = 0; i < 32; i++) blk->qs[i] = round_scaled_to_i8(x[i], inv);
}

/* quant_q8.rs:447-475 quantize_block_q8_k_scalar (one scale per 256, i16 sums per 16) */
static void quantize_block_q8_k(const float *x, or_block_q8_k *blk) {
    float amax = 0.0f;
    for (int i = 0; i < 256; i++)
        if (isfinite(x[i])) amax = fmaxf(amax, fabsf(x[i]));
    if (amax == 0.0f || !isfinite(amax)) {
        memset(blk, 0, sizeof(*blk));
        return;
    }
    float d = amax / 127.0f;
    float inv = 127.0f / amax;
    blk->d = d;
    for (int sb = 0; sb < 16; sb++) {
        int16_t s = 0;
        for (int j = 0; j < 16; j++) {
            int8_t q = round_scaled_to_i8(x[sb * 16 + j], inv);
            blk->qs[sb * 16 + j] = q;
            s = (int16_t)(s + q);
        }
        blk->bsums[sb] = s;
    }
}

/* quant_q8.rs:370-388 quantize_row_q8_0_f32 + validate_activation_quant_slice (:111-149) */
int or_quantize_row_q8_0(const float *x, size_t n, or_block_q8_0 *out, size_t out_len) {
    if (n == 0 || n % 32 != 0 || out_len != n / 32) return 1;
    for (size_t b = 0; b < n / 32; b++) quantize_block_q8_0(x + 32 * b, out + b);
    return 0;
}

/* quant_q8.rs:576-594 quantize_row_q8_k */
int or_quantize_row_q8_k(const float *x, size_t n, or_block_q8_k *out, size_t out_len) {
    if (n == 0 || n % 256 != 0 || out_len != n / 256) return 1;
    for (size_t b = 0; b < n / 256; b++) quantize_block_q8_k(x + 256 * b, out + b);
    return 0;
}

/* M independent rows of quantize_row_q8_0 (the reference quantizes one token per call). */
int or_quantize_rows_q8_0(const float *x, size_t m, size_t k, or_block_q8_0 *out) {
    for (size_t r = 0; r < m; r++)
        if (or_quantize_row_q8_0(x + r * k, k, out + r * (k / 32), k / 32)) return 1;
    return 0;
}

int or_quantize_rows_q8_k(const float *x, size_t m, size_t k, or_block_q8_k *out) {
    for (size_t r = 0; r < m; r++)
        if (or_quantize_row_q8_k(x + r * k, k, out + r * (k / 256), k / 256)) return 1;
    return 0;
}

/* repack.rs:175-204 quantize_block32_scalar: sanitize non-finite to 0, sequential f32 sum from
 * 0.0, absmax < 1e-30 -> zero block with scale 0. */
void or_quantize_block32(const float *src, int8_t *dst, float *scale, float *sum) {
    float clean[32];
    float absmax = 0.0f, s = 0.0f;
    for (int i = 0; i < 32; i++) {
        float v = isfinite(src[i]) ? src[i] : 0.0f;
        clean[i] = v;
        s += v;
        float a = fabsf(v);
        if (a > absmax) absmax = a;
    }
    if (absmax < 1e-30f) {
        memset(dst, 0, 32);
        *scale = 0.0f;
        *sum = s;
        return;
    }
    float d = absmax / 127.0f;
    float inv = 127.0f / absmax;
    for (int i = 0; i < 32; i++) {
        float q = roundf(clean[i] * inv);
        if (q < -127.0f) q = -127.0f;
        if (q > 127.0f) q = 127.0f;
        dst[i] = (int8_t)q;
    }
    *scale = d;
    *sum = s;
}

/* repack.rs:542-650 QuantizedActQ8::quantize_into, stored row-major:
 *   q            [m][k_pad] i8          (tiles hold the same values)
 *   x_scales     [m][k_pad/32]
 *   x_sums       [m][k_pad/32]
 *   x_sums_16    [m][k_pad/16]          (Iterator::sum over the sanitized row, from -0.0)
 *   super_scales [m][ceil(k/256)]       (max of the 32-block scales inside each 256 span)
 * Tail elements of a ragged last block are zero-padded (repack.rs:389-399). */
int or_act_q8_quantize(const float *act, size_t m, size_t k, int8_t *q, float *x_scales,
                       float *x_sums, float *x_sums_16, float *super_scales) {
    if (m == 0 || k == 0) return 1;
    size_t kp = (k + 31) / 32 * 32, kb = kp / 32, kc = kp / 16, nsb = (k + 255) / 256;
    float *row = (float *)malloc(kp * sizeof(float));
    if (!row) return 1;
    for (size_t r = 0; r < m; r++) {
        const float *src = act + r * k;
        for (size_t i = 0; i < kp; i++) row[i] = (i < k && isfinite(src[i])) ? src[i] : 0.0f;
        if (super_scales)
            for (size_t s = 0; s < nsb; s++) super_scales[r * nsb + s] = 0.0f;
        for (size_t b = 0; b < kb; b++) {
            float buf[32];
            for (int i = 0; i < 32; i++) {
                size_t idx = b * 32 + i;
                buf[i] = idx < k ? src[idx] : 0.0f;
            }
            float sc, sm;
            or_quantize_block32(buf, q + r * kp + b * 32, &sc, &sm);
            x_scales[r * kb + b] = sc;
            if (x_sums) x_sums[r * kb + b] = sm;
            size_t sb = (b * 32) / 256;
            if (super_scales && sb < nsb && sc > super_scales[r * nsb + sb])
                super_scales[r * nsb + sb] = sc;
        }
        if (x_sums_16)
            for (size_t c = 0; c < kc; c++) {
                float s = -0.0f;
                for (int i = 0; i < 16; i++) s += row[c * 16 + i];
                x_sums_16[r * kc + c] = s;
            }
    }
    free(row);
    return 0;
}

/* lib.rs:770-777 dot_product_f32_scalar: sequential sum from 0.0. */
float or_dot_product_f32(const float *a, const float *b, size_t n) {
    float s = 0.0f;
    for (size_t i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* lib.rs:1042-1101 subln_quantize_absmax_i8: RMSNorm, per-tensor absmax, RMM round, clamp to
 * [-128, 127]; NaN or < 1e-12 max -> zeros with scale 1/127. `as i8` of NaN is 0. */
int or_subln_quantize_absmax_i8(int8_t *out, const float *in, const float *norm_w, size_t len,
                                float eps, float *scale_out) {
    if (len == 0) return 1;
    float sum_sq = or_dot_product_f32(in, in, len);
    float mean_sq = sum_sq / (float)len;
    float inv_rms = 1.0f / sqrtf(mean_sq + eps);
    float max_val = 0.0f;
    for (size_t i = 0; i < len; i++) {
        float xn = in[i] * inv_rms * norm_w[i];
        float a = fabsf(xn);
        if (a > max_val) max_val = a;
    }
    if (isnan(max_val) || max_val < 1e-12f) {
        memset(out, 0, len);
        *scale_out = 1.0f / 127.0f;
        return 0;
    }
    float scale = max_val / 127.0f;
    for (size_t i = 0; i < len; i++) {
        float xn = in[i] * inv_rms * norm_w[i];
        float q = roundf(xn / scale);
        if (isnan(q)) {
            out[i] = 0;
            continue;
        }
        if (q < -128.0f) q = -128.0f;
        if (q > 127.0f) q = 127.0f;
        out[i] = (int8_t)q;
    }
    *scale_out = scale;
    return 0;
}

/* relu_squared_gate_scalar (lib.rs:1130-1137): out[i] = (relu * relu) * up[i] with
 * relu = g > 0 ? g : 0 (NaN and -0 gates give +0). */
int or_relu_squared_gate_f32(float *out, const float *gate, const float *up, size_t len) {
    if (len == 0) return 1;
    for (size_t i = 0; i < len; i++) {
        float g = gate[i];
        float relu = g > 0.0f ? g : 0.0f;
        out[i] = relu * relu * up[i];
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Block dots (quant_q8.rs)                                                                    */
/* ------------------------------------------------------------------------------------------ */

static inline float i2f(int32_t v) { return (float)v; }

/* quant_q8.rs:672-684: low nibble -> element j, high nibble -> element j+16, value - 8. */
float or_dot_q4_0_q8_0_block(const uint8_t *w, const or_block_q8_0 *x, int32_t *sumi_out) {
    float dw = or_f16_to_f32_finite(rd16(w));
    int32_t sumi = 0;
    for (int i = 0; i < 16; i++) {
        int32_t q0 = (int32_t)(w[2 + i] & 0x0F) - 8;
        int32_t q1 = (int32_t)((w[2 + i] >> 4) & 0x0F) - 8;
        sumi += q0 * x->qs[i] + q1 * x->qs[i + 16];
    }
    if (sumi_out) *sumi_out = sumi;
    if (dw == 0.0f || x->d == 0.0f) return 0.0f;
    return i2f(sumi) * (dw * x->d);
}

/* quant_q8.rs:707-717 */
float or_dot_q8_0_q8_0_block(const uint8_t *w, const or_block_q8_0 *x, int32_t *sumi_out) {
    float dw = or_f16_to_f32_finite(rd16(w));
    int32_t sumi = 0;
    for (int i = 0; i < 32; i++) sumi += (int32_t)(int8_t)w[2 + i] * x->qs[i];
    if (sumi_out) *sumi_out = sumi;
    if (dw == 0.0f || x->d == 0.0f) return 0.0f;
    return i2f(sumi) * (dw * x->d);
}

/* quant_q8.rs:1817-1830 unpack_q4_q5_k_scales_mins (6-bit scales and mins). */
static void unpack_k4_scales(const uint8_t *s, uint8_t sc[8], uint8_t m[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 0x3F;
        m[j] = s[j + 4] & 0x3F;
    }
    for (int j = 4; j < 8; j++) {
        sc[j] = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        m[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* quant_q8.rs:1834-1862: (d*xd)*sumi - (dmin*xd)*summins, mins from the i16 bsums. */
float or_dot_q4_k_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi_out,
                             int32_t *summins_out) {
    float d = or_f16_to_f32_finite(rd16(w));
    float dmin = or_f16_to_f32_finite(rd16(w + 2));
    uint8_t sc[8], mn[8];
    unpack_k4_scales(w + 4, sc, mn);
    const uint8_t *qs = w + 16;
    int32_t sumi = 0, summins = 0;
    for (int c = 0; c < 4; c++) {
        int32_t slo = 0, shi = 0;
        for (int l = 0; l < 32; l++) {
            uint8_t b = qs[c * 32 + l];
            slo += (int32_t)(b & 0x0F) * x->qs[c * 64 + l];
            shi += (int32_t)(b >> 4) * x->qs[c * 64 + 32 + l];
        }
        sumi += (int32_t)sc[2 * c] * slo + (int32_t)sc[2 * c + 1] * shi;
        int32_t blo = (int32_t)x->bsums[4 * c] + x->bsums[4 * c + 1];
        int32_t bhi = (int32_t)x->bsums[4 * c + 2] + x->bsums[4 * c + 3];
        summins += (int32_t)mn[2 * c] * blo + (int32_t)mn[2 * c + 1] * bhi;
    }
    if (sumi_out) *sumi_out = sumi;
    if (summins_out) *summins_out = summins;
    if ((d == 0.0f && dmin == 0.0f) || x->d == 0.0f) return 0.0f;
    return (d * x->d) * i2f(sumi) - (dmin * x->d) * i2f(summins);
}

/* quant_q8.rs:688-703 (dot_q5_0_q8_0_block_scalar): f16 d, u32 qh, 16 nibble bytes; element j
 * = (low nibble of byte j | bit j of qh << 4) - 16, element j + 16 = (high nibble | bit j + 16
 * << 4) - 16. Zero when d == 0 or xd == 0; else (f32)sumi * (d * xd). */
float or_dot_q5_0_q8_0_block(const uint8_t *w, const or_block_q8_0 *x, int32_t *sumi_out) {
    float dw = or_f16_to_f32_finite(rd16(w));
    uint32_t qh = (uint32_t)w[2] | ((uint32_t)w[3] << 8) | ((uint32_t)w[4] << 16) |
                  ((uint32_t)w[5] << 24);
    int32_t sumi = 0;
    for (int j = 0; j < 16; j++) {
        int32_t q0 = (int32_t)((w[6 + j] & 0x0F) | (((qh >> j) & 1) << 4)) - 16;
        int32_t q1 = (int32_t)(((w[6 + j] >> 4) & 0x0F) | (((qh >> (j + 16)) & 1) << 4)) - 16;
        sumi += q0 * x->qs[j] + q1 * x->qs[j + 16];
    }
    if (sumi_out) *sumi_out = sumi;
    if (dw == 0.0f || x->d == 0.0f) return 0.0f;
    return i2f(sumi) * (dw * x->d);
}

/* quant_q8.rs:1866-1899 (dot_q5_k_q8_k_block_scalar): the Q4_K block with a fifth bit per
 * element from qh[32] @16 (bit 2c for the low half of chunk c, 2c + 1 for the high half); qs
 * @48. Block value (d * xd) * sumi - (dmin * xd) * summins. */
float or_dot_q5_k_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi_out,
                             int32_t *summins_out) {
    float d = or_f16_to_f32_finite(rd16(w));
    float dmin = or_f16_to_f32_finite(rd16(w + 2));
    uint8_t sc[8], mn[8];
    unpack_k4_scales(w + 4, sc, mn);
    const uint8_t *qh = w + 16, *qs = w + 48;
    int32_t sumi = 0, summins = 0;
    for (int c = 0; c < 4; c++) {
        int32_t slo = 0, shi = 0;
        for (int l = 0; l < 32; l++) {
            uint8_t b = qs[c * 32 + l];
            int32_t h1 = (qh[l] >> (2 * c)) & 1 ? 16 : 0, h2 = (qh[l] >> (2 * c + 1)) & 1 ? 16 : 0;
            slo += ((int32_t)(b & 0x0F) | h1) * x->qs[c * 64 + l];
            shi += ((int32_t)(b >> 4) | h2) * x->qs[c * 64 + 32 + l];
        }
        sumi += (int32_t)sc[2 * c] * slo + (int32_t)sc[2 * c + 1] * shi;
        int32_t blo = (int32_t)x->bsums[4 * c] + x->bsums[4 * c + 1];
        int32_t bhi = (int32_t)x->bsums[4 * c + 2] + x->bsums[4 * c + 3];
        summins += (int32_t)mn[2 * c] * blo + (int32_t)mn[2 * c + 1] * bhi;
    }
    if (sumi_out) *sumi_out = sumi;
    if (summins_out) *summins_out = summins;
    if ((d == 0.0f && dmin == 0.0f) || x->d == 0.0f) return 0.0f;
    return (d * x->d) * i2f(sumi) - (dmin * x->d) * i2f(summins);
}

/* quant_q8.rs:1903-1942: ql[128] qh[64] i8 scales[16] f16 d @208; quads of 16 with i8 scales. */
float or_dot_q6_k_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi_out) {
    float d = or_f16_to_f32_finite(rd16(w + 208));
    const uint8_t *ql = w, *qh = w + 128;
    const int8_t *scales = (const int8_t *)(w + 192);
    int32_t sumi = 0;
    for (int h = 0; h < 2; h++) {
        int n = h * 128, qlo = h * 64, qho = h * 32, sb = h * 8;
        for (int is = 0; is < 2; is++) {
            int32_t s1 = 0, s2 = 0, s3 = 0, s4 = 0;
            for (int l = is * 16; l < is * 16 + 16; l++) {
                uint8_t blo = ql[qlo + l], bhi = ql[qlo + l + 32], hb = qh[qho + l];
                int32_t q1 = (int32_t)((blo & 0x0F) | ((hb & 3) << 4)) - 32;
                int32_t q2 = (int32_t)((bhi & 0x0F) | (((hb >> 2) & 3) << 4)) - 32;
                int32_t q3 = (int32_t)((blo >> 4) | (((hb >> 4) & 3) << 4)) - 32;
                int32_t q4 = (int32_t)((bhi >> 4) | (((hb >> 6) & 3) << 4)) - 32;
                s1 += q1 * x->qs[n + l];
                s2 += q2 * x->qs[n + l + 32];
                s3 += q3 * x->qs[n + l + 64];
                s4 += q4 * x->qs[n + l + 96];
            }
            sumi += scales[sb + is] * s1 + scales[sb + is + 2] * s2 + scales[sb + is + 4] * s3 +
                    scales[sb + is + 6] * s4;
        }
    }
    if (sumi_out) *sumi_out = sumi;
    if (d == 0.0f || x->d == 0.0f) return 0.0f;
    return (d * x->d) * i2f(sumi);
}

/* ime.rs:636-658 unpack_tq2_0_block_i8: f16 d first, element 4i+j = ((qs[i] >> 2j) & 3) - 1. */
static float unpack_tq2_0(const uint8_t *blk, int8_t *out) {
    for (int i = 0; i < 64; i++) {
        uint8_t b = blk[2 + i];
        out[4 * i + 0] = (int8_t)((b & 3) - 1);
        out[4 * i + 1] = (int8_t)(((b >> 2) & 3) - 1);
        out[4 * i + 2] = (int8_t)(((b >> 4) & 3) - 1);
        out[4 * i + 3] = (int8_t)(((b >> 6) & 3) - 1);
    }
    return or_f16_to_f32_finite(rd16(blk));
}

/* ime.rs:595-624 unpack_tq1_0_block_i8: 51 bytes of five base-3 digits (b % 3, b /= 3) plus
 * one byte for element 255; f16 d first. */
static float unpack_tq1_0(const uint8_t *blk, int8_t *out) {
    for (int i = 0; i < 51; i++) {
        unsigned b = blk[2 + i];
        for (int j = 0; j < 5; j++) {
            out[i * 5 + j] = (int8_t)((int)(b % 3) - 1);
            b /= 3;
        }
    }
    out[255] = (int8_t)((int)(blk[53] % 3) - 1);
    return or_f16_to_f32_finite(rd16(blk));
}

/* quant.rs:370-377 unpack_i2_s_block_i8: byte g -> elements g, 32+g, 64+g, 96+g from bits
 * [7:6], [5:4], [3:2], [1:0], each minus 1. */
static void unpack_i2_s(const uint8_t *blk, int8_t *out) {
    for (int g = 0; g < 32; g++) {
        uint8_t b = blk[g];
        out[g] = (int8_t)(((b >> 6) & 3) - 1);
        out[32 + g] = (int8_t)(((b >> 4) & 3) - 1);
        out[64 + g] = (int8_t)(((b >> 2) & 3) - 1);
        out[96 + g] = (int8_t)((b & 3) - 1);
    }
}

/* ime.rs:490-495 dot_i8_scalar */
static int32_t dot_i8(const int8_t *a, const int8_t *b, int n) {
    int32_t s = 0;
    for (int i = 0; i < n; i++) s += (int32_t)a[i] * b[i];
    return s;
}

/* quant_q8.rs:1992-2003: zero if xd == 0 or dw == 0; (float)dot * (dw * xd). */
float or_dot_tq2_0_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi_out) {
    int8_t wv[256];
    float dw = unpack_tq2_0(w, wv);
    int32_t s = dot_i8(wv, x->qs, 256);
    if (sumi_out) *sumi_out = s;
    if (x->d == 0.0f || dw == 0.0f) return 0.0f;
    return i2f(s) * (dw * x->d);
}

/* quant_q8.rs:1960-1972 dot_tq1_0_q8_k_block (the LUT restates the same base-3 digits). */
float or_dot_tq1_0_q8_k_block(const uint8_t *w, const or_block_q8_k *x, int32_t *sumi_out) {
    int8_t wv[256];
    float dw = unpack_tq1_0(w, wv);
    int32_t s = dot_i8(wv, x->qs, 256);
    if (sumi_out) *sumi_out = s;
    if (x->d == 0.0f || dw == 0.0f) return 0.0f;
    return i2f(s) * (dw * x->d);
}

/* ------------------------------------------------------------------------------------------ */
/* Format table                                                                                */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    int quant;
    size_t be, bb; /* block elements, block bytes */
    int act_k;     /* 1: BlockQ8K activations, 0: BlockQ8_0 */
    int dot;       /* 1: has an integer block dot / GEMV in the reference's quant_q8.rs */
} fmt_t;

static const fmt_t FMTS[] = {
    {OR_Q4_0, 32, 18, 0, 1},   {OR_Q8_0, 32, 34, 0, 1},    {OR_Q4_K, 256, 144, 1, 1},
    {OR_Q6_K, 256, 210, 1, 1}, {OR_TQ2_0, 256, 66, 1, 1}, {OR_TQ1_0, 256, 54, 1, 1},
    {OR_I2_S, 128, 32, 0, 1},  {OR_Q4_1, 32, 20, 0, 0},   {OR_IQ4_NL, 32, 18, 0, 0},
    {OR_Q5_0, 32, 22, 0, 1},   {OR_Q5_K, 256, 176, 1, 1},  {OR_Q5_1, 32, 24, 0, 0},
    {OR_Q2_K, 256, 84, 1, 0},  {OR_Q3_K, 256, 110, 1, 0},
};

static const fmt_t *fmt_of(int quant) {
    for (size_t i = 0; i < sizeof(FMTS) / sizeof(FMTS[0]); i++)
        if (FMTS[i].quant == quant) return &FMTS[i];
    return NULL;
}

/* The IQ4_NL non-linear code book (quant.rs:80-82, the published ggml table). */
static const int8_t OR_KVALUES_IQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                            1,    13,   25,  38,  53,  69,  89,  113};

/* Formats with a block dot against Q8 activations (GEMV, vec_dot, BitLinear paths). */
static const fmt_t *dot_fmt(int quant) {
    const fmt_t *f = fmt_of(quant);
    return f && f->dot ? f : NULL;
}

size_t or_weight_bytes(int quant, size_t rows, size_t cols) {
    const fmt_t *f = fmt_of(quant);
    if (!f || cols % f->be) return 0;
    return rows * (cols / f->be) * f->bb + (quant == OR_I2_S ? 32 : 0);
}

static float block_value(int quant, const uint8_t *w, const void *x, size_t b, int32_t *si,
                         int32_t *sm) {
    switch (quant) {
    case OR_Q4_0: return or_dot_q4_0_q8_0_block(w, (const or_block_q8_0 *)x + b, si);
    case OR_Q8_0: return or_dot_q8_0_q8_0_block(w, (const or_block_q8_0 *)x + b, si);
    case OR_Q4_K: return or_dot_q4_k_q8_k_block(w, (const or_block_q8_k *)x + b, si, sm);
    case OR_Q5_0: return or_dot_q5_0_q8_0_block(w, (const or_block_q8_0 *)x + b, si);
    case OR_Q5_K: return or_dot_q5_k_q8_k_block(w, (const or_block_q8_k *)x + b, si, sm);
    case OR_Q6_K: return or_dot_q6_k_q8_k_block(w, (const or_block_q8_k *)x + b, si);
    case OR_TQ2_0: return or_dot_tq2_0_q8_k_block(w, (const or_block_q8_k *)x + b, si);
    case OR_TQ1_0: return or_dot_tq1_0_q8_k_block(w, (const or_block_q8_k *)x + b, si);
    default: return 0.0f;
    }
}

int or_block_dots(int quant, const uint8_t *w, size_t rows, size_t cols, const void *x,
                  int32_t *sumi, int32_t *summins, float *contrib) {
    const fmt_t *f = dot_fmt(quant);
    if (!f || quant == OR_I2_S || cols % f->be) return 1;
    size_t nb = cols / f->be;
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < nb; b++) {
            int32_t si = 0, sm = 0;
            float v = block_value(quant, w + (r * nb + b) * f->bb, x, b, &si, &sm);
            if (sumi) sumi[r * nb + b] = si;
            if (summins) summins[r * nb + b] = sm;
            if (contrib) contrib[r * nb + b] = v;
        }
    return 0;
}

/* dot_*_row (quant_q8.rs:1217-1235, :2817-2830, :2972-3004): `.map(block).sum()` -> -0.0 start. */
float or_vec_dot(int quant, const uint8_t *w_row, const void *x, size_t n_blocks) {
    const fmt_t *f = dot_fmt(quant);
    if (!f) return NAN;
    float s = -0.0f;
    for (size_t b = 0; b < n_blocks; b++) s += block_value(quant, w_row + b * f->bb, x, b, 0, 0);
    return s;
}

/* run_4row_chunked_gemv (quant_q8.rs:1510-1560) over rows [r0, r1): groups of four rows
 * accumulate from 0.0 block by block; tail rows use the 1-row `.sum()` path. */
static void gemv_range(int quant, float *out, const uint8_t *w, size_t cols, const void *x,
                       size_t r0, size_t r1) {
    const fmt_t *f = dot_fmt(quant);
    size_t nb = cols / f->be, rs = nb * f->bb;
    size_t r = r0;
    for (; r + 4 <= r1; r += 4) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (size_t b = 0; b < nb; b++)
            for (int k = 0; k < 4; k++)
                acc[k] += block_value(quant, w + (r + k) * rs + b * f->bb, x, b, 0, 0);
        for (int k = 0; k < 4; k++) out[r - r0 + k] = acc[k];
    }
    for (; r < r1; r++) out[r - r0] = or_vec_dot(quant, w + r * rs, x, nb);
}

/* gemv_q4_0_q8_0 :1586, gemv_q8_0_q8_0 :1670, gemv_q4_k_q8_k :3101, gemv_q6_k_q8_k :3189,
 * gemv_tq1_0_q8_k :3221, gemv_tq2_0_q8_k :3250 (validation done by the caller). */
int or_gemv(int quant, float *out, const uint8_t *w, size_t rows, size_t cols, const void *x) {
    const fmt_t *f = dot_fmt(quant);
    if (!f || quant == OR_I2_S || cols == 0 || cols % f->be) return 1;
    gemv_range(quant, out, w, cols, x, 0, rows);
    return 0;
}

typedef struct {
    int quant;
    float *out;
    const uint8_t *w;
    size_t cols;
    const void *x;
    size_t r0, r1;
} gemv_job;

static void *gemv_job_run(void *p) {
    gemv_job *j = (gemv_job *)p;
    gemv_range(j->quant, j->out, j->w, j->cols, j->x, j->r0, j->r1);
    return NULL;
}

/* Row-range partitioned across threads, as a caller of gemv_repacked_rows (repack.rs:4014)
 * would split work. Output covers [row_begin, row_end). */
int or_gemv_rows_mt(int quant, float *out, const uint8_t *w, size_t rows, size_t cols,
                    const void *x, size_t row_begin, size_t row_end, int nthreads) {
    const fmt_t *f = dot_fmt(quant);
    if (!f || quant == OR_I2_S || cols % f->be || row_end > rows || row_begin > row_end) return 1;
    if (nthreads < 1) nthreads = 1;
    size_t n = row_end - row_begin;
    size_t per = ((n + nthreads - 1) / nthreads + 3) / 4 * 4;
    pthread_t th[256];
    gemv_job jobs[256];
    int nt = 0;
    for (size_t r = row_begin; r < row_end && nt < 256; r += per, nt++) {
        size_t e = r + per < row_end ? r + per : row_end;
        jobs[nt] = (gemv_job){quant, out + (r - row_begin), w, cols, x, r, e};
        pthread_create(&th[nt], NULL, gemv_job_run, &jobs[nt]);
    }
    for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* f32-activation host fallback: dequantize block -> f32 dot (quant.rs, lib.rs)                */
/* ------------------------------------------------------------------------------------------ */

/* unpack_q5_1_block_i8 (quant.rs:169-190): unsigned 5-bit codes (nibble | high bit << 4, the
 * high bits of elements j and j + 16 in bits j and j + 16 of qh); returns d and *m. */
static float unpack_q5_1(const uint8_t *blk, int8_t *q, float *m) {
    float d = or_f16_to_f32_finite(rd16(blk));
    *m = or_f16_to_f32_finite(rd16(blk + 2));
    uint32_t qh = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) | ((uint32_t)blk[6] << 16) |
                  ((uint32_t)blk[7] << 24);
    for (int j = 0; j < 16; j++) {
        q[j] = (int8_t)((blk[8 + j] & 0x0F) | (((qh >> j) & 1) << 4));
        q[j + 16] = (int8_t)(((blk[8 + j] >> 4) & 0x0F) | (((qh >> (j + 16)) & 1) << 4));
    }
    return d;
}

/* unpack_q2_k_block_i8 (quant.rs:198-246): 84-byte super-block = scales[16] (low nibble scale,
 * high nibble min), qs[64], f16 d, f16 dmin. Sub-block is (0..15) covers elements 16 is ..;
 * half h = is / 8, shift 2 * ((is % 8) / 2), bytes qs[32 h + 16 (is % 2) + l]. Codes 0..3,
 * scale d * (sc & 15), min dmin * (sc >> 4). */
static void unpack_q2_k(const uint8_t *blk, int8_t *q, float *sc, float *mn) {
    float d = or_f16_to_f32_finite(rd16(blk + 80)), dmin = or_f16_to_f32_finite(rd16(blk + 82));
    const uint8_t *qs = blk + 16;
    for (int is = 0; is < 16; is++) {
        int h = is / 8, shift = 2 * ((is % 8) / 2), half16 = is % 2;
        sc[is] = d * (float)(blk[is] & 0x0F);
        mn[is] = dmin * (float)(blk[is] >> 4);
        for (int l = 0; l < 16; l++)
            q[16 * is + l] = (int8_t)((qs[32 * h + 16 * half16 + l] >> shift) & 3);
    }
}

/* unpack_q3_k_block_i8 (quant.rs:255-330): 110-byte super-block = hmask[32], qs[64],
 * scales[12] (sixteen 6-bit values: low 4 bits from bytes 0..7, top 2 bits from bytes 8..11),
 * f16 d. Sub-block is: the 2-bit code of qs[32 h + 16 (is % 2) + l] at shift 2 ((is % 8) / 2),
 * minus 4 when bit (is / 2) of hmask[16 (is % 2) + l] is clear; scale d * (s6 - 32). */
static void unpack_q3_k(const uint8_t *blk, int8_t *q, float *sc) {
    const uint8_t *hm = blk, *qs = blk + 32, *raw = blk + 96;
    float d = or_f16_to_f32_finite(rd16(blk + 108));
    for (int is = 0; is < 16; is++) {
        int lo = is < 8 ? raw[is] & 0x0F : raw[is - 8] >> 4;
        int hi = (raw[8 + (is % 4)] >> (2 * (is / 4))) & 3;
        int s6 = lo | (hi << 4);
        sc[is] = d * (float)(s6 - 32);
        int h = is / 8, shift = 2 * ((is % 8) / 2), half16 = is % 2;
        for (int l = 0; l < 16; l++) {
            int code = (qs[32 * h + 16 * half16 + l] >> shift) & 3;
            int high = (hm[16 * half16 + l] >> (is / 2)) & 1;
            q[16 * is + l] = (int8_t)(code - (high ? 0 : 4));
        }
    }
}

/* quant.rs:551-568 (Q4_0), :570-588 (Q8_0), :594-648 (Q6_K), lib.rs:720-766 (Q4_K_M),
 * quant.rs:380-388 (I2_S with the tensor scale), ime.rs:636-658 / :595-624 (TQ2_0 / TQ1_0 times d). */
void or_dequantize_block(int quant, const uint8_t *blk, float i2s_scale, float *out) {
    switch (quant) {
    case OR_Q4_0: {
        float d = or_f16_to_f32_finite(rd16(blk));
        if (d == 0.0f) {
            memset(out, 0, 32 * sizeof(float));
            return;
        }
        for (int i = 0; i < 16; i++) {
            out[i] = d * (float)((int)(blk[2 + i] & 0x0F) - 8);
            out[i + 16] = d * (float)((int)((blk[2 + i] >> 4) & 0x0F) - 8);
        }
        return;
    }
    case OR_Q8_0: {
        float d = or_f16_to_f32_finite(rd16(blk));
        if (d == 0.0f) {
            memset(out, 0, 32 * sizeof(float));
            return;
        }
        for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)blk[2 + i];
        return;
    }
    case OR_Q6_K: {
        float d = or_f16_to_f32_finite(rd16(blk + 208));
        if (d == 0.0f) {
            memset(out, 0, 256 * sizeof(float));
            return;
        }
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        for (int h = 0; h < 2; h++) {
            int n = h * 128, lb = h * 64, hb = h * 32, sb = h * 8;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = (int)((ql[lb + l] & 0x0F) | ((qh[hb + l] & 3) << 4)) - 32;
                int q2 = (int)((ql[lb + l + 32] & 0x0F) | (((qh[hb + l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)(((ql[lb + l] >> 4) & 0x0F) | (((qh[hb + l] >> 4) & 3) << 4)) - 32;
                int q4 =
                    (int)(((ql[lb + l + 32] >> 4) & 0x0F) | (((qh[hb + l] >> 6) & 3) << 4)) - 32;
                out[n + l] = d * (float)sc[sb + is] * (float)q1;
                out[n + l + 32] = d * (float)sc[sb + is + 2] * (float)q2;
                out[n + l + 64] = d * (float)sc[sb + is + 4] * (float)q3;
                out[n + l + 96] = d * (float)sc[sb + is + 6] * (float)q4;
            }
        }
        return;
    }
    case OR_Q4_K: {
        float d = or_f16_to_f32_finite(rd16(blk));
        float dmin = or_f16_to_f32_finite(rd16(blk + 2));
        uint8_t sc[8], m[8];
        unpack_k4_scales(blk + 4, sc, m);
        const uint8_t *qs = blk + 16;
        for (int c = 0; c < 4; c++) {
            float d1 = d * (float)sc[2 * c], m1 = dmin * (float)m[2 * c];
            float d2 = d * (float)sc[2 * c + 1], m2 = dmin * (float)m[2 * c + 1];
            for (int l = 0; l < 32; l++) out[64 * c + l] = d1 * (float)(qs[32 * c + l] & 0x0F) - m1;
            for (int l = 0; l < 32; l++)
                out[64 * c + 32 + l] = d2 * (float)((qs[32 * c + l] >> 4) & 0x0F) - m2;
        }
        return;
    }
    case OR_Q5_0: {
        /* quant.rs:140-163: y = d * ((nibble | high bit << 4) - 16); zeros when d == 0 */
        float d = or_f16_to_f32_finite(rd16(blk));
        if (d == 0.0f) {
            memset(out, 0, 32 * sizeof(float));
            return;
        }
        uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) |
                      ((uint32_t)blk[5] << 24);
        for (int j = 0; j < 16; j++) {
            int q0 = (int)((blk[6 + j] & 0x0F) | (((qh >> j) & 1) << 4)) - 16;
            int q1 = (int)(((blk[6 + j] >> 4) & 0x0F) | (((qh >> (j + 16)) & 1) << 4)) - 16;
            out[j] = d * (float)q0;
            out[j + 16] = d * (float)q1;
        }
        return;
    }
    case OR_Q5_K: {
        /* quant.rs:651-705: y = (d * sc) * q - dmin * m, q = nibble + 16 * high bit; zeros when
         * d == dmin == 0 */
        float d = or_f16_to_f32_finite(rd16(blk)), dmin = or_f16_to_f32_finite(rd16(blk + 2));
        if (d == 0.0f && dmin == 0.0f) {
            memset(out, 0, 256 * sizeof(float));
            return;
        }
        uint8_t sc[8], m[8];
        unpack_k4_scales(blk + 4, sc, m);
        const uint8_t *qh = blk + 16, *qs = blk + 48;
        for (int c = 0; c < 4; c++) {
            float d1 = d * (float)sc[2 * c], m1 = dmin * (float)m[2 * c];
            float d2 = d * (float)sc[2 * c + 1], m2 = dmin * (float)m[2 * c + 1];
            for (int l = 0; l < 32; l++) {
                int q1 = (qs[32 * c + l] & 0x0F) + (((qh[l] >> (2 * c)) & 1) ? 16 : 0);
                out[64 * c + l] = d1 * (float)q1 - m1;
            }
            for (int l = 0; l < 32; l++) {
                int q2 = (qs[32 * c + l] >> 4) + (((qh[l] >> (2 * c + 1)) & 1) ? 16 : 0);
                out[64 * c + 32 + l] = d2 * (float)q2 - m2;
            }
        }
        return;
    }
    case OR_Q4_1: {
        /* quant.rs:118-136: y = d * q + m over unsigned nibbles; zeros when d == m == 0 */
        float d = or_f16_to_f32_finite(rd16(blk)), m = or_f16_to_f32_finite(rd16(blk + 2));
        if (d == 0.0f && m == 0.0f) {
            memset(out, 0, 32 * sizeof(float));
            return;
        }
        for (int i = 0; i < 16; i++) {
            out[i] = d * (float)(blk[4 + i] & 0x0F) + m;
            out[i + 16] = d * (float)((blk[4 + i] >> 4) & 0x0F) + m;
        }
        return;
    }
    case OR_IQ4_NL: {
        /* quant.rs:332-356: y = d * KVALUES_IQ4NL[nibble]; zeros when d == 0 */
        float d = or_f16_to_f32_finite(rd16(blk));
        if (d == 0.0f) {
            memset(out, 0, 32 * sizeof(float));
            return;
        }
        for (int i = 0; i < 16; i++) {
            out[i] = d * (float)OR_KVALUES_IQ4NL[blk[2 + i] & 0x0F];
            out[i + 16] = d * (float)OR_KVALUES_IQ4NL[blk[2 + i] >> 4];
        }
        return;
    }
    case OR_Q5_1: {
        /* quant.rs:192-196: y = d * q + m over unsigned 5-bit codes; zeros when d == m == 0 */
        int8_t q[32];
        float m, d = unpack_q5_1(blk, q, &m);
        if (d == 0.0f && m == 0.0f) {
            memset(out, 0, 32 * sizeof(float));
            return;
        }
        for (int i = 0; i < 32; i++) out[i] = d * (float)q[i] + m;
        return;
    }
    case OR_Q2_K: {
        /* quant.rs:249-252: y = dl * q - ml per 16-element sub-block */
        int8_t q[256];
        float sc[16], mn[16];
        unpack_q2_k(blk, q, sc, mn);
        for (int i = 0; i < 256; i++) out[i] = sc[i / 16] * (float)q[i] - mn[i / 16];
        return;
    }
    case OR_Q3_K: {
        /* quant.rs:333-342: y = dl * q per 16-element sub-block */
        int8_t q[256];
        float sc[16];
        unpack_q3_k(blk, q, sc);
        for (int i = 0; i < 256; i++) out[i] = sc[i / 16] * (float)q[i];
        return;
    }
    case OR_I2_S: {
        int8_t q[128];
        unpack_i2_s(blk, q);
        if (i2s_scale == 0.0f) {
            memset(out, 0, 128 * sizeof(float));
            return;
        }
        for (int i = 0; i < 128; i++) out[i] = i2s_scale * (float)q[i];
        return;
    }
    case OR_TQ2_0:
    case OR_TQ1_0: {
        int8_t q[256];
        float d = quant == OR_TQ2_0 ? unpack_tq2_0(blk, q) : unpack_tq1_0(blk, q);
        if (d == 0.0f) {
            memset(out, 0, 256 * sizeof(float));
            return;
        }
        for (int i = 0; i < 256; i++) out[i] = d * (float)q[i];
        return;
    }
    default: return;
    }
}

/* Whole-matrix dequantization (each block through or_dequantize_block) for f64 reference
 * products in the tests (the role of ref_matvec_blocks, tests/wave4_quant_gemv_and_argmax.rs:
 * 228-251). */
int or_dequantize_rows(int quant, const uint8_t *w, size_t rows, size_t cols, float *out) {
    const fmt_t *f = fmt_of(quant);
    if (!f || cols % f->be) return 1;
    size_t nb = cols / f->be;
    float i2s = 0.0f;
    if (quant == OR_I2_S) {
        memcpy(&i2s, w + rows * nb * f->bb, 4);
        if (!isfinite(i2s)) i2s = 0.0f;
    }
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < nb; b++)
            or_dequantize_block(quant, w + (r * nb + b) * f->bb, i2s, out + r * cols + b * f->be);
    return 0;
}

/* vec_dot_q4_0_scalar quant.rs:1401-1436, vec_dot_q8_0_scalar :899-934, vec_dot_q6_k_scalar
 * :1012-1047, vec_dot_q4_k_m_scalar lib.rs:1268-1303, vec_dot_i2_s quant.rs:2199-2240:
 * row_sum from 0.0 of per-block dot_product_f32_scalar; I2_S rows are 0.0 when the scale is 0. */
int or_vec_dot_f32(int quant, float *out, const uint8_t *w, size_t w_len, size_t rows,
                   size_t cols, const float *input) {
    const fmt_t *f = dot_fmt(quant);
    if (!f || cols % f->be || quant == OR_TQ1_0) return 1;
    size_t nb = cols / f->be;
    if (w_len < or_weight_bytes(quant, rows, cols)) return 1;
    float i2s = 0.0f;
    if (quant == OR_I2_S) {
        float v;
        memcpy(&v, w + rows * nb * f->bb, 4);
        i2s = isfinite(v) ? v : 0.0f;
    }
    float buf[256];
    for (size_t r = 0; r < rows; r++) {
        if (quant == OR_I2_S && i2s == 0.0f) {
            out[r] = 0.0f;
            continue;
        }
        float s = 0.0f;
        for (size_t b = 0; b < nb; b++) {
            or_dequantize_block(quant, w + (r * nb + b) * f->bb, i2s, buf);
            s += or_dot_product_f32(buf, input + b * f->be, f->be);
        }
        out[r] = s;
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* BitLinear (ime.rs:882-938)                                                                  */
/* ------------------------------------------------------------------------------------------ */

/* unpack_bitlinear_block_i8 ime.rs:792-871: returns block elements and the block scale. */
static int bitlinear_block(int quant, const uint8_t *blk, float i2s, int8_t *wv, float *scale) {
    switch (quant) {
    case OR_TQ1_0: *scale = unpack_tq1_0(blk, wv); return 256;
    case OR_TQ2_0: *scale = unpack_tq2_0(blk, wv); return 256;
    case OR_Q8_0:
        *scale = or_f16_to_f32_finite(rd16(blk));
        for (int i = 0; i < 32; i++) wv[i] = (int8_t)blk[2 + i];
        return 32;
    case OR_I2_S: unpack_i2_s(blk, wv); *scale = i2s; return 128;
    default: return 0;
    }
}

static void bitlinear_rows(float *out, int quant, const uint8_t *w, size_t rows, size_t cols,
                           const int8_t *act, float act_scale, float i2s, size_t r0, size_t r1) {
    const fmt_t *f = dot_fmt(quant);
    size_t nb = cols / f->be;
    int8_t wv[256];
    for (size_t r = r0; r < r1; r++) {
        float row_sum = 0.0f;
        for (size_t b = 0; b < nb; b++) {
            float bs = 0.0f;
            int n = bitlinear_block(quant, w + (r * nb + b) * f->bb, i2s, wv, &bs);
            int32_t d = dot_i8(wv, act + b * f->be, n);
            float eff = bs * act_scale;
            row_sum += (float)d * eff;
        }
        out[r] = row_sum;
    }
    (void)rows;
}

static float i2s_trailer(int quant, const uint8_t *w, size_t rows, size_t cols) {
    if (quant != OR_I2_S) return 0.0f;
    float v;
    memcpy(&v, w + rows * (cols / 128) * 32, 4);
    return isfinite(v) ? v : 0.0f;
}

/* bitlinear_i8_rvv ime.rs:882-938 (bitlinear_i8_ime :1005-1114 is bit-identical). */
int or_bitlinear_i8(float *out, int quant, const uint8_t *w, size_t w_len, size_t rows,
                    size_t cols, const int8_t *act, float act_scale) {
    const fmt_t *f = dot_fmt(quant);
    if (!f || (quant != OR_TQ1_0 && quant != OR_TQ2_0 && quant != OR_Q8_0 && quant != OR_I2_S))
        return 2;
    if (rows == 0 || cols == 0 || cols % f->be || w_len < or_weight_bytes(quant, rows, cols))
        return 1;
    bitlinear_rows(out, quant, w, rows, cols, act, act_scale, i2s_trailer(quant, w, rows, cols), 0,
                   rows);
    return 0;
}

typedef struct {
    float *out;
    int quant;
    const uint8_t *w;
    size_t rows, cols;
    const int8_t *act;
    const float *scales;
    float i2s;
    size_t t0, t1;
} bl_job;

static void *bl_job_run(void *p) {
    bl_job *j = (bl_job *)p;
    for (size_t t = j->t0; t < j->t1; t++)
        bitlinear_rows(j->out + t * j->rows, j->quant, j->w, j->rows, j->cols, j->act + t * j->cols,
                       j->scales[t], j->i2s, 0, j->rows);
    return NULL;
}

/* M tokens, each an independent bitlinear_i8 call (the reference path is M=1), threads split
 * the tokens. out is [m][rows]. */
int or_bitlinear_i8_rows_mt(float *out, int quant, const uint8_t *w, size_t w_len, size_t rows,
                            size_t cols, const int8_t *act, float act_scale, size_t m,
                            const float *act_scales, int nthreads) {
    const fmt_t *f = dot_fmt(quant);
    if (!f || cols % f->be || w_len < or_weight_bytes(quant, rows, cols)) return 1;
    (void)act_scale;
    if (nthreads < 1) nthreads = 1;
    if ((size_t)nthreads > m) nthreads = (int)m;
    pthread_t th[256];
    bl_job jobs[256];
    size_t per = (m + nthreads - 1) / nthreads;
    int nt = 0;
    float i2s = i2s_trailer(quant, w, rows, cols);
    for (size_t t = 0; t < m && nt < 256; t += per, nt++) {
        jobs[nt] = (bl_job){out, quant, w, rows, cols, act, act_scales, i2s, t,
                            t + per < m ? t + per : m};
        pthread_create(&th[nt], NULL, bl_job_run, &jobs[nt]);
    }
    for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Repacked block-scaled weights (repack.rs:1724-2103) and the scalar GEMM (:2995-3093)        */
/* ------------------------------------------------------------------------------------------ */

/* BlockScaledTileLayout::from_validated_dims repack.rs:1330-1366: Q6_K, Q3_K and Q2_K use
 * 16-element scale groups (chunks_per_scale = 1), every other format 32-element groups;
 * Q4_K_M, Q5_K, Q4_1, Q5_1 and Q2_K carry mins. */
static int g16(int quant) { return quant == OR_Q6_K || quant == OR_Q2_K || quant == OR_Q3_K; }

size_t or_repack_scale_groups(int quant, size_t cols) {
    size_t kp = (cols + 31) / 32 * 32;
    return g16(quant) ? kp / 16 : kp / 32;
}

int or_repack_has_mins(int quant) {
    return quant == OR_Q4_K || quant == OR_Q4_1 || quant == OR_Q5_K || quant == OR_Q5_1 ||
           quant == OR_Q2_K;
}

int or_repack_block_scaled(int quant, const uint8_t *raw, size_t raw_len, size_t rows,
                           size_t cols, int8_t *q, float *scales, float *mins) {
    const fmt_t *f = fmt_of(quant);
    if (!f || rows == 0 || cols == 0 || cols % f->be) return 1;
    if (raw_len < or_weight_bytes(quant, rows, cols)) return 1;
    size_t kp = (cols + 31) / 32 * 32, sg = or_repack_scale_groups(quant, cols);
    size_t nb = cols / f->be, rb = nb * f->bb;
    memset(q, 0, rows * kp);
    memset(scales, 0, rows * sg * sizeof(float));
    if (mins) memset(mins, 0, rows * sg * sizeof(float));
    float i2s = i2s_trailer(quant, raw, rows, cols);
    for (size_t r = 0; r < rows; r++) {
        const uint8_t *row = raw + r * rb;
        int8_t *qr = q + r * kp;
        float *sr = scales + r * sg;
        float *mr = mins ? mins + r * sg : NULL;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * f->bb;
            switch (quant) {
            case OR_Q8_0: {
                float d = or_f16_to_f32_finite(rd16(blk));
                sr[b] = d;
                if (d != 0.0f)
                    for (int i = 0; i < 32; i++) qr[32 * b + i] = (int8_t)blk[2 + i];
                break;
            }
            case OR_Q4_0: {
                float d = or_f16_to_f32_finite(rd16(blk));
                sr[b] = d;
                if (d != 0.0f)
                    for (int i = 0; i < 16; i++) {
                        qr[32 * b + i] = (int8_t)((blk[2 + i] & 0x0F) - 8);
                        qr[32 * b + 16 + i] = (int8_t)(((blk[2 + i] >> 4) & 0x0F) - 8);
                    }
                break;
            }
            case OR_Q4_K: {
                float d = or_f16_to_f32_finite(rd16(blk));
                float dmin = or_f16_to_f32_finite(rd16(blk + 2));
                uint8_t sc[8], m[8];
                unpack_k4_scales(blk + 4, sc, m);
                for (int c = 0; c < 4; c++) {
                    size_t g0 = b * 8 + 2 * c;
                    sr[g0] = d * (float)sc[2 * c];
                    mr[g0] = dmin * (float)m[2 * c];
                    sr[g0 + 1] = d * (float)sc[2 * c + 1];
                    mr[g0 + 1] = dmin * (float)m[2 * c + 1];
                    for (int l = 0; l < 32; l++) {
                        qr[256 * b + 64 * c + l] = (int8_t)(blk[16 + 32 * c + l] & 0x0F);
                        qr[256 * b + 64 * c + 32 + l] = (int8_t)((blk[16 + 32 * c + l] >> 4) & 0x0F);
                    }
                }
                break;
            }
            case OR_Q6_K: {
                float d = or_f16_to_f32_finite(rd16(blk + 208));
                for (int s = 0; s < 16; s++) sr[b * 16 + s] = d * (float)(int8_t)blk[192 + s];
                if (d != 0.0f) {
                    float tmp[256];
                    /* element values q - 32 (same unpack as the dequantizer, without scales) */
                    const uint8_t *ql = blk, *qh = blk + 128;
                    for (int h = 0; h < 2; h++)
                        for (int l = 0; l < 32; l++) {
                            int lb = 64 * h, hb = 32 * h, n = 128 * h;
                            tmp[n + l] = (float)((int)((ql[lb + l] & 0x0F) | ((qh[hb + l] & 3) << 4)) - 32);
                            tmp[n + l + 32] =
                                (float)((int)((ql[lb + l + 32] & 0x0F) | (((qh[hb + l] >> 2) & 3) << 4)) - 32);
                            tmp[n + l + 64] =
                                (float)((int)(((ql[lb + l] >> 4) & 0x0F) | (((qh[hb + l] >> 4) & 3) << 4)) - 32);
                            tmp[n + l + 96] = (float)(
                                (int)(((ql[lb + l + 32] >> 4) & 0x0F) | (((qh[hb + l] >> 6) & 3) << 4)) - 32);
                        }
                    for (int i = 0; i < 256; i++) qr[256 * b + i] = (int8_t)tmp[i];
                }
                break;
            }
            case OR_TQ2_0:
            case OR_TQ1_0: {
                int8_t t[256];
                float d = quant == OR_TQ2_0 ? unpack_tq2_0(blk, t) : unpack_tq1_0(blk, t);
                for (int s = 0; s < 8; s++) sr[b * 8 + s] = d;
                memcpy(qr + 256 * b, t, 256);
                break;
            }
            case OR_Q5_0: {
                /* repack.rs:1827-1840: scale d; quants (5-bit code - 16) left 0 when d == 0 */
                float d = or_f16_to_f32_finite(rd16(blk));
                sr[b] = d;
                uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) |
                              ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
                if (d != 0.0f)
                    for (int j = 0; j < 16; j++) {
                        qr[32 * b + j] =
                            (int8_t)((int)((blk[6 + j] & 0x0F) | (((qh >> j) & 1) << 4)) - 16);
                        qr[32 * b + 16 + j] = (int8_t)(
                            (int)(((blk[6 + j] >> 4) & 0x0F) | (((qh >> (j + 16)) & 1) << 4)) - 16);
                    }
                break;
            }
            case OR_Q5_K: {
                /* repack.rs:1959-1995: scales d * sc, mins dmin * m, unsigned 5-bit quants */
                float d = or_f16_to_f32_finite(rd16(blk));
                float dmin = or_f16_to_f32_finite(rd16(blk + 2));
                uint8_t sc[8], m[8];
                unpack_k4_scales(blk + 4, sc, m);
                const uint8_t *qh = blk + 16, *qs = blk + 48;
                for (int c = 0; c < 4; c++) {
                    size_t g0 = b * 8 + 2 * c;
                    sr[g0] = d * (float)sc[2 * c];
                    mr[g0] = dmin * (float)m[2 * c];
                    sr[g0 + 1] = d * (float)sc[2 * c + 1];
                    mr[g0 + 1] = dmin * (float)m[2 * c + 1];
                    for (int l = 0; l < 32; l++) {
                        qr[256 * b + 64 * c + l] =
                            (int8_t)((qs[32 * c + l] & 0x0F) + (((qh[l] >> (2 * c)) & 1) ? 16 : 0));
                        qr[256 * b + 64 * c + 32 + l] =
                            (int8_t)((qs[32 * c + l] >> 4) + (((qh[l] >> (2 * c + 1)) & 1) ? 16 : 0));
                    }
                }
                break;
            }
            case OR_Q4_1: {
                /* repack.rs:1814-1826: scale d, min -m (0.0 when m == 0), unsigned quants */
                float d = or_f16_to_f32_finite(rd16(blk)), m = or_f16_to_f32_finite(rd16(blk + 2));
                sr[b] = d;
                mr[b] = m == 0.0f ? 0.0f : -m;
                for (int i = 0; i < 16; i++) {
                    qr[32 * b + i] = (int8_t)(blk[4 + i] & 0x0F);
                    qr[32 * b + 16 + i] = (int8_t)((blk[4 + i] >> 4) & 0x0F);
                }
                break;
            }
            case OR_IQ4_NL: {
                /* repack.rs:1861-1873: scale d; quants left 0 when d == 0 */
                float d = or_f16_to_f32_finite(rd16(blk));
                sr[b] = d;
                if (d != 0.0f)
                    for (int i = 0; i < 16; i++) {
                        qr[32 * b + i] = OR_KVALUES_IQ4NL[blk[2 + i] & 0x0F];
                        qr[32 * b + 16 + i] = OR_KVALUES_IQ4NL[blk[2 + i] >> 4];
                    }
                break;
            }
            case OR_Q5_1: {
                /* repack.rs:1841-1855: scale d, min -m (0.0 when m == 0), unsigned 5-bit codes */
                float m, d = unpack_q5_1(blk, qr + 32 * b, &m);
                sr[b] = d;
                mr[b] = m == 0.0f ? 0.0f : -m;
                break;
            }
            case OR_Q2_K: {
                /* repack.rs:1874-1892: 16 (scale, min) pairs per super-block, codes 0..3 */
                unpack_q2_k(blk, qr + 256 * b, sr + 16 * b, mr + 16 * b);
                break;
            }
            case OR_Q3_K: {
                /* repack.rs:1893-1908: 16 signed scales per super-block, codes -4..3 */
                unpack_q3_k(blk, qr + 256 * b, sr + 16 * b);
                break;
            }
            case OR_I2_S: {
                int8_t t[128];
                unpack_i2_s(blk, t);
                for (int s = 0; s < 4; s++) sr[b * 4 + s] = i2s;
                if (i2s != 0.0f) memcpy(qr + 128 * b, t, 128);
                break;
            }
            default: return 1;
            }
        }
    }
    return 0;
}

typedef struct {
    float *out;
    int cps; /* 16-element chunks per scale group: 2 (32-element groups) or 1 (Q6_K/Q3_K/Q2_K) */
    const int8_t *wq;
    const float *ws, *wm;
    size_t cols;
    const int8_t *xq;
    const float *xs, *xsum, *xsum16;
    size_t m, row_begin, row_end, n0, n1;
} gemm_job;

/* execute_gemm_repacked_rows scalar branch repack.rs:2995-3025 + accumulate_scaled_tile_scalar
 * :3045-3093: per output, acc from 0.0; per scale group in K order, i32 group dot, then
 * acc += dot_f * (x_sc * ws) [- x_sum * wm]. Output [m][row_end - row_begin]. */
static void *gemm_job_run(void *p) {
    gemm_job *j = (gemm_job *)p;
    size_t kp = (j->cols + 31) / 32 * 32, kb = kp / 32, kc = kp / 16;
    int cps = j->cps;
    size_t gsz = 16 * (size_t)cps, sg = kp / gsz;
    size_t sub_n = j->row_end - j->row_begin;
    for (size_t n = j->n0; n < j->n1; n++) {
        const int8_t *wr = j->wq + n * kp;
        const float *wsr = j->ws + n * sg;
        const float *wmr = j->wm ? j->wm + n * sg : NULL;
        for (size_t mm = 0; mm < j->m; mm++) {
            const int8_t *xr = j->xq + mm * kp;
            float acc = 0.0f;
            for (size_t g = 0; g < sg; g++) {
                int32_t c = 0;
                for (size_t k = g * gsz; k < (g + 1) * gsz; k++) c += (int32_t)xr[k] * wr[k];
                size_t b32 = cps == 2 ? g : g / 2;
                float x_sc = j->xs[mm * kb + b32];
                float dot_f = (float)c;
                if (wmr) {
                    float xsm = cps == 2 ? j->xsum[mm * kb + b32] : j->xsum16[mm * kc + g];
                    acc += dot_f * (x_sc * wsr[g]) - xsm * wmr[g];
                } else {
                    acc += dot_f * (x_sc * wsr[g]);
                }
            }
            j->out[mm * sub_n + (n - j->row_begin)] = acc;
        }
    }
    return NULL;
}

static int gemm_run(float *out, int cps, const int8_t *wq, const float *ws, const float *wm,
                    size_t cols, const int8_t *xq, const float *xs, const float *xsum,
                    const float *xsum16, size_t m, size_t row_begin, size_t row_end,
                    int nthreads) {
    if (nthreads < 1) nthreads = 1;
    size_t n = row_end - row_begin;
    if (n == 0) return 0;
    size_t per = (n + nthreads - 1) / nthreads;
    pthread_t th[256];
    gemm_job jobs[256];
    int nt = 0;
    for (size_t r = row_begin; r < row_end && nt < 256; r += per, nt++) {
        jobs[nt] = (gemm_job){out,  cps,       wq,      ws,    wm, cols, xq,
                              xs,   xsum,      xsum16,  m,     row_begin, row_end,
                              r,    r + per < row_end ? r + per : row_end};
        pthread_create(&th[nt], NULL, gemm_job_run, &jobs[nt]);
    }
    for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
    return 0;
}

int or_gemm_repacked(float *out, int quant, const int8_t *wq, const float *ws, const float *wm,
                     size_t rows, size_t cols, const int8_t *xq, const float *xs,
                     const float *xsum, const float *xsum16, size_t m, size_t row_begin,
                     size_t row_end, int nthreads) {
    if (row_begin > row_end || row_end > rows || m == 0) return 1;
    if (or_repack_has_mins(quant) && (!wm || !xsum)) return 1;
    return gemm_run(out, g16(quant) ? 1 : 2, wq, ws, or_repack_has_mins(quant) ? wm : NULL,
                    cols, xq, xs, xsum, xsum16, m, row_begin, row_end, nthreads);
}

/* ------------------------------------------------------------------------------------------ */
/* Compact 4-bit nibble matrices (PackedNibbleMatrix, repack.rs:4188-5545)                      */
/* ------------------------------------------------------------------------------------------ */

int or_nibble_supported(int quant) {
    /* validate_nibble_quant, repack.rs:4231-4236 */
    return quant == OR_Q4_0 || quant == OR_Q4_1 || quant == OR_IQ4_NL || quant == OR_Q4_K;
}

/* pack_pair_split_nibbles_into_tile (repack.rs:4281-4305, scalar branch): even row in the low
 * nibbles, odd row in the high nibbles; bytes 0..64 hold columns 0..15 (low nibbles of the GGUF
 * bytes), bytes 64..128 columns 16..31 (high nibbles). */
static void pack_pair(const uint8_t *e, const uint8_t *o, uint8_t *tile, int pair) {
    for (int k = 0; k < 16; k++) {
        tile[pair * 16 + k] = (uint8_t)((e[k] & 0x0F) | ((o[k] & 0x0F) << 4));
        tile[64 + pair * 16 + k] = (uint8_t)((e[k] >> 4) | (o[k] & 0xF0));
    }
}

/* repack_nibble_into_tile_range over all tiles (repack.rs:4414-4645). Q4_0 / IQ4_NL blocks whose
 * scale decodes to zero (including non-finite scales) keep zero scale bits and zero nibbles. */
int or_nibble_pack_tiles(int quant, const uint8_t *raw, size_t raw_len, size_t rows, size_t cols,
                         uint8_t *tiles, uint16_t *scales_f16, uint16_t *mins_f16,
                         uint8_t *headers) {
    const fmt_t *f = fmt_of(quant);
    if (!or_nibble_supported(quant) || !f || rows == 0 || cols == 0 || cols % f->be) return 1;
    if (raw_len < or_weight_bytes(quant, rows, cols)) return 1;
    size_t nt_count = (rows + 7) / 8, kb = cols / 32, nsb = cols / 256;
    size_t rb = cols / f->be * f->bb;
    memset(tiles, 0, nt_count * kb * 128);
    if (quant == OR_Q4_K) {
        if (!headers) return 1;
        memset(headers, 0, nt_count * nsb * 8 * 16);
    } else {
        if (!scales_f16 || (quant == OR_Q4_1 && !mins_f16)) return 1;
        memset(scales_f16, 0, nt_count * kb * 8 * 2);
        if (quant == OR_Q4_1) memset(mins_f16, 0, nt_count * kb * 8 * 2);
    }
    static const uint8_t zero[32] = {0};
    for (size_t nt = 0; nt < nt_count; nt++) {
        uint8_t *tl = tiles + nt * kb * 128;
        for (int pair = 0; pair < 4; pair++) {
            size_t re = nt * 8 + 2 * (size_t)pair;
            if (re >= rows) break;
            int has_odd = re + 1 < rows;
            const uint8_t *er = raw + re * rb, *orw = has_odd ? raw + (re + 1) * rb : NULL;
            if (quant == OR_Q4_0 || quant == OR_IQ4_NL) {
                for (size_t b = 0; b < kb; b++) {
                    const uint8_t *be = er + b * 18;
                    uint16_t eb = rd16(be);
                    int ez = or_f16_to_f32_finite(eb) == 0.0f;
                    scales_f16[(nt * kb + b) * 8 + 2 * pair] = ez ? 0 : eb;
                    int oz = 1;
                    const uint8_t *no = zero;
                    if (has_odd) {
                        const uint8_t *bo = orw + b * 18;
                        uint16_t ob = rd16(bo);
                        oz = or_f16_to_f32_finite(ob) == 0.0f;
                        scales_f16[(nt * kb + b) * 8 + 2 * pair + 1] = oz ? 0 : ob;
                        if (!oz) no = bo + 2;
                    }
                    const uint8_t *ne = ez ? zero : be + 2;
                    if (!ez || !oz) pack_pair(ne, no, tl + b * 128, pair);
                }
            } else if (quant == OR_Q4_1) {
                for (size_t b = 0; b < kb; b++) {
                    const uint8_t *be = er + b * 20;
                    size_t ie = (nt * kb + b) * 8 + 2 * pair;
                    scales_f16[ie] = rd16(be);
                    mins_f16[ie] = rd16(be + 2);
                    const uint8_t *no = zero;
                    if (has_odd) {
                        const uint8_t *bo = orw + b * 20;
                        scales_f16[ie + 1] = rd16(bo);
                        mins_f16[ie + 1] = rd16(bo + 2);
                        no = bo + 4;
                    }
                    pack_pair(be + 4, no, tl + b * 128, pair);
                }
            } else { /* Q4_K_M: pack_q4k_pair_chunk32_into_tiles, repack.rs:4307-4392 */
                for (size_t sb = 0; sb < nsb; sb++) {
                    const uint8_t *be = er + sb * 144;
                    memcpy(headers + ((nt * nsb + sb) * 8 + 2 * pair) * 16, be, 16);
                    const uint8_t *bo = NULL;
                    if (has_odd) {
                        bo = orw + sb * 144;
                        memcpy(headers + ((nt * nsb + sb) * 8 + 2 * pair + 1) * 16, bo, 16);
                    }
                    for (int c = 0; c < 4; c++) {
                        const uint8_t *qe = be + 16 + 32 * c, *qo = bo ? bo + 16 + 32 * c : zero;
                        uint8_t *lo = tl + (sb * 8 + 2 * c) * 128, *hi = lo + 128;
                        for (int k = 0; k < 16; k++) {
                            lo[pair * 16 + k] = (uint8_t)((qe[k] & 0x0F) | ((qo[k] & 0x0F) << 4));
                            hi[pair * 16 + k] = (uint8_t)((qe[k] >> 4) | (qo[k] & 0xF0));
                            lo[64 + pair * 16 + k] =
                                (uint8_t)((qe[16 + k] & 0x0F) | ((qo[16 + k] & 0x0F) << 4));
                            hi[64 + pair * 16 + k] = (uint8_t)((qe[16 + k] >> 4) | (qo[16 + k] & 0xF0));
                        }
                    }
                }
            }
        }
    }
    return 0;
}

/* decode_tile_scales (repack.rs:5038-5092) and unpack_nibble_tile_to_chunks (:5095-5134), laid
 * out row-major for the checker: q [rows][cols] (Q4_0 nibble - 8, IQ4_NL code book, else the
 * unsigned nibble), ws [rows][cols / 32], wm [rows][cols / 32] (Q4_1: -m or 0.0; Q4_K_M:
 * dmin * m; untouched for formats without mins). */
int or_nibble_decode_tiles(int quant, size_t rows, size_t cols, const uint8_t *tiles,
                           const uint16_t *scales_f16, const uint16_t *mins_f16,
                           const uint8_t *headers, int8_t *q, float *ws, float *wm) {
    if (!or_nibble_supported(quant) || rows == 0 || cols == 0 || cols % 32) return 1;
    if (quant == OR_Q4_K && cols % 256) return 1;
    int mins = quant == OR_Q4_1 || quant == OR_Q4_K;
    if (mins && !wm) return 1;
    size_t kb = cols / 32, nsb = cols / 256;
    for (size_t r = 0; r < rows; r++) {
        size_t nt = r / 8, j = r % 8, pair = j / 2;
        int odd = (int)(j & 1);
        for (size_t b = 0; b < kb; b++) {
            const uint8_t *t = tiles + (nt * kb + b) * 128;
            for (int k = 0; k < 32; k++) {
                uint8_t byte = t[(k < 16 ? 0 : 64) + pair * 16 + (size_t)(k & 15)];
                uint8_t nib = odd ? (uint8_t)(byte >> 4) : (uint8_t)(byte & 0x0F);
                int8_t v = quant == OR_Q4_0      ? (int8_t)((int)nib - 8)
                           : quant == OR_IQ4_NL ? OR_KVALUES_IQ4NL[nib]
                                                : (int8_t)nib;
                q[r * cols + b * 32 + (size_t)k] = v;
            }
            size_t mi = (nt * kb + b) * 8 + j;
            if (quant == OR_Q4_0 || quant == OR_IQ4_NL) {
                ws[r * kb + b] = or_f16_to_f32_finite(scales_f16[mi]);
            } else if (quant == OR_Q4_1) {
                ws[r * kb + b] = or_f16_to_f32_finite(scales_f16[mi]);
                float m = or_f16_to_f32_finite(mins_f16[mi]);
                wm[r * kb + b] = m == 0.0f ? 0.0f : -m;
            }
        }
        if (quant == OR_Q4_K)
            for (size_t sb = 0; sb < nsb; sb++) {
                const uint8_t *h = headers + ((nt * nsb + sb) * 8 + j) * 16;
                float d = or_f16_to_f32_finite(rd16(h)), dmin = or_f16_to_f32_finite(rd16(h + 2));
                uint8_t sc[8], mm[8];
                unpack_k4_scales(h + 4, sc, mm);
                for (int is = 0; is < 8; is++) {
                    ws[r * kb + sb * 8 + (size_t)is] = d * (float)sc[is];
                    wm[r * kb + sb * 8 + (size_t)is] = dmin * (float)mm[is];
                }
            }
    }
    return 0;
}

/* PackedNibbleMatrix::dequantize_row (repack.rs:5001-5036): q * scale - min, min 0.0 for the
 * formats without mins. */
int or_nibble_dequantize_row(int quant, const int8_t *q, const float *ws, const float *wm,
                             size_t cols, size_t row, float *out) {
    if (!or_nibble_supported(quant) || cols % 32) return 1;
    int mins = quant == OR_Q4_1 || quant == OR_Q4_K;
    size_t kb = cols / 32;
    for (size_t b = 0; b < kb; b++) {
        float sc = ws[row * kb + b], mn = mins ? wm[row * kb + b] : 0.0f;
        for (int k = 0; k < 32; k++)
            out[b * 32 + (size_t)k] = (float)q[row * cols + b * 32 + (size_t)k] * sc - mn;
    }
    return 0;
}

/* execute_nibble_gemm_rows host branch (repack.rs:5181-5397): per output, acc from 0.0; per
 * 32-element block in K order the i32 dot of the unpacked tile, then
 * accumulate_scaled_tile_scalar (:3045-3093) with chunks_per_scale = 2 and the mins term for
 * Q4_1 / Q4_K_M. Output [m][row_end - row_begin]. */
int or_gemm_nibble(float *out, int quant, const int8_t *q, const float *ws, const float *wm,
                   size_t rows, size_t cols, const int8_t *xq, const float *xs,
                   const float *xsum, size_t m, size_t row_begin, size_t row_end, int nthreads) {
    if (!or_nibble_supported(quant) || cols % 32) return 1;
    if (row_begin > row_end || row_end > rows || m == 0) return 1;
    int mins = quant == OR_Q4_1 || quant == OR_Q4_K;
    if (mins && (!wm || !xsum)) return 1;
    return gemm_run(out, 2, q, ws, mins ? wm : NULL, cols, xq, xs, xsum, NULL, m, row_begin,
                    row_end, nthreads);
}

/* ------------------------------------------------------------------------------------------ */
/* Seeded synthetic inputs and this project's own weight quantizers                            */
/* ------------------------------------------------------------------------------------------ */

uint64_t or_splitmix64(uint64_t *state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* N(0, sigma) by Box-Muller over splitmix64 uniforms (53-bit, never exactly 0). */
void or_fill_normal(float *out, size_t n, uint64_t seed, float sigma) {
    uint64_t s = seed;
    for (size_t i = 0; i < n; i += 2) {
        double u1 = ((double)(or_splitmix64(&s) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        double u2 = ((double)(or_splitmix64(&s) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        out[i] = (float)(r * cos(6.283185307179586 * u2) * sigma);
        if (i + 1 < n) out[i + 1] = (float)(r * sin(6.283185307179586 * u2) * sigma);
    }
}

/* iid uniform on {-1, 0, +1}. */
void or_fill_ternary(int8_t *out, size_t n, uint64_t seed) {
    uint64_t s = seed;
    for (size_t i = 0; i < n; i++) out[i] = (int8_t)((int)((or_splitmix64(&s) >> 32) % 3) - 1);
}

static inline float f16r(float x) { return or_f16_to_f32_ieee(or_f32_to_f16(x)); }
static inline void wr16(uint8_t *p, uint16_t v) {
    p[0] = (uint8_t)(v & 0xFF);
    p[1] = (uint8_t)(v >> 8);
}

/* Q4_0: the published ggml reference rule (signed max / -8, q = min(15, trunc(x/d + 8.5))). */
static void quant_q4_0_block(const float *x, uint8_t *o) {
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < 32; i++)
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            mx = x[i];
        }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(o, or_f32_to_f16(d));
    for (int j = 0; j < 16; j++) {
        int q0 = (int)(x[j] * id + 8.5f), q1 = (int)(x[16 + j] * id + 8.5f);
        if (q0 > 15) q0 = 15;
        if (q1 > 15) q1 = 15;
        if (q0 < 0) q0 = 0;
        if (q1 < 0) q1 = 0;
        o[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* Q8_0: symmetric absmax / 127 with an f16 scale. */
static void quant_q8_0_block(const float *x, uint8_t *o) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(o, or_f32_to_f16(d));
    for (int i = 0; i < 32; i++) {
        float q = roundf(x[i] * id);
        if (q > 127.0f) q = 127.0f;
        if (q < -127.0f) q = -127.0f;
        o[2 + i] = (uint8_t)(int8_t)q;
    }
}

/* Q4_K: per 32-element sub-block an affine (scale, min) pair, both re-quantized to 6 bits
 * against super-block f16 d / dmin; packing is the inverse of the 12-byte unpack rule. */
static void quant_q4_k_block(const float *x, uint8_t *o) {
    float scale[8], minv[8], max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int i = 1; i < 32; i++) {
            lo = fminf(lo, x[32 * j + i]);
            hi = fmaxf(hi, x[32 * j + i]);
        }
        if (lo > 0.0f) lo = 0.0f;
        scale[j] = (hi - lo) / 15.0f;
        minv[j] = -lo;
        max_scale = fmaxf(max_scale, scale[j]);
        max_min = fmaxf(max_min, minv[j]);
    }
    float d = f16r(max_scale / 63.0f), dmin = f16r(max_min / 63.0f);
    uint8_t sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        int a = d > 0.0f ? (int)roundf(scale[j] / d) : 0;
        int b = dmin > 0.0f ? (int)roundf(minv[j] / dmin) : 0;
        sc[j] = (uint8_t)(a > 63 ? 63 : (a < 0 ? 0 : a));
        m[j] = (uint8_t)(b > 63 ? 63 : (b < 0 ? 0 : b));
    }
    wr16(o, or_f32_to_f16(d));
    wr16(o + 2, or_f32_to_f16(dmin));
    uint8_t *s = o + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((m[j + 4] & 0x0F) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        float ds = d * (float)sc[j], dm = dmin * (float)m[j];
        for (int i = 0; i < 32; i++) {
            int v = ds > 0.0f ? (int)roundf((x[32 * j + i] + dm) / ds) : 0;
            q[32 * j + i] = (uint8_t)(v > 15 ? 15 : (v < 0 ? 0 : v));
        }
    }
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++)
            o[16 + 32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

/* Q6_K: per 16-element sub-block scale absmax/31 re-quantized to i8 against an f16 d; values
 * q+32 in 0..63 packed into ql/qh as the Q6_K decoder (quant.rs:594-648) reads them. */
static void quant_q6_k_block(const float *x, uint8_t *o) {
    float s[16], smax = 0.0f;
    for (int j = 0; j < 16; j++) {
        float a = 0.0f;
        for (int i = 0; i < 16; i++) a = fmaxf(a, fabsf(x[16 * j + i]));
        s[j] = a / 31.0f;
        smax = fmaxf(smax, s[j]);
    }
    float d = f16r(smax / 127.0f);
    int8_t sc[16];
    for (int j = 0; j < 16; j++) {
        int v = d > 0.0f ? (int)roundf(s[j] / d) : 0;
        sc[j] = (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v));
    }
    uint8_t u[256];
    for (int j = 0; j < 16; j++) {
        float ds = d * (float)sc[j];
        for (int i = 0; i < 16; i++) {
            int v = ds != 0.0f ? (int)roundf(x[16 * j + i] / ds) : 0;
            if (v < -32) v = -32;
            if (v > 31) v = 31;
            u[16 * j + i] = (uint8_t)(v + 32);
        }
    }
    uint8_t *ql = o, *qh = o + 128;
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            int n = 128 * h;
            ql[64 * h + l] = (uint8_t)((u[n + l] & 0x0F) | ((u[n + l + 64] & 0x0F) << 4));
            ql[64 * h + l + 32] = (uint8_t)((u[n + l + 32] & 0x0F) | ((u[n + l + 96] & 0x0F) << 4));
            qh[32 * h + l] = (uint8_t)((u[n + l] >> 4) | ((u[n + l + 32] >> 4) << 2) |
                                       ((u[n + l + 64] >> 4) << 4) | ((u[n + l + 96] >> 4) << 6));
        }
    for (int j = 0; j < 16; j++) o[192 + j] = (uint8_t)sc[j];
    wr16(o + 208, or_f32_to_f16(d));
}

/* Q4_1: the published ggml reference rule (min / (max - min) / 15, q = min(15, trunc(x/d + 0.5))). */
static void quant_q4_1_block(const float *x, uint8_t *o) {
    float lo = x[0], hi = x[0];
    for (int i = 1; i < 32; i++) {
        lo = fminf(lo, x[i]);
        hi = fmaxf(hi, x[i]);
    }
    float d = (hi - lo) / 15.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(o, or_f32_to_f16(d));
    wr16(o + 2, or_f32_to_f16(lo));
    for (int j = 0; j < 16; j++) {
        int q0 = (int)((x[j] - lo) * id + 0.5f), q1 = (int)((x[16 + j] - lo) * id + 0.5f);
        if (q0 > 15) q0 = 15;
        if (q1 > 15) q1 = 15;
        o[4 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* IQ4_NL (this project's own rule): d = signed absmax / -127 so the extreme maps to code 0,
 * each element to its nearest code-book value, then one least-squares refit of d. */
static void quant_iq4_nl_block(const float *x, uint8_t *o) {
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < 32; i++)
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            mx = x[i];
        }
    float d = mx / -127.0f;
    uint8_t idx[32];
    for (int i = 0; i < 32; i++) {
        int best = 0;
        float be = INFINITY;
        for (int c = 0; c < 16; c++) {
            float e = fabsf(x[i] - d * (float)OR_KVALUES_IQ4NL[c]);
            if (e < be) {
                be = e;
                best = c;
            }
        }
        idx[i] = (uint8_t)best;
    }
    float sxv = 0.0f, svv = 0.0f;
    for (int i = 0; i < 32; i++) {
        float v = (float)OR_KVALUES_IQ4NL[idx[i]];
        sxv += x[i] * v;
        svv += v * v;
    }
    if (svv > 0.0f && d != 0.0f) d = sxv / svv;
    wr16(o, or_f32_to_f16(d));
    for (int j = 0; j < 16; j++) o[2 + j] = (uint8_t)(idx[j] | (idx[16 + j] << 4));
}

/* Q5_0: the published ggml reference rule (signed max / -16, q = min(31, trunc(x/d + 16.5)),
 * the fifth bits in qh). */
static void quant_q5_0_block(const float *x, uint8_t *o) {
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < 32; i++)
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            mx = x[i];
        }
    float d = mx / -16.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(o, or_f32_to_f16(d));
    uint32_t qh = 0;
    for (int j = 0; j < 16; j++) {
        int q0 = (int)(x[j] * id + 16.5f), q1 = (int)(x[16 + j] * id + 16.5f);
        if (q0 > 31) q0 = 31;
        if (q1 > 31) q1 = 31;
        if (q0 < 0) q0 = 0;
        if (q1 < 0) q1 = 0;
        o[6 + j] = (uint8_t)((q0 & 0x0F) | ((q1 & 0x0F) << 4));
        qh |= (uint32_t)((q0 >> 4) & 1) << j;
        qh |= (uint32_t)((q1 >> 4) & 1) << (j + 16);
    }
    o[2] = (uint8_t)qh;
    o[3] = (uint8_t)(qh >> 8);
    o[4] = (uint8_t)(qh >> 16);
    o[5] = (uint8_t)(qh >> 24);
}

/* Q5_K: the Q4_K rule with 5-bit codes (0..31), the fifth bits in qh[32]. */
static void quant_q5_k_block(const float *x, uint8_t *o) {
    float scale[8], minv[8], max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int i = 1; i < 32; i++) {
            lo = fminf(lo, x[32 * j + i]);
            hi = fmaxf(hi, x[32 * j + i]);
        }
        if (lo > 0.0f) lo = 0.0f;
        scale[j] = (hi - lo) / 31.0f;
        minv[j] = -lo;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (minv[j] > max_min) max_min = minv[j];
    }
    float d = max_scale / 63.0f, dmin = max_min / 63.0f;
    uint8_t ls[8], lm[8];
    for (int j = 0; j < 8; j++) {
        int a = d > 0.0f ? (int)lrintf(scale[j] / d) : 0, b = dmin > 0.0f ? (int)lrintf(minv[j] / dmin) : 0;
        ls[j] = (uint8_t)(a < 0 ? 0 : a > 63 ? 63 : a);
        lm[j] = (uint8_t)(b < 0 ? 0 : b > 63 ? 63 : b);
    }
    uint16_t dh = or_f32_to_f16(d), mh = or_f32_to_f16(dmin);
    wr16(o, dh);
    wr16(o + 2, mh);
    uint8_t *s = o + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((ls[j] & 63) | ((ls[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((lm[j] & 63) | ((lm[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((ls[j + 4] & 15) | ((lm[j + 4] & 15) << 4));
    }
    float df = or_f16_to_f32_ieee(dh), mf = or_f16_to_f32_ieee(mh);
    uint8_t *qh = o + 16, *qs = o + 48;
    memset(qh, 0, 32);
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++) {
            int q[2];
            for (int h = 0; h < 2; h++) {
                int j = 2 * c + h;
                float dl = df * (float)ls[j], ml = mf * (float)lm[j];
                int v = dl > 0.0f ? (int)lrintf((x[64 * c + 32 * h + l] + ml) / dl) : 0;
                q[h] = v < 0 ? 0 : v > 31 ? 31 : v;
            }
            qs[32 * c + l] = (uint8_t)((q[0] & 15) | ((q[1] & 15) << 4));
            qh[l] |= (uint8_t)(((q[0] >> 4) << (2 * c)) | ((q[1] >> 4) << (2 * c + 1)));
        }
}

int or_quantize_weights(int quant, const float *w, size_t rows, size_t cols, uint8_t *out) {
    const fmt_t *f = fmt_of(quant);
    if (!f || cols % f->be) return 1;
    size_t nb = cols / f->be;
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < nb; b++) {
            const float *x = w + r * cols + b * f->be;
            uint8_t *o = out + (r * nb + b) * f->bb;
            switch (quant) {
            case OR_Q4_0: quant_q4_0_block(x, o); break;
            case OR_Q8_0: quant_q8_0_block(x, o); break;
            case OR_Q4_K: quant_q4_k_block(x, o); break;
            case OR_Q6_K: quant_q6_k_block(x, o); break;
            case OR_Q4_1: quant_q4_1_block(x, o); break;
            case OR_Q5_0: quant_q5_0_block(x, o); break;
            case OR_Q5_K: quant_q5_k_block(x, o); break;
            case OR_IQ4_NL: quant_iq4_nl_block(x, o); break;
            default: return 1;
            }
        }
    return 0;
}

/* Ternary packers (layouts of ime.rs:595-658 and quant.rs:360-377): TQ2_0 / TQ1_0 carry the
 * f16 scale in every block; I2_S carries one f32 scale in a 32-byte trailer. */
int or_pack_ternary(int quant, const int8_t *t, size_t rows, size_t cols, float scale,
                    uint8_t *out) {
    const fmt_t *f = fmt_of(quant);
    if (!f || cols % f->be) return 1;
    size_t nb = cols / f->be;
    uint16_t h = or_f32_to_f16(scale);
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < nb; b++) {
            const int8_t *x = t + r * cols + b * f->be;
            uint8_t *o = out + (r * nb + b) * f->bb;
            switch (quant) {
            case OR_TQ2_0:
                wr16(o, h);
                for (int i = 0; i < 64; i++)
                    o[2 + i] = (uint8_t)((x[4 * i] + 1) | ((x[4 * i + 1] + 1) << 2) |
                                         ((x[4 * i + 2] + 1) << 4) | ((x[4 * i + 3] + 1) << 6));
                break;
            case OR_TQ1_0:
                wr16(o, h);
                for (int i = 0; i < 51; i++) {
                    int v = 0, p = 1;
                    for (int j = 0; j < 5; j++) {
                        v += (x[5 * i + j] + 1) * p;
                        p *= 3;
                    }
                    o[2 + i] = (uint8_t)v;
                }
                o[53] = (uint8_t)(x[255] + 1);
                break;
            case OR_I2_S:
                for (int g = 0; g < 32; g++)
                    o[g] = (uint8_t)(((x[g] + 1) << 6) | ((x[32 + g] + 1) << 4) |
                                     ((x[64 + g] + 1) << 2) | (x[96 + g] + 1));
                break;
            default: return 1;
            }
        }
    if (quant == OR_I2_S) {
        uint8_t *tr = out + rows * nb * f->bb;
        memset(tr, 0, 32);
        memcpy(tr, &scale, 4);
    }
    return 0;
}
