// Single-row block dots over raw GGUF bytes (vec_dot_*_q8_*), the f32-activation
// VectorKernel entries (dequantize -> f32 dot) and the BitLinear ABI glue.
#include <cstring>

#include "gpu_layout.cuh"
#include "jkb_internal.h"

namespace jkb {

__device__ __forceinline__ uint32_t rd16d(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
__device__ __forceinline__ float f16_fin(uint32_t bits) {
    float v = __half2float(__ushort_as_half((unsigned short)bits));
    return ((bits >> 10) & 0x1F) == 0x1F ? 0.0f : v;
}

// ---------------------------------------------------------------- raw GGUF block dots
// Device restatements of the block functions on the original 18/34/144/210/54/66-byte layout
// (quant_q8.rs:672-717, :1834-1862, :1903-1942, :1960-2003).

__device__ float raw_block(int quant, const uint8_t *w, const uint8_t *xb) {
    if (quant == JKB_Q5_0) {  // quant_q8.rs:688-703
        float xd = *reinterpret_cast<const float *>(xb);
        const int8_t *xq = reinterpret_cast<const int8_t *>(xb + 4);
        float dw = f16_fin(rd16d(w));
        const uint32_t qh = (uint32_t)w[2] | ((uint32_t)w[3] << 8) | ((uint32_t)w[4] << 16) |
                            ((uint32_t)w[5] << 24);
        int sumi = 0;
        for (int j = 0; j < 16; j++) {
            const int q0 = (int)((w[6 + j] & 0x0F) | (((qh >> j) & 1) << 4)) - 16;
            const int q1 = (int)((w[6 + j] >> 4) | (((qh >> (j + 16)) & 1) << 4)) - 16;
            sumi += q0 * xq[j] + q1 * xq[j + 16];
        }
        if (dw == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn((float)sumi, __fmul_rn(dw, xd));
    }
    if (quant == JKB_Q4_0 || quant == JKB_Q8_0) {
        float xd = *reinterpret_cast<const float *>(xb);
        const int8_t *xq = reinterpret_cast<const int8_t *>(xb + 4);
        float dw = f16_fin(rd16d(w));
        int sumi = 0;
        if (quant == JKB_Q4_0) {
            for (int i = 0; i < 16; i++)
                sumi += ((int)(w[2 + i] & 0x0F) - 8) * xq[i] + ((int)(w[2 + i] >> 4) - 8) * xq[i + 16];
        } else {
            for (int i = 0; i < 32; i++) sumi += (int)(int8_t)w[2 + i] * xq[i];
        }
        if (dw == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn((float)sumi, __fmul_rn(dw, xd));
    }
    float xd = *reinterpret_cast<const float *>(xb);
    const int8_t *xq = reinterpret_cast<const int8_t *>(xb + 4);
    const int16_t *bs = reinterpret_cast<const int16_t *>(xb + 260);
    switch (quant) {
    case JKB_Q4_K_M: {
        float d = f16_fin(rd16d(w)), dmin = f16_fin(rd16d(w + 2));
        const uint8_t *s = w + 4;
        int sumi = 0, mins = 0;
        for (int c = 0; c < 4; c++) {
            int j0 = 2 * c, j1 = 2 * c + 1;
            int sc0 = j0 < 4 ? (s[j0] & 63) : ((s[j0 + 4] & 0x0F) | ((s[j0 - 4] >> 6) << 4));
            int sc1 = j1 < 4 ? (s[j1] & 63) : ((s[j1 + 4] & 0x0F) | ((s[j1 - 4] >> 6) << 4));
            int m0 = j0 < 4 ? (s[j0 + 4] & 63) : ((s[j0 + 4] >> 4) | ((s[j0] >> 6) << 4));
            int m1 = j1 < 4 ? (s[j1 + 4] & 63) : ((s[j1 + 4] >> 4) | ((s[j1] >> 6) << 4));
            int lo = 0, hi = 0;
            for (int l = 0; l < 32; l++) {
                uint8_t b = w[16 + 32 * c + l];
                lo += (int)(b & 0x0F) * xq[64 * c + l];
                hi += (int)(b >> 4) * xq[64 * c + 32 + l];
            }
            sumi += sc0 * lo + sc1 * hi;
            mins += m0 * ((int)bs[4 * c] + bs[4 * c + 1]) + m1 * ((int)bs[4 * c + 2] + bs[4 * c + 3]);
        }
        if ((d == 0.0f && dmin == 0.0f) || xd == 0.0f) return 0.0f;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, xd), (float)sumi),
                         __fmul_rn(__fmul_rn(dmin, xd), (float)mins));
    }
    case JKB_Q5_K: {  // quant_q8.rs:1866-1899
        float d = f16_fin(rd16d(w)), dmin = f16_fin(rd16d(w + 2));
        const uint8_t *s = w + 4, *qh = w + 16, *qs = w + 48;
        int sumi = 0, mins = 0;
        for (int c = 0; c < 4; c++) {
            int j0 = 2 * c, j1 = 2 * c + 1;
            int sc0 = j0 < 4 ? (s[j0] & 63) : ((s[j0 + 4] & 0x0F) | ((s[j0 - 4] >> 6) << 4));
            int sc1 = j1 < 4 ? (s[j1] & 63) : ((s[j1 + 4] & 0x0F) | ((s[j1 - 4] >> 6) << 4));
            int m0 = j0 < 4 ? (s[j0 + 4] & 63) : ((s[j0 + 4] >> 4) | ((s[j0] >> 6) << 4));
            int m1 = j1 < 4 ? (s[j1 + 4] & 63) : ((s[j1 + 4] >> 4) | ((s[j1] >> 6) << 4));
            int lo = 0, hi = 0;
            for (int l = 0; l < 32; l++) {
                uint8_t b = qs[32 * c + l];
                lo += ((int)(b & 0x0F) | (((qh[l] >> j0) & 1) << 4)) * xq[64 * c + l];
                hi += ((int)(b >> 4) | (((qh[l] >> j1) & 1) << 4)) * xq[64 * c + 32 + l];
            }
            sumi += sc0 * lo + sc1 * hi;
            mins += m0 * ((int)bs[4 * c] + bs[4 * c + 1]) + m1 * ((int)bs[4 * c + 2] + bs[4 * c + 3]);
        }
        if ((d == 0.0f && dmin == 0.0f) || xd == 0.0f) return 0.0f;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, xd), (float)sumi),
                         __fmul_rn(__fmul_rn(dmin, xd), (float)mins));
    }
    case JKB_Q6_K: {
        float d = f16_fin(rd16d(w + 208));
        const uint8_t *ql = w, *qh = w + 128;
        const int8_t *sc = reinterpret_cast<const int8_t *>(w + 192);
        int sumi = 0;
        for (int h = 0; h < 2; h++)
            for (int is = 0; is < 2; is++) {
                int s1 = 0, s2 = 0, s3 = 0, s4 = 0;
                for (int l = 16 * is; l < 16 * is + 16; l++) {
                    uint8_t a = ql[64 * h + l], b = ql[64 * h + l + 32], hb = qh[32 * h + l];
                    s1 += ((int)((a & 0x0F) | ((hb & 3) << 4)) - 32) * xq[128 * h + l];
                    s2 += ((int)((b & 0x0F) | (((hb >> 2) & 3) << 4)) - 32) * xq[128 * h + l + 32];
                    s3 += ((int)((a >> 4) | (((hb >> 4) & 3) << 4)) - 32) * xq[128 * h + l + 64];
                    s4 += ((int)((b >> 4) | (((hb >> 6) & 3) << 4)) - 32) * xq[128 * h + l + 96];
                }
                int o = 8 * h + is;
                sumi += sc[o] * s1 + sc[o + 2] * s2 + sc[o + 4] * s3 + sc[o + 6] * s4;
            }
        if (d == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn(__fmul_rn(d, xd), (float)sumi);
    }
    case JKB_TQ2_0:
    case JKB_TQ1_0: {
        int sumi = 0;
        if (quant == JKB_TQ2_0) {
            for (int e = 0; e < 256; e++)
                sumi += ((int)((w[2 + e / 4] >> (2 * (e % 4))) & 3) - 1) * xq[e];
        } else {
            for (int i = 0; i < 51; i++) {
                unsigned v = w[2 + i];
                for (int j = 0; j < 5; j++) {
                    sumi += ((int)(v % 3) - 1) * xq[5 * i + j];
                    v /= 3;
                }
            }
            sumi += ((int)(w[53] % 3) - 1) * xq[255];
        }
        if (xd == 0.0f) return 0.0f;
        float dw = f16_fin(rd16d(w));
        if (dw == 0.0f) return 0.0f;
        return __fmul_rn((float)sumi, __fmul_rn(dw, xd));
    }
    default: return 0.0f;
    }
}

// dot_*_row (quant_q8.rs:1217-1235, :2817-2830, :2972-3004): block values in parallel, then
// the reference's sequential `.sum()` (from -0.0) in block order by one thread.
__global__ void vec_dot_raw_kernel(int quant, const uint8_t *__restrict__ w, int bb,
                                   const uint8_t *__restrict__ x, int xbb, int nb,
                                   float *__restrict__ result) {
    extern __shared__ float vals[];
    for (int b = threadIdx.x; b < nb; b += blockDim.x)
        vals[b] = raw_block(quant, w + (size_t)b * bb, x + (size_t)b * xbb);
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = -0.0f;
        for (int b = 0; b < nb; b++) s = __fadd_rn(s, vals[b]);
        *result = s;
    }
}

static int vec_dot_raw(const char *fn, int quant, const uint8_t *w, size_t w_len,
                       const void *x, size_t x_len, float *result, void *stream) {
    const Fmt *f = fmt_of(quant);
    // validate_q8_block_row_bytes (quant_q8.rs:648-667)
    if (x_len == 0 || w_len != x_len * (size_t)f->block_bytes)
        return fail(JKB_E_BOUNDS, fn, 0, w_len, x_len * f->block_bytes,
                    "%s: expected %zu weight bytes for %zu blocks, got %zu", fn,
                    x_len * (size_t)f->block_bytes, x_len, w_len);
    if (!w || !x || !result) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    int rc;
    if ((rc = check_align(x, 4, fn, "x_blocks")) || (rc = check_align(result, 4, fn, "result")) ||
        (rc = push_reject(result, result + 1, fn)))
        return rc;
    if (x_len > 16384)
        return fail(JKB_E_BOUNDS, fn, 0, x_len, 16384, "%s: %zu blocks exceed the 16384-block row "
                    "limit of the GPU kernel", fn, x_len);
    int xbb = (quant == JKB_Q4_0 || quant == JKB_Q8_0 || quant == JKB_Q5_0) ? 36 : 292;
    vec_dot_raw_kernel<<<1, 256, x_len * sizeof(float), as_stream(stream)>>>(
        quant, w, f->block_bytes, (const uint8_t *)x, xbb, (int)x_len, result);
    return check_launch(fn);
}

// ---------------------------------------------------------------- f32-activation GEMV
// VectorKernel host fallback (lib.rs:1268-1303, quant.rs:899-934, :1012-1047, :1401-1436,
// :2199-2240): per block, dequantize (same f32 expression as the reference dequantizer) and
// take the sequential f32 dot from 0.0; the row sums the block dots sequentially from 0.0.
// One warp per row, one lane per block, in-order row sum by lane 0 -> bit-exact.

struct DqArgs {
    const uint8_t *qs;
    size_t qs_row;
    const uint8_t *sc;
    size_t sc_row;
    const uint16_t *d;
    float i2s;
    int quant, gpu_format, nb, be;
    const float *x;
    float *out;
    size_t rows;
};

__device__ float block_dot_f32(const DqArgs &a, size_t r, int b) {
    const float *x = a.x + (size_t)b * a.be;
    // the block's quant bytes in GGUF order (gathered from the lane-interleaved chunks)
    uint8_t q[192];
    const int qch = qs_chunks(a.gpu_format);
    const uint8_t *rowp = a.qs + r * a.qs_row;
    for (int j = 0; j < qch; j++) {
        const uint8_t *c = rowp + qs_chunk_offset(a.nb, qch, b, j);
        for (int i = 0; i < 16; i++) q[16 * j + i] = c[i];
    }
    float s = 0.0f;
    switch (a.quant) {
    case JKB_Q4_0: {
        float d = f16_fin(a.d[r * a.nb + b]);
        for (int i = 0; i < 32; i++) {
            int n = i < 16 ? (q[i] & 0x0F) : (q[i - 16] >> 4);
            float v = d == 0.0f ? 0.0f : __fmul_rn(d, (float)(n - 8));
            s = __fadd_rn(s, __fmul_rn(v, x[i]));
        }
        return s;
    }
    case JKB_Q8_0: {
        float d = f16_fin(a.d[r * a.nb + b]);
        for (int i = 0; i < 32; i++) {
            float v = d == 0.0f ? 0.0f : __fmul_rn(d, (float)(int8_t)q[i]);
            s = __fadd_rn(s, __fmul_rn(v, x[i]));
        }
        return s;
    }
    case JKB_Q4_K_M: {
        const uint8_t *sv = a.sc + r * a.sc_row + 16 * (size_t)b;
        float d = f16_fin(rd16d(sv)), dmin = f16_fin(rd16d(sv + 2));
        const uint8_t *s6 = sv + 4;
        for (int c = 0; c < 4; c++) {
            int j0 = 2 * c, j1 = 2 * c + 1;
            int sc0 = j0 < 4 ? (s6[j0] & 63) : ((s6[j0 + 4] & 0x0F) | ((s6[j0 - 4] >> 6) << 4));
            int sc1 = j1 < 4 ? (s6[j1] & 63) : ((s6[j1 + 4] & 0x0F) | ((s6[j1 - 4] >> 6) << 4));
            int m0 = j0 < 4 ? (s6[j0 + 4] & 63) : ((s6[j0 + 4] >> 4) | ((s6[j0] >> 6) << 4));
            int m1 = j1 < 4 ? (s6[j1 + 4] & 63) : ((s6[j1 + 4] >> 4) | ((s6[j1] >> 6) << 4));
            float d1 = __fmul_rn(d, (float)sc0), mm1 = __fmul_rn(dmin, (float)m0);
            float d2 = __fmul_rn(d, (float)sc1), mm2 = __fmul_rn(dmin, (float)m1);
            for (int l = 0; l < 32; l++) {
                float v = __fsub_rn(__fmul_rn(d1, (float)(q[32 * c + l] & 0x0F)), mm1);
                s = __fadd_rn(s, __fmul_rn(v, x[64 * c + l]));
            }
            for (int l = 0; l < 32; l++) {
                float v = __fsub_rn(__fmul_rn(d2, (float)(q[32 * c + l] >> 4)), mm2);
                s = __fadd_rn(s, __fmul_rn(v, x[64 * c + 32 + l]));
            }
        }
        return s;
    }
    case JKB_Q5_0: {  // dequantize_q5_0_block (quant.rs:140-163); qh in the scale plane
        float d = f16_fin(a.d[r * a.nb + b]);
        const uint8_t *hp = a.sc + r * a.sc_row + 4 * (size_t)b;
        const uint32_t qh = (uint32_t)hp[0] | ((uint32_t)hp[1] << 8) | ((uint32_t)hp[2] << 16) |
                            ((uint32_t)hp[3] << 24);
        for (int i = 0; i < 32; i++) {
            int n = i < 16 ? (q[i] & 0x0F) : (q[i - 16] >> 4);
            n |= (int)((qh >> i) & 1) << 4;
            float v = d == 0.0f ? 0.0f : __fmul_rn(d, (float)(n - 16));
            s = __fadd_rn(s, __fmul_rn(v, x[i]));
        }
        return s;
    }
    case JKB_Q5_K: {  // dequantize_q5_k_block (quant.rs:651-705); q = qs[128] | qh[32]
        const uint8_t *sv = a.sc + r * a.sc_row + 16 * (size_t)b;
        float d = f16_fin(rd16d(sv)), dmin = f16_fin(rd16d(sv + 2));
        if (d == 0.0f && dmin == 0.0f) {
            for (int e = 0; e < 256; e++) s = __fadd_rn(s, __fmul_rn(0.0f, x[e]));
            return s;
        }
        const uint8_t *s6 = sv + 4, *qh = q + 128;
        for (int c = 0; c < 4; c++) {
            int j0 = 2 * c, j1 = 2 * c + 1;
            int sc0 = j0 < 4 ? (s6[j0] & 63) : ((s6[j0 + 4] & 0x0F) | ((s6[j0 - 4] >> 6) << 4));
            int sc1 = j1 < 4 ? (s6[j1] & 63) : ((s6[j1 + 4] & 0x0F) | ((s6[j1 - 4] >> 6) << 4));
            int m0 = j0 < 4 ? (s6[j0 + 4] & 63) : ((s6[j0 + 4] >> 4) | ((s6[j0] >> 6) << 4));
            int m1 = j1 < 4 ? (s6[j1 + 4] & 63) : ((s6[j1 + 4] >> 4) | ((s6[j1] >> 6) << 4));
            float d1 = __fmul_rn(d, (float)sc0), mm1 = __fmul_rn(dmin, (float)m0);
            float d2 = __fmul_rn(d, (float)sc1), mm2 = __fmul_rn(dmin, (float)m1);
            for (int l = 0; l < 32; l++) {
                int n = (q[32 * c + l] & 0x0F) + (((qh[l] >> j0) & 1) ? 16 : 0);
                float v = __fsub_rn(__fmul_rn(d1, (float)n), mm1);
                s = __fadd_rn(s, __fmul_rn(v, x[64 * c + l]));
            }
            for (int l = 0; l < 32; l++) {
                int n = (q[32 * c + l] >> 4) + (((qh[l] >> j1) & 1) ? 16 : 0);
                float v = __fsub_rn(__fmul_rn(d2, (float)n), mm2);
                s = __fadd_rn(s, __fmul_rn(v, x[64 * c + 32 + l]));
            }
        }
        return s;
    }
    case JKB_Q6_K: {  // dequantize_q6_k_block (quant.rs:594-648); q = ql[128] | qh[64]
        const int8_t *sc = reinterpret_cast<const int8_t *>(a.sc + r * a.sc_row + 16 * (size_t)b);
        float d = f16_fin(a.d[r * a.nb + b]);
        const uint8_t *ql = q, *qh = q + 128;
        float vals[256];
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 32; l++) {
                int lb = 64 * h, hb = 32 * h, n = 128 * h, is = l / 16, sb = 8 * h;
                int q1 = (int)((ql[lb + l] & 0x0F) | ((qh[hb + l] & 3) << 4)) - 32;
                int q2 = (int)((ql[lb + l + 32] & 0x0F) | (((qh[hb + l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)((ql[lb + l] >> 4) | (((qh[hb + l] >> 4) & 3) << 4)) - 32;
                int q4 = (int)((ql[lb + l + 32] >> 4) | (((qh[hb + l] >> 6) & 3) << 4)) - 32;
                vals[n + l] = __fmul_rn(__fmul_rn(d, (float)sc[sb + is]), (float)q1);
                vals[n + l + 32] = __fmul_rn(__fmul_rn(d, (float)sc[sb + is + 2]), (float)q2);
                vals[n + l + 64] = __fmul_rn(__fmul_rn(d, (float)sc[sb + is + 4]), (float)q3);
                vals[n + l + 96] = __fmul_rn(__fmul_rn(d, (float)sc[sb + is + 6]), (float)q4);
            }
        for (int e = 0; e < 256; e++) {
            float v = d == 0.0f ? 0.0f : vals[e];
            s = __fadd_rn(s, __fmul_rn(v, x[e]));
        }
        return s;
    }
    case JKB_I2_S: {
        float vals[128];
        for (int g = 0; g < 32; g++) {
            vals[g] = (float)((int)((q[g] >> 6) & 3) - 1);
            vals[32 + g] = (float)((int)((q[g] >> 4) & 3) - 1);
            vals[64 + g] = (float)((int)((q[g] >> 2) & 3) - 1);
            vals[96 + g] = (float)((int)(q[g] & 3) - 1);
        }
        for (int e = 0; e < 128; e++) {
            float v = a.i2s == 0.0f ? 0.0f : __fmul_rn(a.i2s, vals[e]);
            s = __fadd_rn(s, __fmul_rn(v, x[e]));
        }
        return s;
    }
    default: return 0.0f;
    }
}

__global__ void __launch_bounds__(256) vec_dot_f32_kernel(DqArgs a) {
    const int lane = threadIdx.x & 31;
    const size_t row = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= a.rows) return;
    if (a.quant == JKB_I2_S && a.i2s == 0.0f) {  // quant.rs:2214-2217
        if (lane == 0) a.out[row] = 0.0f;
        return;
    }
    float acc = 0.0f;
    for (int base = 0; base < a.nb; base += 32) {
        int b = base + lane;
        float v = b < a.nb ? block_dot_f32(a, row, b) : 0.0f;
        int n = min(32, a.nb - base);
        for (int k = 0; k < n; k++) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, v, k));
    }
    if (lane == 0) a.out[row] = acc;
}

static int vec_dot_f32_call(const char *fn, int quant, float *out, size_t out_len,
                            const jkb_weight *w, const float *input, size_t in_len,
                            void *stream) {
    int rc = validate_weight_call(fn, w, quant, out_len, in_len);
    if (rc) return rc;
    if (!out || !input) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    if ((rc = check_align(out, 4, fn, "output")) || (rc = check_align(input, 4, fn, "input")) ||
        (rc = push_reject(out, out + out_len, fn)))
        return rc;
    DqArgs a;
    a.qs = w->p.qs;
    a.qs_row = w->p.qs_row;
    a.sc = w->p.sc;
    a.sc_row = w->p.sc_row;
    a.d = w->p.d;
    a.i2s = w->p.i2s_scale;
    a.quant = quant;
    a.gpu_format = w->gpu_format;
    a.nb = (int)w->nb;
    a.be = fmt_of(quant)->block_elems;
    a.x = input;
    a.out = out;
    a.rows = w->rows;
    vec_dot_f32_kernel<<<(unsigned)((w->rows + 7) / 8), 256, 0, as_stream(stream)>>>(a);
    return check_launch(fn);
}

// ---------------------------------------------------------------- BitLinear glue

// validate_bitlinear_dimensions (ime.rs:660-763)
int validate_bitlinear(const jkb_weight *w, size_t output_len, size_t input_len) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->quant != JKB_TQ1_0 && w->quant != JKB_TQ2_0 && w->quant != JKB_Q8_0 &&
        w->quant != JKB_I2_S)
        return fail(JKB_E_BOUNDS, w->name, w->offset, w->byte_len, w->gguf_bytes,
                    "unsupported quantization format for BitLinear: %s; expected TQ1_0, TQ2_0, "
                    "Q8_0, or I2_S",
                    quant_name(w->quant));
    size_t r = 0, c = 0;
    rc = validate_matvec_shape(w->name, w->offset, w->byte_len, w->gguf_bytes, w->quant, w->shape,
                               w->ndim, output_len, input_len, &r, &c);
    if (rc) return rc;
    if (r != w->rows || c != w->cols)
        return fail(JKB_E_BOUNDS, w->name, w->offset, w->byte_len, w->gguf_bytes,
                    "bitlinear: call interprets the tensor as [%zu, %zu] but it was uploaded as "
                    "[%zu, %zu]",
                    r, c, w->rows, w->cols);
    return JKB_OK;
}

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_vec_dot_q4_0_q8_0(const uint8_t *w, size_t w_len, const jkb_block_q8_0 *x, size_t x_len,
                          float *result, void *stream) {
    return vec_dot_raw("vec_dot_q4_0_q8_0", JKB_Q4_0, w, w_len, x, x_len, result, stream);
}
int jkb_vec_dot_q8_0_q8_0(const uint8_t *w, size_t w_len, const jkb_block_q8_0 *x, size_t x_len,
                          float *result, void *stream) {
    return vec_dot_raw("vec_dot_q8_0_q8_0", JKB_Q8_0, w, w_len, x, x_len, result, stream);
}
int jkb_vec_dot_q4_k_q8_k(const uint8_t *w, size_t w_len, const jkb_block_q8_k *x, size_t x_len,
                          float *result, void *stream) {
    return vec_dot_raw("vec_dot_q4_k_q8_k", JKB_Q4_K_M, w, w_len, x, x_len, result, stream);
}
int jkb_vec_dot_q6_k_q8_k(const uint8_t *w, size_t w_len, const jkb_block_q8_k *x, size_t x_len,
                          float *result, void *stream) {
    return vec_dot_raw("vec_dot_q6_k_q8_k", JKB_Q6_K, w, w_len, x, x_len, result, stream);
}
int jkb_vec_dot_q5_0_q8_0_blocks(const uint8_t *w, size_t w_len, const jkb_block_q8_0 *x,
                                 size_t x_len, float *result, void *stream) {
    return vec_dot_raw("vec_dot_q5_0_q8_0_blocks", JKB_Q5_0, w, w_len, x, x_len, result, stream);
}
int jkb_vec_dot_q5_k_q8_k(const uint8_t *w, size_t w_len, const jkb_block_q8_k *x, size_t x_len,
                          float *result, void *stream) {
    return vec_dot_raw("vec_dot_q5_k_q8_k", JKB_Q5_K, w, w_len, x, x_len, result, stream);
}
int jkb_vec_dot_tq1_0_q8_k(const uint8_t *w, size_t w_len, const jkb_block_q8_k *x,
                           size_t x_len, float *result, void *stream) {
    return vec_dot_raw("vec_dot_tq1_0_q8_k", JKB_TQ1_0, w, w_len, x, x_len, result, stream);
}
int jkb_vec_dot_tq2_0_q8_k(const uint8_t *w, size_t w_len, const jkb_block_q8_k *x,
                           size_t x_len, float *result, void *stream) {
    return vec_dot_raw("vec_dot_tq2_0_q8_k", JKB_TQ2_0, w, w_len, x, x_len, result, stream);
}

int jkb_vec_dot_q4_k_m(float *out, size_t out_len, const jkb_weight *w, const float *input,
                       size_t in_len, void *stream) {
    return vec_dot_f32_call("vec_dot_q4_k_m", JKB_Q4_K_M, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q8_0(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream) {
    return vec_dot_f32_call("vec_dot_q8_0", JKB_Q8_0, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q6_k(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream) {
    return vec_dot_f32_call("vec_dot_q6_k", JKB_Q6_K, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q4_0(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream) {
    return vec_dot_f32_call("vec_dot_q4_0", JKB_Q4_0, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q5_0(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream) {
    return vec_dot_f32_call("vec_dot_q5_0", JKB_Q5_0, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q5_k(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream) {
    return vec_dot_f32_call("vec_dot_q5_k", JKB_Q5_K, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_i2_s(float *out, size_t out_len, const jkb_weight *w, const float *input,
                     size_t in_len, void *stream) {
    return vec_dot_f32_call("vec_dot_i2_s", JKB_I2_S, out, out_len, w, input, in_len, stream);
}

int jkb_bitlinear_i8(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                     size_t act_len, float act_scale, void *stream) {
    int rc = validate_bitlinear(w, out_len, act_len);
    if (rc) return rc;
    if (!out || !act_i8) return fail(JKB_E_INVALID, "bitlinear_i8", 0, 0, 0, "null pointer");
    if ((rc = check_align(out, 4, "bitlinear_i8", "output"))) return rc;
    GemvLaunch L{};
    L.w = w;
    L.x = act_i8;
    L.act_kind = ACT_I8;
    L.act_scale = act_scale;
    L.out = out;
    L.row_begin = 0;
    L.row_end = w->rows;
    L.m = 1;
    return launch_gemv(L, as_stream(stream));
}

int jkb_bitlinear_i8_rvv(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                         size_t act_len, float act_scale, void *stream) {
    return jkb_bitlinear_i8(out, out_len, w, act_i8, act_len, act_scale, stream);
}

int jkb_bitlinear_i8_ime(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                         size_t act_len, float act_scale, void *stream) {
    return jkb_bitlinear_i8(out, out_len, w, act_i8, act_len, act_scale, stream);
}

int jkb_bitlinear_i8_batch(float *out, size_t out_len, const jkb_weight *w, const int8_t *act_i8,
                           size_t act_len, const float *act_scales, size_t m, void *stream) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (m == 0 || act_len != m * w->cols || out_len != m * w->rows)
        return fail(JKB_E_BOUNDS, w->name, w->offset, act_len, m * w->cols,
                    "bitlinear batch: act len %zu / out len %zu do not match m=%zu x [%zu, %zu]",
                    act_len, out_len, m, w->rows, w->cols);
    rc = validate_bitlinear(w, w->rows, w->cols);
    if (rc) return rc;
    if (!out || !act_i8 || !act_scales)
        return fail(JKB_E_INVALID, "bitlinear_i8_batch", 0, 0, 0, "null pointer");
    if ((rc = check_align(out, 4, "bitlinear_i8_batch", "output")) ||
        (rc = check_align(act_scales, 4, "bitlinear_i8_batch", "act_scales")))
        return rc;
    GemvLaunch L{};
    L.w = w;
    L.x = act_i8;
    L.x_row_stride = w->cols;
    L.act_kind = ACT_I8;
    L.act_scales = act_scales;
    L.out = out;
    L.out_ld = w->rows;
    L.row_begin = 0;
    L.row_end = w->rows;
    L.m = m;
    return launch_gemv(L, as_stream(stream));
}

}  // extern "C"
