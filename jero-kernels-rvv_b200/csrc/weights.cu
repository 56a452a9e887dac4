// Load-time weight handles: validation (repack.rs:1208-1284), upload and relayout into the
// GPU layouts used by the GEMV / BitLinear kernels (jkb_weight) and by the GEMM
// (jkb_repacked_weight, the i8-expanded RepackedWeight of repack.rs:1092-1133).
//
// jkb_weight planes (every row contiguous, rows back to back, block order kept; the quant
// plane's 16-byte chunks are lane-interleaved in groups of 32 blocks, see gpu_layout.cuh):
//   Q4_0   qs: 16 B/block, the GGUF nibble bytes        d: f16 per block
//   Q8_0   qs: 32 B/block, the GGUF i8 quants           d: f16 per block
//   Q4_K_M qs: 128 B/block, GGUF qs bytes               sc: 16 B/block = d, dmin, scales[12]
//   Q5_0   qs: 16 B/block, the GGUF nibble bytes        sc: 4 B/block = qh   d: f16 per block
//   Q5_K   qs: 160 B/block, GGUF qs[128] then qh[32]    sc: 16 B/block = d, dmin, scales[12]
//   Q6_K   qs: 192 B/block, GGUF ql[128] then qh[64]    sc: 16 B/block i8 scales, d: f16
//   TQ2_0  qs: 64 B/block, 2-bit codes re-ordered so that chunk p, word W, bit pair j, byte b
//          holds element 64p+16W+4j+b                   d: f16 per block
//   TQ1_0  decoded at load into the TQ2_0 GPU layout (same codes 0..2)
//   I2_S   qs: 32 B/block, GGUF bytes unchanged; the trailer scale is kept on the host
// Byte counts equal the GGUF payload (except TQ1_0, whose base-3 bytes grow from 54 to 66).
#include <cstdio>
#include <cstring>
#include <vector>

#include "gpu_layout.cuh"
#include "jkb_internal.h"

namespace jkb {

__device__ __forceinline__ uint16_t rd16(const uint8_t *p) {
    return (uint16_t)(p[0] | (p[1] << 8));
}

// One thread per (row, block): scale planes are written [row][block], quant bytes go to the
// lane-interleaved chunk positions of gpu_layout.cuh. `payload` holds the block's quant bytes
// in GPU chunk order (chunk j = payload[16j .. 16j+16]).
__global__ void relayout_kernel(int quant, int gpu_format, const uint8_t *__restrict__ raw,
                                size_t rows, size_t nb, size_t raw_row, int bb,
                                uint8_t *__restrict__ qs, size_t qs_row, uint8_t *__restrict__ sc,
                                size_t sc_row, uint16_t *__restrict__ d) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * nb) return;
    size_t r = idx / nb, b = idx % nb;
    const uint8_t *blk = raw + r * raw_row + b * (size_t)bb;
    uint8_t payload[192];
    switch (quant) {
    case JKB_Q4_0:  // 16 nibble bytes, GGUF order
        d[idx] = rd16(blk);
        for (int i = 0; i < 16; i++) payload[i] = blk[2 + i];
        break;
    case JKB_Q8_0:  // 32 i8 quants
        d[idx] = rd16(blk);
        for (int i = 0; i < 32; i++) payload[i] = blk[2 + i];
        break;
    case JKB_Q4_K_M: {  // d, dmin, scales[12] to the scale plane; qs[128] in GGUF order
        uint8_t *s = sc + r * sc_row + 16 * b;
        for (int i = 0; i < 16; i++) s[i] = blk[i];
        for (int i = 0; i < 128; i++) payload[i] = blk[16 + i];
        break;
    }
    case JKB_Q5_0: {  // 16 nibble bytes, GGUF order; qh to the scale plane, d to its plane
        uint8_t *s = sc + r * sc_row + 4 * b;
        for (int i = 0; i < 4; i++) s[i] = blk[2 + i];
        d[idx] = rd16(blk);
        for (int i = 0; i < 16; i++) payload[i] = blk[6 + i];
        break;
    }
    case JKB_Q5_K: {  // d, dmin, scales[12] to the scale plane; qs[128] then qh[32]
        uint8_t *s = sc + r * sc_row + 16 * b;
        for (int i = 0; i < 16; i++) s[i] = blk[i];
        for (int i = 0; i < 128; i++) payload[i] = blk[48 + i];
        for (int i = 0; i < 32; i++) payload[128 + i] = blk[16 + i];
        break;
    }
    case JKB_Q6_K: {  // ql[128] qh[64] in GGUF order; i8 scales and d to their planes
        uint8_t *s = sc + r * sc_row + 16 * b;
        for (int i = 0; i < 16; i++) s[i] = blk[192 + i];
        d[idx] = rd16(blk + 208);
        for (int i = 0; i < 192; i++) payload[i] = blk[i];
        break;
    }
    case JKB_TQ2_0:
    case JKB_TQ1_0: {
        // 2-bit codes (value + 1) re-ordered so that chunk p, word W, bit pair j, byte q holds
        // element 64p + 16W + 4j + q: (word >> 2j) & 0x03030303 then lines up with four
        // consecutive activations.
        d[idx] = rd16(blk);
        uint8_t codes[256];
        if (quant == JKB_TQ2_0) {
            for (int e = 0; e < 256; e++) codes[e] = (blk[2 + e / 4] >> (2 * (e % 4))) & 3;
        } else {
            for (int i = 0; i < 51; i++) {
                unsigned v = blk[2 + i];
                for (int j = 0; j < 5; j++) {
                    codes[5 * i + j] = (uint8_t)(v % 3);
                    v /= 3;
                }
            }
            codes[255] = (uint8_t)(blk[53] % 3);
        }
        for (int i = 0; i < 64; i++) payload[i] = 0;
        for (int e = 0; e < 256; e++) {
            int p = e >> 6, W = (e & 63) >> 4, j = (e & 15) >> 2, bq = e & 3;
            payload[16 * p + 4 * W + bq] |= (uint8_t)(codes[e] << (2 * j));
        }
        break;
    }
    case JKB_I2_S:  // 32 bytes, GGUF order (byte g carries elements g, 32+g, 64+g, 96+g)
        for (int i = 0; i < 32; i++) payload[i] = blk[i];
        break;
    default: return;
    }
    const int qch = qs_chunks(gpu_format);
    uint8_t *row = qs + r * qs_row;
    for (int j = 0; j < qch; j++) {
        uint8_t *o = row + qs_chunk_offset((int)nb, qch, (int)b, j);
        for (int i = 0; i < 16; i++) o[i] = payload[16 * j + i];
    }
}

__device__ __forceinline__ float f16_finite_dev(uint16_t bits) {
    float v = __half2float(__ushort_as_half(bits));
    return ((bits >> 10) & 0x1F) == 0x1F ? 0.0f : v;
}

// repack_block_scaled_range_into_i8 (repack.rs:1724-2103) for the covered formats, one thread
// per (row, block): i8 values row-major [rows][k_pad], f32 scales [rows][groups].
__global__ void repack_i8_kernel(int quant, const uint8_t *__restrict__ raw, size_t rows,
                                 size_t nb, size_t raw_row, int bb, float i2s, int8_t *q,
                                 size_t k_pad, float *scales, float *mins, size_t groups) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * nb) return;
    size_t r = idx / nb, b = idx % nb;
    const uint8_t *blk = raw + r * raw_row + b * (size_t)bb;
    int8_t *qr = q + r * k_pad;
    float *sr = scales + r * groups;
    float *mr = mins ? mins + r * groups : nullptr;
    switch (quant) {
    case JKB_Q8_0: {
        float dd = f16_finite_dev(rd16(blk));
        sr[b] = dd;
        for (int i = 0; i < 32; i++) qr[32 * b + i] = dd != 0.0f ? (int8_t)blk[2 + i] : 0;
        break;
    }
    case JKB_Q4_0: {
        float dd = f16_finite_dev(rd16(blk));
        sr[b] = dd;
        for (int i = 0; i < 16; i++) {
            qr[32 * b + i] = dd != 0.0f ? (int8_t)((blk[2 + i] & 0x0F) - 8) : 0;
            qr[32 * b + 16 + i] = dd != 0.0f ? (int8_t)(((blk[2 + i] >> 4) & 0x0F) - 8) : 0;
        }
        break;
    }
    case JKB_Q4_K_M: {
        float dd = f16_finite_dev(rd16(blk)), dmin = f16_finite_dev(rd16(blk + 2));
        const uint8_t *s = blk + 4;
        uint8_t scv[8], mv[8];
        for (int j = 0; j < 4; j++) {
            scv[j] = s[j] & 0x3F;
            mv[j] = s[j + 4] & 0x3F;
        }
        for (int j = 4; j < 8; j++) {
            scv[j] = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
            mv[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
        }
        for (int c = 0; c < 4; c++) {
            size_t g0 = b * 8 + 2 * c;
            sr[g0] = __fmul_rn(dd, (float)scv[2 * c]);
            mr[g0] = __fmul_rn(dmin, (float)mv[2 * c]);
            sr[g0 + 1] = __fmul_rn(dd, (float)scv[2 * c + 1]);
            mr[g0 + 1] = __fmul_rn(dmin, (float)mv[2 * c + 1]);
            for (int l = 0; l < 32; l++) {
                qr[256 * b + 64 * c + l] = (int8_t)(blk[16 + 32 * c + l] & 0x0F);
                qr[256 * b + 64 * c + 32 + l] = (int8_t)((blk[16 + 32 * c + l] >> 4) & 0x0F);
            }
        }
        break;
    }
    case JKB_Q5_0: {  // repack.rs:1827-1840: (5-bit code - 16), left 0 when d == 0
        float dd = f16_finite_dev(rd16(blk));
        sr[b] = dd;
        const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) |
                            ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
        for (int i = 0; i < 16; i++) {
            const int q0 = (int)((blk[6 + i] & 0x0F) | (((qh >> i) & 1) << 4)) - 16;
            const int q1 = (int)(((blk[6 + i] >> 4) & 0x0F) | (((qh >> (i + 16)) & 1) << 4)) - 16;
            qr[32 * b + i] = dd != 0.0f ? (int8_t)q0 : 0;
            qr[32 * b + 16 + i] = dd != 0.0f ? (int8_t)q1 : 0;
        }
        break;
    }
    case JKB_Q5_K: {  // repack.rs:1959-1995: scales d * sc, mins dmin * m, unsigned 5-bit codes
        float dd = f16_finite_dev(rd16(blk)), dmin = f16_finite_dev(rd16(blk + 2));
        const uint8_t *s = blk + 4, *qh = blk + 16, *qs = blk + 48;
        uint8_t scv[8], mv[8];
        for (int j = 0; j < 4; j++) {
            scv[j] = s[j] & 0x3F;
            mv[j] = s[j + 4] & 0x3F;
        }
        for (int j = 4; j < 8; j++) {
            scv[j] = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
            mv[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
        }
        for (int c = 0; c < 4; c++) {
            size_t g0 = b * 8 + 2 * c;
            sr[g0] = __fmul_rn(dd, (float)scv[2 * c]);
            mr[g0] = __fmul_rn(dmin, (float)mv[2 * c]);
            sr[g0 + 1] = __fmul_rn(dd, (float)scv[2 * c + 1]);
            mr[g0 + 1] = __fmul_rn(dmin, (float)mv[2 * c + 1]);
            for (int l = 0; l < 32; l++) {
                qr[256 * b + 64 * c + l] =
                    (int8_t)((qs[32 * c + l] & 0x0F) + (((qh[l] >> (2 * c)) & 1) ? 16 : 0));
                qr[256 * b + 64 * c + 32 + l] =
                    (int8_t)((qs[32 * c + l] >> 4) + (((qh[l] >> (2 * c + 1)) & 1) ? 16 : 0));
            }
        }
        break;
    }
    case JKB_Q6_K: {
        float dd = f16_finite_dev(rd16(blk + 208));
        for (int s = 0; s < 16; s++) sr[b * 16 + s] = __fmul_rn(dd, (float)(int8_t)blk[192 + s]);
        const uint8_t *ql = blk, *qh = blk + 128;
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 32; l++) {
                int lb = 64 * h, hb = 32 * h, n = 256 * (int)b + 128 * h;
                int q1 = (int)((ql[lb + l] & 0x0F) | ((qh[hb + l] & 3) << 4)) - 32;
                int q2 = (int)((ql[lb + l + 32] & 0x0F) | (((qh[hb + l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)(((ql[lb + l] >> 4) & 0x0F) | (((qh[hb + l] >> 4) & 3) << 4)) - 32;
                int q4 = (int)(((ql[lb + l + 32] >> 4) & 0x0F) | (((qh[hb + l] >> 6) & 3) << 4)) - 32;
                bool z = dd == 0.0f;
                qr[n + l] = z ? 0 : (int8_t)q1;
                qr[n + l + 32] = z ? 0 : (int8_t)q2;
                qr[n + l + 64] = z ? 0 : (int8_t)q3;
                qr[n + l + 96] = z ? 0 : (int8_t)q4;
            }
        break;
    }
    case JKB_TQ2_0:
    case JKB_TQ1_0: {
        float dd = f16_finite_dev(rd16(blk));
        for (int s = 0; s < 8; s++) sr[b * 8 + s] = dd;
        if (quant == JKB_TQ2_0) {
            for (int e = 0; e < 256; e++)
                qr[256 * b + e] = (int8_t)(((blk[2 + e / 4] >> (2 * (e % 4))) & 3) - 1);
        } else {
            for (int i = 0; i < 51; i++) {
                unsigned v = blk[2 + i];
                for (int j = 0; j < 5; j++) {
                    qr[256 * b + 5 * i + j] = (int8_t)((int)(v % 3) - 1);
                    v /= 3;
                }
            }
            qr[256 * b + 255] = (int8_t)((int)(blk[53] % 3) - 1);
        }
        break;
    }
    case JKB_Q4_1: {  // repack.rs:1814-1826: scale d, min -m (0.0 when m == 0), unsigned codes
        const float dd = f16_finite_dev(rd16(blk)), m = f16_finite_dev(rd16(blk + 2));
        sr[b] = dd;
        mr[b] = m == 0.0f ? 0.0f : -m;
        for (int i = 0; i < 16; i++) {
            qr[32 * b + i] = (int8_t)(blk[4 + i] & 0x0F);
            qr[32 * b + 16 + i] = (int8_t)(blk[4 + i] >> 4);
        }
        break;
    }
    case JKB_Q5_1: {  // repack.rs:1841-1855 with unpack_q5_1_block_i8 (quant.rs:169-190)
        const float dd = f16_finite_dev(rd16(blk)), m = f16_finite_dev(rd16(blk + 2));
        sr[b] = dd;
        mr[b] = m == 0.0f ? 0.0f : -m;
        const uint32_t qh = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) |
                            ((uint32_t)blk[6] << 16) | ((uint32_t)blk[7] << 24);
        for (int i = 0; i < 16; i++) {
            qr[32 * b + i] = (int8_t)((blk[8 + i] & 0x0F) | (((qh >> i) & 1) << 4));
            qr[32 * b + 16 + i] = (int8_t)((blk[8 + i] >> 4) | (((qh >> (i + 16)) & 1) << 4));
        }
        break;
    }
    case JKB_IQ4_NL: {  // repack.rs:1856-1873: the code book values, left 0 when d == 0
        // KVALUES_IQ4NL (quant.rs:80-82)
        constexpr int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                   1,    13,   25,  38,  53,  69,  89,  113};
        const float dd = f16_finite_dev(rd16(blk));
        sr[b] = dd;
        for (int i = 0; i < 16; i++) {
            qr[32 * b + i] = dd != 0.0f ? kv[blk[2 + i] & 0x0F] : 0;
            qr[32 * b + 16 + i] = dd != 0.0f ? kv[blk[2 + i] >> 4] : 0;
        }
        break;
    }
    case JKB_Q2_K: {  // repack.rs:1874-1892 with unpack_q2_k_block_i8 (quant.rs:198-246)
        // sub-block s (16 elements) takes the 2-bit field 2 * ((s % 8) / 2) of
        // qs[32 (s / 8) + 16 (s % 2) + l]; scale d * (sc & 15), min dmin * (sc >> 4)
        const float dd = f16_finite_dev(rd16(blk + 80)), dmin = f16_finite_dev(rd16(blk + 82));
        for (int s = 0; s < 16; s++) {
            sr[16 * b + s] = __fmul_rn(dd, (float)(blk[s] & 0x0F));
            mr[16 * b + s] = __fmul_rn(dmin, (float)(blk[s] >> 4));
            const int sh = 2 * ((s % 8) / 2);
            const uint8_t *qs = blk + 16 + 32 * (s / 8) + 16 * (s % 2);
            for (int l = 0; l < 16; l++) qr[256 * b + 16 * s + l] = (int8_t)((qs[l] >> sh) & 3);
        }
        break;
    }
    case JKB_Q3_K: {  // repack.rs:1893-1908 with unpack_q3_k_block_i8 (quant.rs:255-330)
        // 6-bit scale s: low 4 bits from byte s (s < 8, low nibble) or s - 8 (high nibble),
        // top 2 bits from byte 8 + s % 4 at bit 2 (s / 4); codes minus 4 where the hmask bit
        // s / 2 of hmask[16 (s % 2) + l] is clear
        const uint8_t *hm = blk, *raw6 = blk + 96;
        const float dd = f16_finite_dev(rd16(blk + 108));
        for (int s = 0; s < 16; s++) {
            const int lo = s < 8 ? raw6[s] & 0x0F : raw6[s - 8] >> 4;
            const int hi = (raw6[8 + s % 4] >> (2 * (s / 4))) & 3;
            sr[16 * b + s] = __fmul_rn(dd, (float)((lo | (hi << 4)) - 32));
            const int sh = 2 * ((s % 8) / 2);
            const uint8_t *qs = blk + 32 + 32 * (s / 8) + 16 * (s % 2);
            for (int l = 0; l < 16; l++) {
                const int code = (qs[l] >> sh) & 3;
                const int high = (hm[16 * (s % 2) + l] >> (s / 2)) & 1;
                qr[256 * b + 16 * s + l] = (int8_t)(code - (high ? 0 : 4));
            }
        }
        break;
    }
    case JKB_I2_S: {
        for (int s = 0; s < 4; s++) sr[b * 4 + s] = i2s;
        for (int g = 0; g < 32; g++) {
            uint8_t v = blk[g];
            bool z = i2s == 0.0f;
            qr[128 * b + g] = z ? 0 : (int8_t)(((v >> 6) & 3) - 1);
            qr[128 * b + 32 + g] = z ? 0 : (int8_t)(((v >> 4) & 3) - 1);
            qr[128 * b + 64 + g] = z ? 0 : (int8_t)(((v >> 2) & 3) - 1);
            qr[128 * b + 96 + g] = z ? 0 : (int8_t)((v & 3) - 1);
        }
        break;
    }
    default: break;
    }
}

// validate_matrix_shape + validate_matrix_view (repack.rs:1151-1284).
int validate_matrix_view(const jkb_tensor_view *v, const Fmt *f, size_t rows,
                                size_t cols) {
    const char *nm = v->name ? v->name : "";
    if (rows == 0 || cols == 0)
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "repack dimensions must be non-zero, got [%zu, %zu]", rows, cols);
    if (cols % (size_t)f->block_elems != 0)
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "columns (%zu) must be a multiple of %s block size (%d)", cols, f->name,
                    f->block_elems);
    if (v->ndim == 1) {
        if (rows * cols != v->shape[0])
            return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                        "1D tensor length %zu does not match rows (%zu) * cols (%zu)",
                        v->shape[0], rows, cols);
    } else if (v->ndim == 2) {
        size_t d0 = v->shape[0], d1 = v->shape[1];
        if (!((d0 == rows && d1 == cols) || (d0 == cols && d1 == rows)))
            return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                        "tensor shape [%zu, %zu] does not match requested rows=%zu, cols=%zu",
                        d0, d1, rows, cols);
    } else {
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "expected 1D or 2D weight tensor, got %uD", v->ndim);
    }
    size_t need = storage_bytes(f, rows * cols);
    if (v->byte_len < need)
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "backing bytes %zu < required %zu", v->byte_len, need);
    return JKB_OK;
}

// RepackedWeight::repack orientation rule (repack.rs:2255-2282; PackedNibbleMatrix::repack
// :4654-4679 is the same rule). `who` names the caller in the error.
int infer_rows_cols(const jkb_tensor_view *v, const Fmt *f, size_t *rows, size_t *cols,
                    const char *who) {
    if (v->ndim != 2)
        return fail(JKB_E_BOUNDS, v->name ? v->name : "", v->offset, v->byte_len, v->byte_len,
                    "%s requires a 2D tensor, got %uD", who, v->ndim);
    size_t d0 = v->shape[0], d1 = v->shape[1], be = (size_t)f->block_elems;
    if (d0 % be == 0 && d1 % be != 0) {
        *rows = d1;
        *cols = d0;
    } else if (d1 % be == 0 && d0 % be != 0) {
        *rows = d0;
        *cols = d1;
    } else {
        *rows = d1;
        *cols = d0;
    }
    return JKB_OK;
}

// Stages the raw GGUF bytes on the device (a load-time temporary) and reads the I2_S trailer.
int stage_raw(const jkb_tensor_view *v, size_t need, cudaStream_t st, uint8_t **dev,
              bool *owned) {
    if (v->data_on_device) {
        *dev = (uint8_t *)v->data;
        *owned = false;
        return JKB_OK;
    }
    cudaError_t e = cudaMalloc(dev, need);
    if (e != cudaSuccess) return fail_cuda(e, "weight upload (staging)");
    *owned = true;
    e = cudaMemcpyAsync(*dev, v->data, need, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
        cudaFree(*dev);
        return fail_cuda(e, "weight upload (copy)");
    }
    return JKB_OK;
}

static float read_i2s_trailer(const jkb_tensor_view *v, size_t payload) {
    float s = 0.0f;
    if (v->data_on_device)
        cudaMemcpy(&s, (const uint8_t *)v->data + payload, 4, cudaMemcpyDeviceToHost);
    else
        memcpy(&s, (const uint8_t *)v->data + payload, 4);
    // read_i2_s_trailer_scale (quant.rs:360-366): non-finite -> 0.0
    uint32_t u;
    memcpy(&u, &s, 4);
    return ((u >> 23) & 0xFF) == 0xFF ? 0.0f : s;
}

static int weight_upload(const jkb_tensor_view *v, size_t rows, size_t cols, cudaStream_t st,
                         jkb_weight **out) {
    if (!v || !out) return fail(JKB_E_INVALID, "jkb_weight_upload", 0, 0, 0, "null argument");
    *out = nullptr;
    const Fmt *f = fmt_of(v->quant);
    const char *nm = v->name ? v->name : "";
    // Q4_1, Q5_1, IQ4_NL, Q2_K and Q3_K have no block dot against Q8 activations in the
    // reference (quant_q8.rs): they exist only as RepackedWeights and nibble matrices
    const bool gemv_fmt = f && v->quant != JKB_Q4_1 && v->quant != JKB_Q5_1 &&
                          v->quant != JKB_IQ4_NL && v->quant != JKB_Q2_K && v->quant != JKB_Q3_K;
    if (!gemv_fmt)
        return fail(JKB_E_CAPABILITY, nm, v->offset, v->byte_len, v->byte_len,
                    "unsupported tensor quant %s for the GEMV layout", quant_name(v->quant));
    if (!v->data) return fail(JKB_E_INVALID, nm, v->offset, 0, 0, "null tensor data");
    int rc = validate_matrix_view(v, f, rows, cols);
    if (rc) return rc;

    jkb_weight *w = new jkb_weight();
    memset(w, 0, sizeof(*w));
    w->magic = WEIGHT_MAGIC;
    w->quant = v->quant;
    w->rows = rows;
    w->cols = cols;
    w->nb = cols / (size_t)f->block_elems;
    w->ndim = v->ndim;
    for (uint32_t i = 0; i < v->ndim && i < 4; i++) w->shape[i] = v->shape[i];
    snprintf(w->name, sizeof(w->name), "%s", nm);
    w->offset = v->offset;
    w->byte_len = v->byte_len;
    w->gguf_bytes = storage_bytes(f, rows * cols);

    size_t qp = 0, scp = 0;
    bool has_d = false;
    switch (v->quant) {
    case JKB_Q4_0: qp = 16; has_d = true; w->gpu_format = GF_Q4_0; break;
    case JKB_Q8_0: qp = 32; has_d = true; w->gpu_format = GF_Q8_0; break;
    case JKB_Q4_K_M: qp = 128; scp = 16; w->gpu_format = GF_Q4_K; break;
    case JKB_Q6_K: qp = 192; scp = 16; has_d = true; w->gpu_format = GF_Q6_K; break;
    case JKB_Q5_0: qp = 16; scp = 4; has_d = true; w->gpu_format = GF_Q5_0; break;
    case JKB_Q5_K: qp = 160; scp = 16; w->gpu_format = GF_Q5_K; break;
    case JKB_TQ1_0:
    case JKB_TQ2_0: qp = 64; has_d = true; w->gpu_format = GF_TQ2_0; break;
    case JKB_I2_S: qp = 32; w->gpu_format = GF_I2_S; break;
    }
    Arena a;
    size_t qs_bytes = rows * w->nb * qp, sc_bytes = rows * w->nb * scp,
           d_bytes = has_d ? rows * w->nb * 2 : 0;
    a.cap = Arena::round(qs_bytes) + Arena::round(sc_bytes) + Arena::round(d_bytes);
    cudaError_t e = cudaMalloc(&a.base, a.cap);
    if (e != cudaSuccess) {
        delete w;
        return fail_cuda(e, "jkb_weight_upload (device planes)");
    }
    w->base = a.base;
    w->device_bytes = a.cap;
    uint8_t *qs = a.take(qs_bytes);
    uint8_t *sc = scp ? a.take(sc_bytes) : nullptr;
    uint16_t *d = has_d ? (uint16_t *)a.take(d_bytes) : nullptr;
    w->p.qs = qs;
    w->p.qs_row = w->nb * qp;
    w->p.sc = sc;
    w->p.sc_row = w->nb * scp;
    w->p.d = d;
    size_t payload = rows * w->nb * (size_t)f->block_bytes;
    if (v->quant == JKB_I2_S) w->p.i2s_scale = read_i2s_trailer(v, payload);

    uint8_t *raw = nullptr;
    bool owned = false;
    rc = stage_raw(v, payload, st, &raw, &owned);
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    size_t n = rows * w->nb;
    relayout_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        v->quant, w->gpu_format, raw, rows, w->nb, w->nb * (size_t)f->block_bytes,
        f->block_bytes, qs, w->p.qs_row, sc, w->p.sc_row, d);
    rc = check_launch("relayout_kernel");
    if (owned) {
        cudaStreamSynchronize(st);
        cudaFree(raw);
    }
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    *out = w;
    return JKB_OK;
}

// RepackedWeight::dequantize_row (repack.rs:2529-2598), BlockScaledI8 storage: per element
// scale * q - min of its group, two roundings.
__global__ void repacked_dequant_row_kernel(const int8_t *__restrict__ q,
                                            const float *__restrict__ scales,
                                            const float *__restrict__ mins, size_t cols,
                                            int group_elems, float *__restrict__ out) {
    const size_t c = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const size_t g = c / (size_t)group_elems;
    const float wm = mins ? mins[g] : 0.0f;
    out[c] = __fsub_rn(__fmul_rn(scales[g], (float)q[c]), wm);
}

static int repacked_upload(const jkb_tensor_view *v, size_t rows, size_t cols, cudaStream_t st,
                           jkb_repacked_weight **out) {
    if (!v || !out)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null argument");
    *out = nullptr;
    const char *nm = v->name ? v->name : "";
    const Fmt *f = fmt_of(v->quant);
    if (!f)
        // Dense F32/F16/BF16 storage (RepackedStorage::DenseF32/DenseHalf) and the formats
        // outside the hot path are not built on the GPU.
        return fail(JKB_E_CAPABILITY, nm, v->offset, v->byte_len, v->byte_len,
                    "unsupported tensor quant %s for repack", quant_name(v->quant));
    if (!v->data) return fail(JKB_E_INVALID, nm, v->offset, 0, 0, "null tensor data");
    int rc = validate_matrix_view(v, f, rows, cols);
    if (rc) return rc;
    jkb_repacked_weight *w = new jkb_repacked_weight();
    memset(w, 0, sizeof(*w));
    w->magic = REPACKED_MAGIC;
    w->quant = v->quant;
    w->rows = rows;
    w->cols = cols;
    w->k_pad = (cols + 31) / 32 * 32;
    // BlockScaledTileLayout::from_validated_dims (repack.rs:1338-1366)
    w->group_elems =
        (v->quant == JKB_Q6_K || v->quant == JKB_Q3_K || v->quant == JKB_Q2_K) ? 16 : 32;
    w->scale_groups = w->k_pad / w->group_elems;
    snprintf(w->name, sizeof(w->name), "%s", nm);
    bool mins = v->quant == JKB_Q4_K_M || v->quant == JKB_Q5_K || v->quant == JKB_Q4_1 ||
                v->quant == JKB_Q5_1 || v->quant == JKB_Q2_K;
    Arena a;
    size_t qb = rows * w->k_pad, sb = rows * w->scale_groups * 4;
    a.cap = Arena::round(qb) + Arena::round(sb) * (mins ? 2 : 1);
    cudaError_t e = cudaMalloc(&a.base, a.cap);
    if (e != cudaSuccess) {
        delete w;
        return fail_cuda(e, "jkb_repacked_weight (device buffers)");
    }
    w->base = a.base;
    w->device_bytes = a.cap;
    w->q = (int8_t *)a.take(qb);
    w->scales = (float *)a.take(sb);
    w->mins = mins ? (float *)a.take(sb) : nullptr;
    size_t nb = cols / (size_t)f->block_elems;
    size_t payload = rows * nb * (size_t)f->block_bytes;
    float i2s = v->quant == JKB_I2_S ? read_i2s_trailer(v, payload) : 0.0f;
    uint8_t *raw = nullptr;
    bool owned = false;
    rc = stage_raw(v, payload, st, &raw, &owned);
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    cudaMemsetAsync(w->q, 0, qb, st);
    size_t n = rows * nb;
    repack_i8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        v->quant, raw, rows, nb, nb * (size_t)f->block_bytes, f->block_bytes, i2s, w->q,
        w->k_pad, w->scales, w->mins, w->scale_groups);
    rc = check_launch("repack_i8_kernel");
    if (owned) {
        cudaStreamSynchronize(st);
        cudaFree(raw);
    }
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    *out = w;
    return JKB_OK;
}

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_weight_upload(const jkb_tensor_view *view, size_t rows, size_t cols, void *stream,
                      jkb_weight **out) {
    return weight_upload(view, rows, cols, as_stream(stream), out);
}

int jkb_weight_upload_infer(const jkb_tensor_view *view, void *stream, jkb_weight **out) {
    if (!view || !out) return fail(JKB_E_INVALID, "jkb_weight_upload_infer", 0, 0, 0, "null");
    const Fmt *f = fmt_of(view->quant);
    if (!f)
        return fail(JKB_E_CAPABILITY, view->name ? view->name : "", view->offset,
                    view->byte_len, view->byte_len, "unsupported tensor quant %s",
                    quant_name(view->quant));
    size_t r = 0, c = 0;
    int rc = infer_rows_cols(view, f, &r, &c, "RepackedWeight::repack");
    if (rc) return rc;
    return weight_upload(view, r, c, as_stream(stream), out);
}

int jkb_weight_destroy(jkb_weight *w) {
    int rc = check_weight(w);
    if (rc) return rc;
    w->magic = 0;
    cudaFree(w->base);
    delete w;
    return JKB_OK;
}

int jkb_weight_info(const jkb_weight *w, size_t *rows, size_t *cols, int32_t *quant,
                    size_t *device_bytes, size_t *gguf_bytes) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (quant) *quant = w->quant;
    if (device_bytes) *device_bytes = w->device_bytes;
    if (gguf_bytes) *gguf_bytes = w->gguf_bytes;
    return JKB_OK;
}

int jkb_repacked_weight_from_tensor(const jkb_tensor_view *view, size_t rows, size_t cols,
                                    void *stream, jkb_repacked_weight **out) {
    return repacked_upload(view, rows, cols, as_stream(stream), out);
}

int jkb_repacked_weight_repack(const jkb_tensor_view *view, void *stream,
                               jkb_repacked_weight **out) {
    if (!view || !out) return fail(JKB_E_INVALID, "jkb_repacked_weight_repack", 0, 0, 0, "null");
    const Fmt *f = fmt_of(view->quant);
    if (!f)
        return fail(JKB_E_CAPABILITY, view->name ? view->name : "", view->offset,
                    view->byte_len, view->byte_len, "unsupported tensor quant %s for repack",
                    quant_name(view->quant));
    size_t r = 0, c = 0;
    int rc = infer_rows_cols(view, f, &r, &c, "RepackedWeight::repack");
    if (rc) return rc;
    return repacked_upload(view, r, c, as_stream(stream), out);
}

int jkb_repacked_weight_destroy(jkb_repacked_weight *w) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null or destroyed handle");
    w->magic = 0;
    cudaFree(w->base);
    delete w;
    return JKB_OK;
}

int jkb_repacked_weight_dequantize_row(const jkb_repacked_weight *w, size_t row, float *out,
                                       size_t out_len, void *stream) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null or destroyed handle");
    if (row >= w->rows || out_len != w->cols)
        return fail(JKB_E_BOUNDS, "RepackedWeight::dequantize_row", row, out_len * 4,
                    w->cols * 4, "invalid row (%zu/%zu) or output length (%zu/%zu)", row,
                    w->rows, out_len, w->cols);
    if (!out) return fail(JKB_E_INVALID, "RepackedWeight::dequantize_row", 0, 0, 0, "null output");
    int rc = check_align(out, 4, "RepackedWeight::dequantize_row", "output");
    if (rc) return rc;
    repacked_dequant_row_kernel<<<(unsigned)((w->cols + 255) / 256), 256, 0, as_stream(stream)>>>(
        w->q + row * w->k_pad, w->scales + row * w->scale_groups,
        w->mins ? w->mins + row * w->scale_groups : nullptr, w->cols, (int)w->group_elems, out);
    return check_launch("repacked_dequant_row_kernel");
}

int jkb_repacked_weight_buffers(const jkb_repacked_weight *w, size_t *rows, size_t *cols,
                                int32_t *quant, size_t *scale_groups, int8_t **q,
                                float **scales, float **mins) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null or destroyed handle");
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (quant) *quant = w->quant;
    if (scale_groups) *scale_groups = w->scale_groups;
    if (q) *q = w->q;
    if (scales) *scales = w->scales;
    if (mins) *mins = w->mins;
    return JKB_OK;
}

}  // extern "C"
