// One GGUF block of a RepackedWeight row expanded to i8 values and f32 group scales (and mins):
// repack_block_scaled_range_into_i8 (repack.rs:1724-2103) for the 14 block-scaled formats.
// Shared by the load-time repack kernel (weights.cu, one thread per block) and the host tile
// packer of the parallel load path (repack_into_tile_range, repack.rs:1579), so both write the
// same values bit for bit.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>

#include "jkb200.h"

namespace jkb {

// Little-endian u16 of a block header field.
__host__ __device__ __forceinline__ uint16_t rd16_le(const uint8_t *p) {
    return (uint16_t)(p[0] | (p[1] << 8));
}

// IEEE binary16 bits -> f32 (exact), non-finite -> 0.0 (f16_to_f32_finite, lib.rs:714-717).
__host__ __device__ __forceinline__ float f16_bits_finite(uint16_t h) {
    if (((h >> 10) & 0x1F) == 0x1F) return 0.0f;
#ifdef __CUDA_ARCH__
    return __half2float(__ushort_as_half(h));
#else
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, f;
    if (e == 0 && m == 0) {
        f = s;
    } else if (e == 0) {  // subnormal: m * 2^-24, renormalized
        int sh = 0;
        while (!(m & 0x400u)) {
            m <<= 1;
            sh++;
        }
        f = s | ((uint32_t)(113 - sh) << 23) | ((m & 0x3FFu) << 13);
    } else {
        f = s | ((e + 112u) << 23) | (m << 13);
    }
    float r;
    memcpy(&r, &f, 4);
    return r;
#endif
}

// One separately rounded f32 product (the reference's `d * sc` scale products).
__host__ __device__ __forceinline__ float mul_rn(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}

// Elements per GGUF block and per scale group of a block-scaled format (0 if not one).
__host__ __device__ inline int repack_block_elems(int quant) {
    switch (quant) {
    case JKB_Q8_0: case JKB_Q4_0: case JKB_Q4_1: case JKB_Q5_0: case JKB_Q5_1: case JKB_IQ4_NL:
        return 32;
    case JKB_I2_S: return 128;
    case JKB_Q4_K_M: case JKB_Q5_K: case JKB_Q6_K: case JKB_Q2_K: case JKB_Q3_K:
    case JKB_TQ1_0: case JKB_TQ2_0:
        return 256;
    default: return 0;
    }
}
// BlockScaledTileLayout::from_validated_dims (repack.rs:1338-1366): 16-element scale groups for
// Q6_K, Q3_K and Q2_K (chunks_per_scale 1), 32 otherwise; mins for the asymmetric formats.
__host__ __device__ inline int repack_group_elems(int quant) {
    return (quant == JKB_Q6_K || quant == JKB_Q3_K || quant == JKB_Q2_K) ? 16 : 32;
}
__host__ __device__ inline bool repack_has_mins(int quant) {
    return quant == JKB_Q4_K_M || quant == JKB_Q5_K || quant == JKB_Q4_1 || quant == JKB_Q5_1 ||
           quant == JKB_Q2_K;
}

// Block `blk` (GGUF bytes) -> q[0 .. block_elems) i8 values, s[0 .. groups) scales and, for the
// formats with mins, m[0 .. groups) mins (groups = block_elems / group_elems). `i2s` is the
// I2_S per-tensor trailer scale.
__host__ __device__ inline void repack_block_i8(int quant, const uint8_t *blk, int8_t *q,
                                                float *s, float *m, float i2s) {
    switch (quant) {
    case JKB_Q8_0: {
        const float dd = f16_bits_finite(rd16_le(blk));
        s[0] = dd;
        for (int i = 0; i < 32; i++) q[i] = dd != 0.0f ? (int8_t)blk[2 + i] : 0;
        break;
    }
    case JKB_Q4_0: {
        const float dd = f16_bits_finite(rd16_le(blk));
        s[0] = dd;
        for (int i = 0; i < 16; i++) {
            q[i] = dd != 0.0f ? (int8_t)((blk[2 + i] & 0x0F) - 8) : 0;
            q[16 + i] = dd != 0.0f ? (int8_t)(((blk[2 + i] >> 4) & 0x0F) - 8) : 0;
        }
        break;
    }
    case JKB_Q4_K_M:
    case JKB_Q5_K: {  // scales d * sc, mins dmin * m; Q4_K_M codes 0..15, Q5_K 0..31
        const float dd = f16_bits_finite(rd16_le(blk)), dmin = f16_bits_finite(rd16_le(blk + 2));
        const uint8_t *sb = blk + 4;
        uint8_t scv[8], mv[8];
        for (int j = 0; j < 4; j++) {
            scv[j] = sb[j] & 0x3F;
            mv[j] = sb[j + 4] & 0x3F;
        }
        for (int j = 4; j < 8; j++) {
            scv[j] = (uint8_t)((sb[j + 4] & 0x0F) | ((sb[j - 4] >> 6) << 4));
            mv[j] = (uint8_t)((sb[j + 4] >> 4) | ((sb[j] >> 6) << 4));
        }
        const bool q5 = quant == JKB_Q5_K;
        const uint8_t *qh = blk + 16, *qs = q5 ? blk + 48 : blk + 16;
        for (int c = 0; c < 4; c++) {
            s[2 * c] = mul_rn(dd, (float)scv[2 * c]);
            m[2 * c] = mul_rn(dmin, (float)mv[2 * c]);
            s[2 * c + 1] = mul_rn(dd, (float)scv[2 * c + 1]);
            m[2 * c + 1] = mul_rn(dmin, (float)mv[2 * c + 1]);
            for (int l = 0; l < 32; l++) {
                int lo = qs[32 * c + l] & 0x0F, hi = (qs[32 * c + l] >> 4) & 0x0F;
                if (q5) {
                    lo += ((qh[l] >> (2 * c)) & 1) ? 16 : 0;
                    hi += ((qh[l] >> (2 * c + 1)) & 1) ? 16 : 0;
                }
                q[64 * c + l] = (int8_t)lo;
                q[64 * c + 32 + l] = (int8_t)hi;
            }
        }
        break;
    }
    case JKB_Q5_0: {  // repack.rs:1827-1840: (5-bit code - 16), left 0 when d == 0
        const float dd = f16_bits_finite(rd16_le(blk));
        s[0] = dd;
        const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) |
                            ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
        for (int i = 0; i < 16; i++) {
            const int q0 = (int)((blk[6 + i] & 0x0F) | (((qh >> i) & 1) << 4)) - 16;
            const int q1 = (int)(((blk[6 + i] >> 4) & 0x0F) | (((qh >> (i + 16)) & 1) << 4)) - 16;
            q[i] = dd != 0.0f ? (int8_t)q0 : 0;
            q[16 + i] = dd != 0.0f ? (int8_t)q1 : 0;
        }
        break;
    }
    case JKB_Q6_K: {
        const float dd = f16_bits_finite(rd16_le(blk + 208));
        for (int g = 0; g < 16; g++) s[g] = mul_rn(dd, (float)(int8_t)blk[192 + g]);
        const uint8_t *ql = blk, *qh = blk + 128;
        const bool z = dd == 0.0f;
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 32; l++) {
                const int lb = 64 * h, hb = 32 * h, n = 128 * h;
                const int q1 = (int)((ql[lb + l] & 0x0F) | ((qh[hb + l] & 3) << 4)) - 32;
                const int q2 = (int)((ql[lb + l + 32] & 0x0F) | (((qh[hb + l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int)(((ql[lb + l] >> 4) & 0x0F) | (((qh[hb + l] >> 4) & 3) << 4)) - 32;
                const int q4 =
                    (int)(((ql[lb + l + 32] >> 4) & 0x0F) | (((qh[hb + l] >> 6) & 3) << 4)) - 32;
                q[n + l] = z ? 0 : (int8_t)q1;
                q[n + l + 32] = z ? 0 : (int8_t)q2;
                q[n + l + 64] = z ? 0 : (int8_t)q3;
                q[n + l + 96] = z ? 0 : (int8_t)q4;
            }
        break;
    }
    case JKB_TQ2_0:
    case JKB_TQ1_0: {
        const float dd = f16_bits_finite(rd16_le(blk));
        for (int g = 0; g < 8; g++) s[g] = dd;
        if (quant == JKB_TQ2_0) {
            for (int e = 0; e < 256; e++)
                q[e] = (int8_t)(((blk[2 + e / 4] >> (2 * (e % 4))) & 3) - 1);
        } else {
            for (int i = 0; i < 51; i++) {
                unsigned v = blk[2 + i];
                for (int j = 0; j < 5; j++) {
                    q[5 * i + j] = (int8_t)((int)(v % 3) - 1);
                    v /= 3;
                }
            }
            q[255] = (int8_t)((int)(blk[53] % 3) - 1);
        }
        break;
    }
    case JKB_Q4_1: {  // repack.rs:1814-1826: scale d, min -m (0.0 when m == 0), unsigned codes
        const float dd = f16_bits_finite(rd16_le(blk)), mm = f16_bits_finite(rd16_le(blk + 2));
        s[0] = dd;
        m[0] = mm == 0.0f ? 0.0f : -mm;
        for (int i = 0; i < 16; i++) {
            q[i] = (int8_t)(blk[4 + i] & 0x0F);
            q[16 + i] = (int8_t)(blk[4 + i] >> 4);
        }
        break;
    }
    case JKB_Q5_1: {  // repack.rs:1841-1855 with unpack_q5_1_block_i8 (quant.rs:169-190)
        const float dd = f16_bits_finite(rd16_le(blk)), mm = f16_bits_finite(rd16_le(blk + 2));
        s[0] = dd;
        m[0] = mm == 0.0f ? 0.0f : -mm;
        const uint32_t qh = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) |
                            ((uint32_t)blk[6] << 16) | ((uint32_t)blk[7] << 24);
        for (int i = 0; i < 16; i++) {
            q[i] = (int8_t)((blk[8 + i] & 0x0F) | (((qh >> i) & 1) << 4));
            q[16 + i] = (int8_t)((blk[8 + i] >> 4) | (((qh >> (i + 16)) & 1) << 4));
        }
        break;
    }
    case JKB_IQ4_NL: {  // repack.rs:1856-1873: the code book values, left 0 when d == 0
        // KVALUES_IQ4NL (quant.rs:80-82)
        constexpr int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                   1,    13,   25,  38,  53,  69,  89,  113};
        const float dd = f16_bits_finite(rd16_le(blk));
        s[0] = dd;
        for (int i = 0; i < 16; i++) {
            q[i] = dd != 0.0f ? kv[blk[2 + i] & 0x0F] : 0;
            q[16 + i] = dd != 0.0f ? kv[blk[2 + i] >> 4] : 0;
        }
        break;
    }
    case JKB_Q2_K: {  // repack.rs:1874-1892 with unpack_q2_k_block_i8 (quant.rs:198-246)
        // sub-block g (16 elements) takes the 2-bit field 2 * ((g % 8) / 2) of
        // qs[32 (g / 8) + 16 (g % 2) + l]; scale d * (sc & 15), min dmin * (sc >> 4)
        const float dd = f16_bits_finite(rd16_le(blk + 80)),
                    dmin = f16_bits_finite(rd16_le(blk + 82));
        for (int g = 0; g < 16; g++) {
            s[g] = mul_rn(dd, (float)(blk[g] & 0x0F));
            m[g] = mul_rn(dmin, (float)(blk[g] >> 4));
            const int sh = 2 * ((g % 8) / 2);
            const uint8_t *qs = blk + 16 + 32 * (g / 8) + 16 * (g % 2);
            for (int l = 0; l < 16; l++) q[16 * g + l] = (int8_t)((qs[l] >> sh) & 3);
        }
        break;
    }
    case JKB_Q3_K: {  // repack.rs:1893-1908 with unpack_q3_k_block_i8 (quant.rs:255-330)
        // 6-bit scale g: low 4 bits from byte g (g < 8, low nibble) or g - 8 (high nibble),
        // top 2 bits from byte 8 + g % 4 at bit 2 (g / 4); codes minus 4 where the hmask bit
        // g / 2 of hmask[16 (g % 2) + l] is clear
        const uint8_t *hm = blk, *raw6 = blk + 96;
        const float dd = f16_bits_finite(rd16_le(blk + 108));
        for (int g = 0; g < 16; g++) {
            const int lo = g < 8 ? raw6[g] & 0x0F : raw6[g - 8] >> 4;
            const int hi = (raw6[8 + g % 4] >> (2 * (g / 4))) & 3;
            s[g] = mul_rn(dd, (float)((lo | (hi << 4)) - 32));
            const int sh = 2 * ((g % 8) / 2);
            const uint8_t *qs = blk + 32 + 32 * (g / 8) + 16 * (g % 2);
            for (int l = 0; l < 16; l++) {
                const int code = (qs[l] >> sh) & 3;
                const int high = (hm[16 * (g % 2) + l] >> (g / 2)) & 1;
                q[16 * g + l] = (int8_t)(code - (high ? 0 : 4));
            }
        }
        break;
    }
    case JKB_I2_S: {
        for (int g = 0; g < 4; g++) s[g] = i2s;
        const bool z = i2s == 0.0f;
        for (int g = 0; g < 32; g++) {
            const uint8_t v = blk[g];
            q[g] = z ? 0 : (int8_t)(((v >> 6) & 3) - 1);
            q[32 + g] = z ? 0 : (int8_t)(((v >> 4) & 3) - 1);
            q[64 + g] = z ? 0 : (int8_t)(((v >> 2) & 3) - 1);
            q[96 + g] = z ? 0 : (int8_t)((v & 3) - 1);
        }
        break;
    }
    default: break;
    }
}

}  // namespace jkb
