// Compact 4-bit weights (jkb_nibble_matrix, the GPU form of PackedNibbleMatrix, repack.rs:
// 4188-5545): format codes and the device arithmetic shared by the tensor-core GEMM's converter
// warps (gemm_tc.cu) and the row kernels (nibble.cu).
//
// Device layout (rows contiguous, blocks in K order, byte counts equal to the GGUF payload):
//   qs    [rows][cols / 2]: each row's GGUF quant bytes. Q4_0 / Q4_1 / IQ4_NL: 16 bytes per
//         32-element block, byte k = element k (low nibble) | element 16 + k (high nibble).
//         Q4_K_M: 128 bytes per 256-element block; byte 32c + l = element 64c + l (low) |
//         element 64c + 32 + l (high).
//   meta  [rows][blocks]: Q4_0 / IQ4_NL the f16 d; Q4_1 the f16 pair (d, m) as one 32-bit word;
//         Q4_K_M the 16-byte header (d, dmin, scales[12]).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace jkb {

enum NibFmt { NIB_NONE = 0, NIB_Q4_0 = 1, NIB_Q4_1 = 2, NIB_IQ4_NL = 3, NIB_Q4_K = 4 };

// f16_to_f32_finite (lib.rs:714-717): exact conversion, NaN / Inf -> 0.
__device__ __forceinline__ float nib_f16_finite(uint32_t bits) {
    const float v = __half2float(__ushort_as_half((unsigned short)(bits & 0xFFFF)));
    return ((bits >> 10) & 0x1F) == 0x1F ? 0.0f : v;
}

// Q4_0 / IQ4_NL block scale as the reference's tiles hold it: blocks whose scale decodes to
// zero (0, -0, NaN, Inf) are stored with scale bits 0, i.e. +0.0 (repack.rs:4458-4500).
__device__ __forceinline__ float nib_d_scale(uint32_t bits) {
    const float v = nib_f16_finite(bits);
    return v == 0.0f ? 0.0f : v;
}

// Q4_1 min term as decode_tile_scales forms it (repack.rs:5057-5070): -m, or +0.0 when m == 0.
__device__ __forceinline__ float nib_q4_1_min(uint32_t bits) {
    const float m = nib_f16_finite(bits);
    return m == 0.0f ? 0.0f : -m;
}

// Scale / min pair j (0..7) of a Q4_K_M header (unpack_q4_q5_k_scales_mins, quant_q8.rs:
// 1818-1830). w1, w2, w3 are header bytes 4..7, 8..11, 12..15 (scales[0..12]).
__device__ __forceinline__ void nib_k4_scale_min(uint32_t w1, uint32_t w2, uint32_t w3, int j,
                                                 int &sc, int &m) {
    auto byte = [&](int i) -> uint32_t {
        const uint32_t w = i < 4 ? w1 : i < 8 ? w2 : w3;
        return (w >> (8 * (i & 3))) & 0xFF;
    };
    if (j < 4) {
        sc = (int)(byte(j) & 0x3F);
        m = (int)(byte(j + 4) & 0x3F);
    } else {
        sc = (int)((byte(j + 4) & 0x0F) | ((byte(j - 4) >> 6) << 4));
        m = (int)((byte(j + 4) >> 4) | ((byte(j) >> 6) << 4));
    }
}

// Byte K (0..3) of w as an exact f32: 0x4B0000XX is 2^23 + XX.
template <int K>
__device__ __forceinline__ float nib_byte_f32(uint32_t w) {
    return __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7540u + K)) - 8388608.0f;
}

// Four nibble codes (one per byte, 0..15) to the int8 weight values of format F:
// Q4_0 code - 8; IQ4_NL the code book KVALUES_IQ4NL (quant.rs:80-82); Q4_1 / Q4_K_M the code.
template <int F>
__device__ __forceinline__ uint32_t nib_values4(uint32_t codes) {
    if (F == NIB_Q4_0) {
        // per byte: (code + 0x78) ^ 0x80 = code - 8 (no carry: code + 0x78 <= 0x87)
        return (codes + 0x78787878u) ^ 0x80808080u;
    } else if (F == NIB_IQ4_NL) {
        // code book bytes: -127 -104 -83 -65 | -49 -35 -22 -10 | 1 13 25 38 | 53 69 89 113
        constexpr uint32_t L0 = 0xBFAD9881u, L1 = 0xF6EADDCFu, L2 = 0x26190D01u,
                           L3 = 0x71594535u;
        // byte-select index of each output byte: code & 7, one nibble per byte in 16 bits
        const uint32_t y = codes | (codes >> 4);  // bytes 0 and 2 hold (c0 | c1 << 4), (c2 | c3 << 4)
        const uint32_t sel = __byte_perm(y, 0u, 0x0020u) & 0x7777u;
        const uint32_t lo8 = __byte_perm(L0, L1, sel), hi8 = __byte_perm(L2, L3, sel);
        const uint32_t upper = ((codes >> 3) & 0x01010101u) * 0xFFu;  // 0xFF where code >= 8
        return (hi8 & upper) | (lo8 & ~upper);
    } else {
        return codes;
    }
}

}  // namespace jkb
