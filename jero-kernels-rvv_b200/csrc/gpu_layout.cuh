// GPU weight layout shared by the relayout (weights.cu) and the kernels that read it
// (gemv.cu, dots.cu).
//
// Every row's quant payload is contiguous and blocks keep their order. Blocks come in groups
// of 32 (the last group of a row may be shorter, n = min(32, nb - 32g)). Inside a group,
// 16-byte chunk j of the group's block l is stored at  group_base + j * 16 * n + 16 * l.
// One GEMV lane owns one block, so a warp-wide 16-byte load of chunk j reads 16 * n contiguous
// bytes. Byte counts equal the GGUF payload; nothing is padded.
#pragma once

#include <cstddef>
#include <cstdint>

namespace jkb {

// 16-byte quant chunks per block in the GPU layout
__host__ __device__ constexpr int qs_chunks(int gpu_format) {
    // GF_Q4_0, GF_Q8_0, GF_Q4_K, GF_Q6_K, GF_TQ2_0, GF_I2_S, GF_Q5_0, GF_Q5_K
    return gpu_format == 0 ? 1 : gpu_format == 1 ? 2 : gpu_format == 2 ? 8
         : gpu_format == 3 ? 12 : gpu_format == 4 ? 4 : gpu_format == 5 ? 2
         : gpu_format == 6 ? 1 : 10;
}

// Byte offset of chunk j of block b inside one row's quant payload.
__host__ __device__ __forceinline__ size_t qs_chunk_offset(int nb, int qch, int b, int j) {
    const int g = b >> 5, l = b & 31;
    const int n = (nb - 32 * g) < 32 ? (nb - 32 * g) : 32;
    return (size_t)32 * g * qch * 16 + (size_t)j * 16 * n + 16 * (size_t)l;
}

}  // namespace jkb
