// Device arithmetic shared by the activation quantizers (quantize.cu) and the GEMV kernels that
// quantize their f32 input while staging it (gemv.cu), so that both produce the same bytes.
#pragma once

#include <cuda_runtime.h>

namespace jkb {

__device__ __forceinline__ bool finite_f(float v) { return isfinite(v); }

// round_scaled_to_i8 (quant_q8.rs:102-108): non-finite -> 0, else round-half-away(v * inv)
// clamped to [-127, 127].
__device__ __forceinline__ int round_scaled(float v, float inv) {
    if (!finite_f(v)) return 0;
    float r = roundf(__fmul_rn(v, inv));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return (int)r;
}

// Block scale of quantize_block_q8_0_scalar / quantize_block_q8_k_scalar (quant_q8.rs:203-219,
// :447-475) from the block's absmax over finite values: d = amax / 127, inv = 127 / amax, both
// 0 for an all-zero (or all non-finite) block.
__device__ __forceinline__ void q8_scale(float amax, float &d, float &inv) {
    d = 0.0f;
    inv = 0.0f;
    if (amax != 0.0f) {
        d = __fdiv_rn(amax, 127.0f);
        inv = __fdiv_rn(127.0f, amax);
    }
}

}  // namespace jkb
