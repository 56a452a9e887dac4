// Activation quantizers: BlockQ8_0 / BlockQ8K rows (quant_q8.rs), QuantizedActQ8 per-32 blocks
// (repack.rs) and the BitNet SubLN absmax quantizer (lib.rs). All are bit-exact restatements:
// IEEE division (__fdiv_rn), round-half-away-from-zero (roundf), separately rounded multiplies
// and adds where the reference sums in f32.
#include <cstring>

#include "jkb_internal.h"
#include "quant_math.cuh"

namespace jkb {

// quantize_block_q8_0_scalar (quant_q8.rs:203-219): 8 lanes per 32-element block, 4 values per
// lane. absmax over finite values (a max is order independent), amax == 0 -> ZERO block.
template <bool VEC>
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float *__restrict__ x,
                                                            size_t nblocks,
                                                            uint8_t *__restrict__ out) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t blk = gid >> 3;
    int sub = (int)(gid & 7);
    bool valid = blk < nblocks;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
        const float *p = x + blk * 32 + 4 * sub;
        if (VEC) {
            float4 t = __ldg(reinterpret_cast<const float4 *>(p));
            v[0] = t.x;
            v[1] = t.y;
            v[2] = t.z;
            v[3] = t.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = __ldg(p + i);
        }
    }
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++)
        if (finite_f(v[i])) a = fmaxf(a, fabsf(v[i]));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
    if (!valid) return;
    uint8_t *ob = out + blk * 36;
    float d = 0.0f;
    uint32_t packed = 0;
    if (a != 0.0f) {
        d = __fdiv_rn(a, 127.0f);
        float inv = __fdiv_rn(127.0f, a);
#pragma unroll
        for (int i = 0; i < 4; i++) packed |= ((uint32_t)(round_scaled(v[i], inv) & 0xFF)) << (8 * i);
    }
    if (sub == 0) *reinterpret_cast<float *>(ob) = d;
    *reinterpret_cast<uint32_t *>(ob + 4 + 4 * sub) = packed;
}

// quantize_block_q8_k_scalar (quant_q8.rs:447-475): one warp per 256-element block, 8 values per
// lane; bsums[j] = sum of the 16 quantized values of lanes 2j and 2j+1.
template <bool VEC>
__global__ void __launch_bounds__(256) quantize_q8_k_kernel(const float *__restrict__ x,
                                                            size_t nblocks,
                                                            uint8_t *__restrict__ out) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    size_t blk = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    bool valid = blk < nblocks;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = 0.0f;
    if (valid) {
        const float *p = x + blk * 256 + 8 * lane;
        if (VEC) {
            float4 t0 = __ldg(reinterpret_cast<const float4 *>(p));
            float4 t1 = __ldg(reinterpret_cast<const float4 *>(p + 4));
            v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
            v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __ldg(p + i);
        }
    }
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++)
        if (finite_f(v[i])) a = fmaxf(a, fabsf(v[i]));
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, m));
    float d = 0.0f, inv = 0.0f;
    if (a != 0.0f) {
        d = __fdiv_rn(a, 127.0f);
        inv = __fdiv_rn(127.0f, a);
    }
    uint32_t p0 = 0, p1 = 0;
    int s = 0;
    if (a != 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int q = round_scaled(v[i], inv);
            s += q;
            if (i < 4)
                p0 |= ((uint32_t)(q & 0xFF)) << (8 * i);
            else
                p1 |= ((uint32_t)(q & 0xFF)) << (8 * (i - 4));
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (!valid) return;
    uint8_t *ob = out + blk * 292;
    if (lane == 0) *reinterpret_cast<float *>(ob) = d;
    *reinterpret_cast<uint32_t *>(ob + 4 + 8 * lane) = p0;
    *reinterpret_cast<uint32_t *>(ob + 8 + 8 * lane) = p1;
    if ((lane & 1) == 0) *reinterpret_cast<int16_t *>(ob + 260 + lane) = (int16_t)s;
}

// quantize_block32_scalar (repack.rs:175-204) on the `valid` leading elements of src (the
// rest of the 32 read as 0, non-finite values as 0): the i8 quants packed in words[8], the scale
// absmax / 127 (0 when absmax < 1e-30), the sequential f32 sum from 0.0 and the two 16-element
// half sums from -0.0 (QuantizedActQ8's x_sums_16), all in element order as in the reference.
struct QBlock32 {
    uint32_t words[8];
    float d, s, h0, h1;
};
__device__ __forceinline__ void quant_block32(const float *__restrict__ src, size_t valid,
                                              QBlock32 &o) {
    float c[32];
    float absmax = 0.0f, s = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        float v = (size_t)i < valid ? __ldg(src + i) : 0.0f;
        v = finite_f(v) ? v : 0.0f;
        c[i] = v;
        s = __fadd_rn(s, v);
        float av = fabsf(v);
        if (av > absmax) absmax = av;
    }
    float h0 = -0.0f, h1 = -0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) h0 = __fadd_rn(h0, c[i]);
#pragma unroll
    for (int i = 16; i < 32; i++) h1 = __fadd_rn(h1, c[i]);
    float d = 0.0f;
    if (absmax < 1e-30f) {
#pragma unroll
        for (int i = 0; i < 8; i++) o.words[i] = 0;
    } else {
        d = __fdiv_rn(absmax, 127.0f);
        float inv = __fdiv_rn(127.0f, absmax);
#pragma unroll
        for (int w = 0; w < 8; w++) {
            uint32_t pk = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float t = roundf(__fmul_rn(c[4 * w + j], inv));
                t = fminf(fmaxf(t, -127.0f), 127.0f);
                pk |= ((uint32_t)((int)t & 0xFF)) << (8 * j);
            }
            o.words[w] = pk;
        }
    }
    o.d = d;
    o.s = s;
    o.h0 = h0;
    o.h1 = h1;
}

// quantize_row_f32_to_q8_32 (repack.rs:376-455): one thread per 32-element block of one row.
__global__ void __launch_bounds__(256) q8_32_row_kernel(const float *__restrict__ x, size_t len,
                                                        int8_t *__restrict__ q,
                                                        float *__restrict__ scales,
                                                        float *__restrict__ sums) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b * 32 >= len) return;
    QBlock32 o;
    quant_block32(x + 32 * b, len - 32 * b < 32 ? len - 32 * b : 32, o);
    int8_t *qb = q + 32 * b;
    if ((((uintptr_t)qb) & 15) == 0) {
        reinterpret_cast<uint4 *>(qb)[0] = make_uint4(o.words[0], o.words[1], o.words[2], o.words[3]);
        reinterpret_cast<uint4 *>(qb)[1] = make_uint4(o.words[4], o.words[5], o.words[6], o.words[7]);
    } else {
        for (int i = 0; i < 32; i++) qb[i] = (int8_t)((o.words[i / 4] >> (8 * (i % 4))) & 0xFF);
    }
    scales[b] = o.d;
    sums[b] = o.s;
}

// QuantizedActQ8::quantize_into (repack.rs:542-650) with quantize_block32_scalar
// (repack.rs:175-204): one thread per 32-element block, so the f32 sums run sequentially in
// element order exactly as in the reference (x_sums from 0.0, x_sums_16 from -0.0).
__global__ void __launch_bounds__(256) act_q8_kernel(const float *__restrict__ act, size_t m,
                                                     size_t k, size_t kp,
                                                     int8_t *__restrict__ q,
                                                     float *__restrict__ xs,
                                                     float *__restrict__ xsum,
                                                     float *__restrict__ xs16,
                                                     float *__restrict__ xs_t,
                                                     float *__restrict__ xsn_t,
                                                     float *__restrict__ xsn16_t,
                                                     size_t xt_pitch) {
    size_t kb = kp / 32;
    size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t m_t = xs_t ? (m + 31) / 32 * 32 : m;  // tokens covered by the transposed plane
    if (gid >= m_t * kb) return;
    size_t r = gid / kb, b = gid % kb;
    // Transposed scales are stored permuted within each 32-token block: token 8u + 2v + e
    // (u, v < 4, e < 2) goes to position 16(u >> 1) + 4v + 2(u & 1) + e, so that the token
    // pairs 2v + {0, 8, 16, 24} of a block (one tensor-core epilogue lane's) are two 16-byte
    // words. Positions of tokens >= m in the last block hold 0.
    const size_t xt_at = b * xt_pitch + (r & ~(size_t)31) + 16 * ((r >> 4) & 1) +
                         4 * ((r >> 1) & 3) + 2 * ((r >> 3) & 1) + (r & 1);
    const size_t xt16_at = xt_at + b * xt_pitch;  // 16-element group 2b (2b + 1 one row on)
    if (r >= m) {
        xs_t[xt_at] = 0.0f;
        xsn_t[xt_at] = 0.0f;
        if (xsn16_t) xsn16_t[xt16_at] = xsn16_t[xt16_at + xt_pitch] = 0.0f;
        return;
    }
    QBlock32 o;
    quant_block32(act + r * k + b * 32, k > b * 32 ? (k - b * 32 < 32 ? k - b * 32 : 32) : 0, o);
    const uint32_t *words = o.words;
    const float d = o.d, s = o.s, h0 = o.h0, h1 = o.h1;
    uint4 *qo = reinterpret_cast<uint4 *>(q + r * kp + b * 32);
    qo[0] = make_uint4(words[0], words[1], words[2], words[3]);
    qo[1] = make_uint4(words[4], words[5], words[6], words[7]);
    xs[r * kb + b] = d;
    if (xs_t) {
        xs_t[xt_at] = d;
        xsn_t[xt_at] = -s;
        if (xsn16_t) {
            xsn16_t[xt16_at] = -h0;
            xsn16_t[xt16_at + xt_pitch] = -h1;
        }
    }
    xsum[r * kb + b] = s;
    xs16[r * (kp / 16) + 2 * b] = h0;
    xs16[r * (kp / 16) + 2 * b + 1] = h1;
}

// i8 BitLinear activations (per-token scale) in the jkb_act_q8 layout the tensor-core GEMM
// reads: q the i8 rows (k == k_pad: BitLinear widths are multiples of the block), every
// 32-element group's scale the token's (x_scales and its transposed, permuted copy, as
// act_q8_kernel places it), sums zero. One thread per (token, 32-element group).
__global__ void __launch_bounds__(256) act_from_i8_kernel(const int8_t *__restrict__ act,
                                                          const float *__restrict__ scales,
                                                          size_t m, size_t kp,
                                                          int8_t *__restrict__ q,
                                                          float *__restrict__ xs,
                                                          float *__restrict__ xsum,
                                                          float *__restrict__ xs_t,
                                                          size_t xt_pitch) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    const size_t kb = kp / 32;
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t m_t = xs_t ? (m + 31) / 32 * 32 : m;
    if (gid >= m_t * kb) return;
    const size_t r = gid / kb, b = gid % kb;
    const size_t xt_at = b * xt_pitch + (r & ~(size_t)31) + 16 * ((r >> 4) & 1) +
                         4 * ((r >> 1) & 3) + 2 * ((r >> 3) & 1) + (r & 1);
    if (r >= m) {
        xs_t[xt_at] = 0.0f;
        return;
    }
    const float s = __ldg(scales + r);
    const int8_t *src = act + r * kp + b * 32;
    uint4 *dst = reinterpret_cast<uint4 *>(q + r * kp + b * 32);
    if ((((uintptr_t)src) & 15) == 0) {
        dst[0] = __ldg(reinterpret_cast<const uint4 *>(src));
        dst[1] = __ldg(reinterpret_cast<const uint4 *>(src) + 1);
    } else {
        uint32_t w[8];
        for (int i = 0; i < 8; i++)
            w[i] = (uint32_t)(uint8_t)src[4 * i] | ((uint32_t)(uint8_t)src[4 * i + 1] << 8) |
                   ((uint32_t)(uint8_t)src[4 * i + 2] << 16) |
                   ((uint32_t)(uint8_t)src[4 * i + 3] << 24);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
    xs[r * kb + b] = s;
    xsum[r * kb + b] = 0.0f;
    if (xs_t) xs_t[xt_at] = s;
}

// super_scales_256 (repack.rs:623-630): slot starts at 0.0, `if sc > slot { slot = sc }` over
// the 32-blocks of each 256 span.
__global__ void act_super_kernel(const float *__restrict__ xs, size_t m, size_t kb, size_t nsb,
                                 float *__restrict__ sup) {
    size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= m * nsb) return;
    size_t r = gid / nsb, s = gid % nsb;
    float v = 0.0f;
    for (size_t b = 8 * s; b < 8 * s + 8 && b < kb; b++) {
        float sc = xs[r * kb + b];
        if (sc > v) v = sc;
    }
    sup[gid] = v;
}

// relu_squared_gate_scalar (lib.rs:1130-1137): max(0, g)^2 * u, the two products rounded in the
// reference's order ((relu * relu) * up). NaN and -0 gates give +0 (g > 0 is false), as in the
// reference and its vfmax form.
__device__ __forceinline__ float relu_squared_gate(float g, float u) {
    const float r = g > 0.0f ? g : 0.0f;
    return __fmul_rn(__fmul_rn(r, r), u);
}

// relu_squared_gate_f32 (lib.rs:1111-1148): elementwise over n values.
__global__ void __launch_bounds__(256) relu_squared_kernel(const float *__restrict__ gate,
                                                           const float *__restrict__ up,
                                                           size_t n, float *__restrict__ out) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = relu_squared_gate(__ldg(gate + i), __ldg(up + i));
}

// subln_quantize_absmax_i8 (lib.rs:1042-1101), one CTA per row. The sum of squares is the
// reference's sequential f32 dot (dot_product_f32_scalar, lib.rs:770-777), so one thread walks
// it in element order; everything else is elementwise (the absmax a max-reduction) and runs on
// all threads. The row is read from global memory once (16-byte loads where the row allows)
// and kept in shared memory for the three passes.
// GATE: the row is relu_squared_gate_f32 of (in, up) (lib.rs:1111-1148), formed here and stored
// to relu_out when that is non-null, so that the BitNet FFN's activation of the down projection
// is one kernel; otherwise the row is in itself.
constexpr int SUBLN_THREADS = 512;

// Elements the one-thread sum takes per step: their 16-byte loads go out a step ahead.
constexpr int SUBLN_STEP = 32;

// The sequential f32 sum of v[0..len) (v 16-byte aligned) in element order, one thread.
// SQ: v holds the squares already, so the chain is adds only; otherwise each element is
// squared (rounded) first. The next step's loads are issued before the current step's adds.
// Measured on B200 (one thread, 5120 elements): 4.2 cycles an element with the squares
// precomputed, 4.4 squaring in the loop, against 5.5 for the earlier loop of 8 elements a step
// loaded one step ahead; a dependent f32 add takes 4.2-4.3 cycles.
template <bool SQ>
__device__ __forceinline__ float sequential_sum_sq(const float *v, size_t len) {
    constexpr int U = SUBLN_STEP / 4;
    float s0 = 0.0f;
    const size_t nsteps = len / SUBLN_STEP;
    const float4 *v4 = reinterpret_cast<const float4 *>(v);
    if (nsteps) {
        float4 cur[U];
#pragma unroll
        for (int k = 0; k < U; k++) cur[k] = v4[k];
        for (size_t j = 0; j < nsteps; j++) {
            float4 nxt[U];
            const size_t base = (j + 1 < nsteps ? j + 1 : j) * U;
#pragma unroll
            for (int k = 0; k < U; k++) nxt[k] = v4[base + k];
#pragma unroll
            for (int k = 0; k < U; k++) {
                if (SQ) {
                    s0 = __fadd_rn(s0, cur[k].x);
                    s0 = __fadd_rn(s0, cur[k].y);
                    s0 = __fadd_rn(s0, cur[k].z);
                    s0 = __fadd_rn(s0, cur[k].w);
                } else {
                    s0 = __fadd_rn(s0, __fmul_rn(cur[k].x, cur[k].x));
                    s0 = __fadd_rn(s0, __fmul_rn(cur[k].y, cur[k].y));
                    s0 = __fadd_rn(s0, __fmul_rn(cur[k].z, cur[k].z));
                    s0 = __fadd_rn(s0, __fmul_rn(cur[k].w, cur[k].w));
                }
            }
#pragma unroll
            for (int k = 0; k < U; k++) cur[k] = nxt[k];
        }
    }
    for (size_t i = nsteps * SUBLN_STEP; i < len; i++)
        s0 = __fadd_rn(s0, SQ ? v[i] : __fmul_rn(v[i], v[i]));
    return s0;
}

// Rows up to this length also keep their squares in shared memory (a second array after the
// row), so that the sequential sum is a chain of adds only.
constexpr size_t SUBLN_SQ_MAX_LEN = SUBLN_MAX_LEN / 2;

template <bool GATE>
__global__ void __launch_bounds__(SUBLN_THREADS) subln_kernel(
    const float *__restrict__ in, const float *__restrict__ up, const float *__restrict__ w,
    size_t len, float eps, int8_t *__restrict__ out, float *__restrict__ scales,
    float *__restrict__ relu_out) {
    extern __shared__ __align__(16) float sx[];
    __shared__ float s_inv_rms, s_red[SUBLN_THREADS / 32];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    const size_t row = (size_t)blockIdx.x * len;
    int8_t *o = out + row;
    // the squares, 16-byte aligned after the row, for rows up to SUBLN_SQ_MAX_LEN
    const bool keep_sq = len <= SUBLN_SQ_MAX_LEN;
    float *sq = sx + (len + 3) / 4 * 4;
    auto aligned16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    const bool vec = (len & 3) == 0 && aligned16(in + row) &&
                     (!GATE || (aligned16(up + row) && (!relu_out || aligned16(relu_out + row))));
    // pass 0: the row (or its ReLU^2 gating) into shared memory, and its squares
    if (vec) {
        const size_t n4 = len / 4;
        const float4 *i4 = reinterpret_cast<const float4 *>(in + row);
        for (size_t i = threadIdx.x; i < n4; i += blockDim.x) {
            float4 v = __ldg(i4 + i);
            if (GATE) {
                const float4 u = __ldg(reinterpret_cast<const float4 *>(up + row) + i);
                v = make_float4(relu_squared_gate(v.x, u.x), relu_squared_gate(v.y, u.y),
                                relu_squared_gate(v.z, u.z), relu_squared_gate(v.w, u.w));
                if (relu_out) reinterpret_cast<float4 *>(relu_out + row)[i] = v;
            }
            reinterpret_cast<float4 *>(sx)[i] = v;
            if (keep_sq)
                reinterpret_cast<float4 *>(sq)[i] =
                    make_float4(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y), __fmul_rn(v.z, v.z),
                                __fmul_rn(v.w, v.w));
        }
    } else {
        for (size_t i = threadIdx.x; i < len; i += blockDim.x) {
            float v = __ldg(in + row + i);
            if (GATE) {
                v = relu_squared_gate(v, __ldg(up + row + i));
                if (relu_out) relu_out[row + i] = v;
            }
            sx[i] = v;
            if (keep_sq) sq[i] = __fmul_rn(v, v);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // sum += x * x in element order: each product rounded, then added in sequence
        const float s0 = keep_sq ? sequential_sum_sq<true>(sq, len)
                                 : sequential_sum_sq<false>(sx, len);
        float mean_sq = __fdiv_rn(s0, (float)len);
        s_inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean_sq, eps)));
    }
    __syncthreads();
    // pass 1: x_norm = x * inv_rms * norm_weight (in place) and its absmax
    const float inv_rms = s_inv_rms;
    float mx = 0.0f;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) {
        const float xn = __fmul_rn(__fmul_rn(sx[i], inv_rms), __ldg(w + i));
        const float av = fabsf(xn);
        sx[i] = xn;
        if (av > mx) mx = av;
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        float t = __shfl_xor_sync(0xffffffffu, mx, m);
        if (t > mx) mx = t;
    }
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = 0.0f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++)
            if (s_red[i] > v) v = s_red[i];
        s_red[0] = v;
    }
    __syncthreads();
    // pass 2: quantize (or the guarded all-zero row)
    const float max_val = s_red[0];
    if (isnan(max_val) || max_val < 1e-12f) {
        for (size_t i = threadIdx.x; i < len; i += blockDim.x) o[i] = 0;
        if (threadIdx.x == 0) scales[blockIdx.x] = __fdiv_rn(1.0f, 127.0f);
        return;
    }
    const float scale = __fdiv_rn(max_val, 127.0f);
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) {
        float q = roundf(__fdiv_rn(sx[i], scale));
        int qi = 0;
        if (!isnan(q)) qi = (int)fminf(fmaxf(q, -128.0f), 127.0f);
        o[i] = (int8_t)qi;
    }
    if (threadIdx.x == 0) scales[blockIdx.x] = scale;
}

// Launches subln_kernel<GATE> over m rows of len (arguments validated by the callers).
int launch_subln(bool gate, int8_t *out_i8, float *relu_out, const float *input,
                 const float *up, const float *norm_weight, size_t m, size_t len, float eps,
                 float *scales_out, cudaStream_t st) {
    auto kern = gate ? subln_kernel<true> : subln_kernel<false>;
    static bool attr[2] = {false, false};
    if (!attr[gate]) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(SUBLN_MAX_LEN * 4));
        attr[gate] = true;
    }
    // the row, and its squares when it is short enough to keep them (subln_kernel)
    const size_t smem =
        (len <= SUBLN_SQ_MAX_LEN ? (len + 3) / 4 * 4 + len : len) * sizeof(float);
    cudaError_t e = launch_pdl(kern, dim3((unsigned)m), dim3(SUBLN_THREADS), smem, st, input, up,
                               norm_weight, len, eps, out_i8, scales_out, relu_out);
    return e == cudaSuccess ? JKB_OK : fail_cuda(e, "subln_kernel");
}

// validate_activation_input / validate_activation_quant_slice (quant_q8.rs:111-149)
static int validate_act(const char *name, size_t x_len, size_t out_len, size_t be) {
    if (x_len == 0 || x_len % be != 0)
        return fail(JKB_E_BOUNDS, name, 0, x_len * 4, out_len,
                    "%s: input length %zu must be a positive multiple of %zu", name, x_len, be);
    if (out_len != x_len / be)
        return fail(JKB_E_BOUNDS, name, 0, x_len * 4, out_len,
                    "%s: output block count %zu != expected %zu", name, out_len, x_len / be);
    return JKB_OK;
}

static int launch_q8_0(const float *x, size_t nblocks, void *out, cudaStream_t st) {
    int rc;
    if ((rc = check_align(x, 4, "quantize_row_q8_0", "x")) ||
        (rc = check_align(out, 4, "quantize_row_q8_0", "output blocks")))
        return rc;
    size_t threads = nblocks * 8;
    unsigned grid = (unsigned)((threads + 255) / 256);
    bool vec = ((uintptr_t)x & 15) == 0;
    cudaError_t e = vec ? launch_pdl(quantize_q8_0_kernel<true>, dim3(grid), dim3(256), 0, st, x,
                                     nblocks, (uint8_t *)out)
                        : launch_pdl(quantize_q8_0_kernel<false>, dim3(grid), dim3(256), 0, st, x,
                                     nblocks, (uint8_t *)out);
    return e == cudaSuccess ? JKB_OK : fail_cuda(e, "quantize_q8_0_kernel");
}

static int launch_q8_k(const float *x, size_t nblocks, void *out, cudaStream_t st) {
    int rc;
    if ((rc = check_align(x, 4, "quantize_row_q8_k", "x")) ||
        (rc = check_align(out, 4, "quantize_row_q8_k", "output blocks")))
        return rc;
    size_t threads = nblocks * 32;
    unsigned grid = (unsigned)((threads + 255) / 256);
    bool vec = ((uintptr_t)x & 15) == 0;
    cudaError_t e = vec ? launch_pdl(quantize_q8_k_kernel<true>, dim3(grid), dim3(256), 0, st, x,
                                     nblocks, (uint8_t *)out)
                        : launch_pdl(quantize_q8_k_kernel<false>, dim3(grid), dim3(256), 0, st, x,
                                     nblocks, (uint8_t *)out);
    return e == cudaSuccess ? JKB_OK : fail_cuda(e, "quantize_q8_k_kernel");
}

static bool check_act(const jkb_act_q8 *a) { return a && a->magic == ACT_MAGIC; }

// Fills act from m rows of i8 BitLinear activations and their per-token scales (device);
// act->k must be a multiple of 32 and m at most its capacity (checked by the caller).
int act_q8_from_i8(jkb_act_q8 *a, const int8_t *act_i8, const float *scales, size_t m,
                   cudaStream_t st) {
    const size_t kb = a->k_pad / 32;
    const size_t m_t = a->x_scales_t ? (m + 31) / 32 * 32 : m;
    const size_t threads = m_t * kb;
    cudaError_t e = launch_pdl(act_from_i8_kernel, dim3((unsigned)((threads + 255) / 256)),
                               dim3(256), 0, st, act_i8, scales, m, a->k_pad, a->q,
                               a->x_scales, a->x_sums, a->x_scales_t, a->xt_pitch);
    if (e != cudaSuccess) return fail_cuda(e, "act_from_i8_kernel");
    a->m = m;
    return JKB_OK;
}

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_quantize_row_q8_0_f32(const float *x, size_t x_len, jkb_block_q8_0 *out, size_t out_len,
                              void *stream) {
    int rc = validate_act("quantize_row_q8_0_f32", x_len, out_len, 32);
    if (rc) return rc;
    if (!x || !out) return fail(JKB_E_INVALID, "quantize_row_q8_0_f32", 0, 0, 0, "null pointer");
    return launch_q8_0(x, out_len, out, as_stream(stream));
}

int jkb_quantize_row_f32_to_q8_32(const float *input, size_t in_len, int8_t *out_quants,
                                  size_t q_len, float *out_scales, size_t scales_len,
                                  float *out_sums, size_t sums_len, void *stream) {
    static const char *fn = "quantize_row_f32_to_q8_32";
    // validate_q8_row_buffers (repack.rs:336-365)
    if (in_len == 0)
        return fail(JKB_E_BOUNDS, fn, 0, 0, 0, "activation slice must be non-empty");
    const size_t blocks = (in_len + 31) / 32, req = blocks * 32;
    if (q_len < req || scales_len < blocks || sums_len < blocks)
        return fail(JKB_E_BOUNDS, fn, 0, req, q_len,
                    "insufficient Q8 output buffers: quants=%zu/%zu, scales=%zu/%zu, sums=%zu/%zu",
                    q_len, req, scales_len, blocks, sums_len, blocks);
    if (!input || !out_quants || !out_scales || !out_sums)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    int rc;
    if ((rc = check_align(input, 4, fn, "input")) ||
        (rc = check_align(out_scales, 4, fn, "out_scales")) ||
        (rc = check_align(out_sums, 4, fn, "out_sums")))
        return rc;
    cudaError_t e = launch_pdl(q8_32_row_kernel, dim3((unsigned)((blocks + 255) / 256)),
                               dim3(256), 0, as_stream(stream), input, in_len, out_quants,
                               out_scales, out_sums);
    return e == cudaSuccess ? JKB_OK : fail_cuda(e, "q8_32_row_kernel");
}

int jkb_quantize_row_q8_0(const float *x, size_t x_len, jkb_block_q8_0 *out, size_t out_len,
                          void *stream) {
    return jkb_quantize_row_q8_0_f32(x, x_len, out, out_len, stream);
}

int jkb_quantize_row_q8_k(const float *x, size_t x_len, jkb_block_q8_k *out, size_t out_len,
                          void *stream) {
    int rc = validate_act("quantize_row_q8_k", x_len, out_len, 256);
    if (rc) return rc;
    if (!x || !out) return fail(JKB_E_INVALID, "quantize_row_q8_k", 0, 0, 0, "null pointer");
    return launch_q8_k(x, out_len, out, as_stream(stream));
}

int jkb_quantize_rows_q8_0(const float *x, size_t m, size_t k, jkb_block_q8_0 *out,
                           size_t out_len, void *stream) {
    if (m == 0) return fail(JKB_E_BOUNDS, "quantize_rows_q8_0", 0, 0, out_len, "m must be > 0");
    int rc = validate_act("quantize_row_q8_0_f32", k, out_len / m, 32);
    if (rc) return rc;
    if (out_len != m * (k / 32))
        return fail(JKB_E_BOUNDS, "quantize_rows_q8_0", 0, m * k * 4, out_len,
                    "output block count %zu != expected %zu", out_len, m * (k / 32));
    if (!x || !out) return fail(JKB_E_INVALID, "quantize_rows_q8_0", 0, 0, 0, "null pointer");
    return launch_q8_0(x, out_len, out, as_stream(stream));
}

int jkb_quantize_rows_q8_k(const float *x, size_t m, size_t k, jkb_block_q8_k *out,
                           size_t out_len, void *stream) {
    if (m == 0) return fail(JKB_E_BOUNDS, "quantize_rows_q8_k", 0, 0, out_len, "m must be > 0");
    int rc = validate_act("quantize_row_q8_k", k, out_len / m, 256);
    if (rc) return rc;
    if (out_len != m * (k / 256))
        return fail(JKB_E_BOUNDS, "quantize_rows_q8_k", 0, m * k * 4, out_len,
                    "output block count %zu != expected %zu", out_len, m * (k / 256));
    if (!x || !out) return fail(JKB_E_INVALID, "quantize_rows_q8_k", 0, 0, 0, "null pointer");
    return launch_q8_k(x, out_len, out, as_stream(stream));
}

int jkb_subln_quantize_absmax_i8_rows(int8_t *out_i8, const float *input,
                                      const float *norm_weight, size_t m, size_t len, float eps,
                                      float *scales_out, void *stream) {
    if (len == 0 || m == 0)
        return fail(JKB_E_BOUNDS, "subln", 0, 0, len * 4,
                    "dimension mismatch: input=%zu, rows=%zu", len, m);
    if (!out_i8 || !input || !norm_weight || !scales_out)
        return fail(JKB_E_INVALID, "subln", 0, 0, 0, "null pointer");
    int rc;
    if ((rc = check_align(input, 4, "subln", "input")) ||
        (rc = check_align(norm_weight, 4, "subln", "norm_weight")) ||
        (rc = check_align(scales_out, 4, "subln", "scale")))
        return rc;
    if (len > SUBLN_MAX_LEN)
        return fail(JKB_E_BOUNDS, "subln", 0, len, SUBLN_MAX_LEN,
                    "row length %zu exceeds the %zu-element limit of the GPU kernel", len,
                    SUBLN_MAX_LEN);
    return launch_subln(false, out_i8, nullptr, input, nullptr, norm_weight, m, len, eps,
                        scales_out, as_stream(stream));
}

int jkb_relu_squared_gate_f32(float *out, size_t out_len, const float *gate, size_t gate_len,
                              const float *up, size_t up_len, void *stream) {
    if (gate_len == 0 || out_len != gate_len || up_len != gate_len)
        return fail(JKB_E_BOUNDS, "relu_squared", 0, out_len * 4, gate_len * 4,
                    "dimension mismatch: gate=%zu, up=%zu, out=%zu", gate_len, up_len, out_len);
    if (!out || !gate || !up) return fail(JKB_E_INVALID, "relu_squared", 0, 0, 0, "null pointer");
    int rc;
    if ((rc = check_align(out, 4, "relu_squared", "out")) ||
        (rc = check_align(gate, 4, "relu_squared", "gate")) ||
        (rc = check_align(up, 4, "relu_squared", "up")))
        return rc;
    size_t grid = (gate_len + 255) / 256;
    const size_t cap = (size_t)num_sms() * 8;
    if (grid > cap) grid = cap;
    cudaError_t e = launch_pdl(relu_squared_kernel, dim3((unsigned)grid), dim3(256), 0,
                               as_stream(stream), gate, up, gate_len, out);
    return e == cudaSuccess ? JKB_OK : fail_cuda(e, "relu_squared_kernel");
}

int jkb_relu_squared_subln_quantize_i8_rows(int8_t *out_i8, float *relu_out, const float *gate,
                                            const float *up, const float *norm_weight, size_t m,
                                            size_t len, float eps, float *scales_out,
                                            void *stream) {
    if (len == 0 || m == 0)
        return fail(JKB_E_BOUNDS, "subln", 0, 0, len * 4,
                    "dimension mismatch: input=%zu, rows=%zu", len, m);
    if (!out_i8 || !gate || !up || !norm_weight || !scales_out)
        return fail(JKB_E_INVALID, "subln", 0, 0, 0, "null pointer");
    int rc;
    if ((rc = check_align(gate, 4, "relu_squared", "gate")) ||
        (rc = check_align(up, 4, "relu_squared", "up")) ||
        (relu_out && (rc = check_align(relu_out, 4, "relu_squared", "out"))) ||
        (rc = check_align(norm_weight, 4, "subln", "norm_weight")) ||
        (rc = check_align(scales_out, 4, "subln", "scale")))
        return rc;
    if (len > SUBLN_MAX_LEN)
        return fail(JKB_E_BOUNDS, "subln", 0, len, SUBLN_MAX_LEN,
                    "row length %zu exceeds the %zu-element limit of the GPU kernel", len,
                    SUBLN_MAX_LEN);
    return launch_subln(true, out_i8, relu_out, gate, up, norm_weight, m, len, eps, scales_out,
                        as_stream(stream));
}

int jkb_subln_quantize_absmax_i8(int8_t *out_i8, size_t out_len, const float *input,
                                 size_t in_len, const float *norm_weight, size_t w_len, float eps,
                                 float *scale_out, void *stream) {
    if (in_len == 0 || out_len != in_len || w_len != in_len)
        return fail(JKB_E_BOUNDS, "subln", 0, out_len, in_len * 4,
                    "dimension mismatch: input=%zu, out_i8=%zu, norm_weight=%zu", in_len,
                    out_len, w_len);
    return jkb_subln_quantize_absmax_i8_rows(out_i8, input, norm_weight, 1, in_len, eps,
                                             scale_out, stream);
}

int jkb_act_q8_create(size_t m_capacity, size_t k, jkb_act_q8 **out) {
    if (!out) return fail(JKB_E_INVALID, "QuantizedActQ8", 0, 0, 0, "null out");
    *out = nullptr;
    if (m_capacity == 0 || k == 0)
        return fail(JKB_E_BOUNDS, "QuantizedActQ8", 0, 0, 0,
                    "capacity must be non-zero, got m=%zu k=%zu", m_capacity, k);
    jkb_act_q8 *a = new jkb_act_q8();
    memset(a, 0, sizeof(*a));
    a->magic = ACT_MAGIC;
    a->m_cap = m_capacity;
    a->k = k;
    a->k_pad = (k + 31) / 32 * 32;
    size_t kb = a->k_pad / 32, kc = a->k_pad / 16, nsb = (k + 255) / 256;
    Arena ar;
    a->xt_pitch = (m_capacity + 31) / 32 * 32;
    size_t qb = m_capacity * a->k_pad, fb = m_capacity * kb * 4, f16b = m_capacity * kc * 4,
           sb = m_capacity * nsb * 4, tb = a->xt_pitch * kb * 4;
    ar.cap = Arena::round(qb) + 2 * Arena::round(fb) + Arena::round(f16b) + Arena::round(sb) +
             2 * Arena::round(tb) + Arena::round(2 * tb);
    cudaError_t e = cudaMalloc(&ar.base, ar.cap);
    if (e != cudaSuccess) {
        delete a;
        return fail_cuda(e, "jkb_act_q8_create");
    }
    a->base = ar.base;
    a->q = (int8_t *)ar.take(qb);
    a->x_scales = (float *)ar.take(fb);
    a->x_sums = (float *)ar.take(fb);
    a->x_sums_16 = (float *)ar.take(f16b);
    a->super_scales = (float *)ar.take(sb);
    a->x_scales_t = (float *)ar.take(tb);
    a->x_nsums_t = (float *)ar.take(tb);
    a->x_nsums16_t = (float *)ar.take(2 * tb);
    *out = a;
    return JKB_OK;
}

int jkb_act_q8_destroy(jkb_act_q8 *a) {
    if (!check_act(a)) return fail(JKB_E_INVALID, "QuantizedActQ8", 0, 0, 0, "null or destroyed");
    a->magic = 0;
    cudaFree(a->base);
    delete a;
    return JKB_OK;
}

int jkb_act_q8_quantize(jkb_act_q8 *a, const float *input, size_t in_len, size_t m, size_t k,
                        void *stream) {
    if (!check_act(a)) return fail(JKB_E_INVALID, "QuantizedActQ8", 0, 0, 0, "null or destroyed");
    // QuantizedActQ8::quantize_into validation (repack.rs:547-560)
    if (m == 0 || k == 0 || in_len != m * k)
        return fail(JKB_E_BOUNDS, "QuantizedActQ8", 0, in_len * 4, m * k * 4,
                    "activation length %zu does not match m (%zu) * k (%zu)", in_len, m, k);
    if (k != a->k || m > a->m_cap)
        return fail(JKB_E_BOUNDS, "QuantizedActQ8", 0, in_len * 4, a->m_cap * a->k * 4,
                    "batch [%zu, %zu] exceeds the handle capacity [%zu, %zu]", m, k, a->m_cap,
                    a->k);
    if (!input) return fail(JKB_E_INVALID, "QuantizedActQ8", 0, 0, 0, "null input");
    int arc = check_align(input, 4, "QuantizedActQ8", "input");
    if (arc) return arc;
    cudaStream_t st = as_stream(stream);
    size_t kb = a->k_pad / 32, nsb = (k + 255) / 256;
    size_t n = (a->x_scales_t ? (m + 31) / 32 * 32 : m) * kb;
    act_q8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(input, m, k, a->k_pad, a->q,
                                                               a->x_scales, a->x_sums,
                                                               a->x_sums_16, a->x_scales_t,
                                                               a->x_nsums_t, a->x_nsums16_t,
                                                               a->xt_pitch);
    int rc = check_launch("act_q8_kernel");
    if (rc) return rc;
    size_t ns = m * nsb;
    act_super_kernel<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(a->x_scales, m, kb, nsb,
                                                                   a->super_scales);
    rc = check_launch("act_super_kernel");
    if (rc) return rc;
    a->m = m;
    return JKB_OK;
}

int jkb_act_q8_buffers(const jkb_act_q8 *a, size_t *m, size_t *k, size_t *k_padded, int8_t **q,
                       float **x_scales, float **x_sums, float **x_sums_16,
                       float **super_scales) {
    if (!check_act(a)) return fail(JKB_E_INVALID, "QuantizedActQ8", 0, 0, 0, "null or destroyed");
    if (m) *m = a->m;
    if (k) *k = a->k;
    if (k_padded) *k_padded = a->k_pad;
    if (q) *q = a->q;
    if (x_scales) *x_scales = a->x_scales;
    if (x_sums) *x_sums = a->x_sums;
    if (x_sums_16) *x_sums_16 = a->x_sums_16;
    if (super_scales) *super_scales = a->super_scales;
    return JKB_OK;
}

}  // extern "C"
