// Memory-bound decode GEMV / BitLinear kernels over the jkb_weight GPU layout.
//
// One warp per weight row (persistent CTAs of 8 warps stride over rows); lane l of the warp
// owns the 16-byte quant chunks l, l+32, l+64, ... of the row, so every warp-wide load reads
// 512 contiguous bytes. A block's chunks sit on CPB consecutive lanes; each lane forms exact
// integer partial sums with dp4a against the activation staged in shared memory, the CPB lanes
// add them with xor-shuffles (integer, so the per-block sums are the reference's bit for bit),
// and the block's first lane applies the reference's f32 block formula with separately rounded
// multiplies (__fmul_rn/__fsub_rn). Only the final f32 sum over a row's blocks runs in a
// different order than the reference's sequential row loop.
//
// Activation staging (shared memory, per CTA and token):
//   BlockQ8K rows: xq i8[K] | xd f32[K/256] | bsums i16[K/16]
//   BlockQ8_0 rows: xq i8[K] | xd f32[K/32] | block sums i32[K/32]
//   i8 rows (BitLinear): xq i8[K] | 16-element sums i32[K/16]
#include <cstdio>

#include "jkb_internal.h"

namespace jkb {

struct KArgs {
    const uint8_t *qs;
    size_t qs_row;
    const uint8_t *sc;
    size_t sc_row;
    const uint16_t *d;
    const uint8_t *x;
    size_t x_row_stride;
    const float *act_scales;
    float act_scale;
    float i2s_scale;
    float *out;
    size_t out_ld;
    size_t row_begin, row_end;
    int nb;  // blocks per row
    int K;
    int32_t *dbg_sumi, *dbg_mins;
    float *dbg_val;
};

// ---------------------------------------------------------------- device helpers

__device__ __forceinline__ uint4 ldg_stream(const uint8_t *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream2(const uint8_t *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg_u16(const uint16_t *p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }
// unsigned bytes of a times signed bytes of b
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// f16_to_f32_finite (lib.rs:714-717): exact conversion, NaN/Inf -> 0.
__device__ __forceinline__ float f16_finite(uint32_t bits) {
    float v = __half2float(__ushort_as_half((unsigned short)bits));
    return ((bits >> 10) & 0x1F) == 0x1F ? 0.0f : v;
}
__device__ __forceinline__ int4 lds_v4(const int8_t *p) {
    return *reinterpret_cast<const int4 *>(p);
}

// ---------------------------------------------------------------- activation staging

struct ActQ8K {
    static __host__ __device__ size_t bytes(int K) { return ((size_t)K + 15) / 16 * 16 + K / 256 * 4 + K / 16 * 2 + 16; }
    static __device__ __forceinline__ const int8_t *xq(const uint8_t *s) { return (const int8_t *)s; }
    static __device__ __forceinline__ const float *xd(const uint8_t *s, int K) {
        return (const float *)(s + (K + 15) / 16 * 16);
    }
    static __device__ __forceinline__ const int16_t *bs(const uint8_t *s, int K) {
        return (const int16_t *)(s + (K + 15) / 16 * 16 + K / 256 * 4);
    }
    static __device__ void stage(const KArgs &a, const uint8_t *x, uint8_t *s) {
        const int nb = a.K / 256;
        const int total = nb * 73;  // 292-byte BlockQ8K = 73 words
        uint32_t *q = (uint32_t *)s;
        float *xd_ = (float *)xd(s, a.K);
        uint32_t *bs_ = (uint32_t *)bs(s, a.K);
        for (int i = threadIdx.x; i < total; i += blockDim.x) {
            int blk = i / 73, w = i - blk * 73;
            uint32_t v = __ldg(reinterpret_cast<const uint32_t *>(x + (size_t)blk * 292) + w);
            if (w == 0)
                xd_[blk] = __uint_as_float(v);
            else if (w <= 64)
                q[blk * 64 + (w - 1)] = v;
            else
                bs_[blk * 8 + (w - 65)] = v;
        }
        __syncthreads();
    }
};

struct ActQ80 {
    static __host__ __device__ size_t bytes(int K) { return ((size_t)K + 15) / 16 * 16 + K / 32 * 8 + 16; }
    static __device__ __forceinline__ const int8_t *xq(const uint8_t *s) { return (const int8_t *)s; }
    static __device__ __forceinline__ const float *xd(const uint8_t *s, int K) {
        return (const float *)(s + (K + 15) / 16 * 16);
    }
    static __device__ __forceinline__ const int *xs(const uint8_t *s, int K) {
        return (const int *)(s + (K + 15) / 16 * 16 + K / 32 * 4);
    }
    static __device__ void stage(const KArgs &a, const uint8_t *x, uint8_t *s) {
        const int nb = a.K / 32;
        const int total = nb * 9;  // 36-byte BlockQ8_0 = 9 words
        uint32_t *q = (uint32_t *)s;
        float *xd_ = (float *)xd(s, a.K);
        for (int i = threadIdx.x; i < total; i += blockDim.x) {
            int blk = i / 9, w = i - blk * 9;
            uint32_t v = __ldg(reinterpret_cast<const uint32_t *>(x + (size_t)blk * 36) + w);
            if (w == 0)
                xd_[blk] = __uint_as_float(v);
            else
                q[blk * 8 + (w - 1)] = v;
        }
        __syncthreads();
        int *xs_ = (int *)xs(s, a.K);
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            int t = 0;
#pragma unroll
            for (int w = 0; w < 8; w++) t = __dp4a((int)q[b * 8 + w], 0x01010101, t);
            xs_[b] = t;
        }
        __syncthreads();
    }
};

struct ActI8 {
    static __host__ __device__ size_t bytes(int K) { return ((size_t)K + 15) / 16 * 16 + K / 16 * 4 + 16; }
    static __device__ __forceinline__ const int8_t *xq(const uint8_t *s) { return (const int8_t *)s; }
    static __device__ __forceinline__ const int *g16(const uint8_t *s, int K) {
        return (const int *)(s + (K + 15) / 16 * 16);
    }
    static __device__ void stage(const KArgs &a, const uint8_t *x, uint8_t *s) {
        if ((((uintptr_t)x) & 15) == 0) {
            const int nv = a.K / 16;
            for (int i = threadIdx.x; i < nv; i += blockDim.x)
                reinterpret_cast<uint4 *>(s)[i] = __ldg(reinterpret_cast<const uint4 *>(x) + i);
        } else {
            for (int i = threadIdx.x; i < a.K; i += blockDim.x) s[i] = x[i];
        }
        __syncthreads();
        int *g = (int *)g16(s, a.K);
        const uint32_t *q = (const uint32_t *)s;
        for (int j = threadIdx.x; j < a.K / 16; j += blockDim.x) {
            int t = 0;
#pragma unroll
            for (int w = 0; w < 4; w++) t = __dp4a((int)q[j * 4 + w], 0x01010101, t);
            g[j] = t;
        }
        __syncthreads();
    }
};

// ---------------------------------------------------------------- formats
// Each format: CPB lanes per block (16-byte chunks per block), MINS (second integer sum),
// Ld (per-chunk registers), load(), dot() -> partial integer sums, finish() -> block value.

struct LdW {
    uint4 w;
    uint32_t d;
};

// Q4_0 x Q8_0 (quant_q8.rs:672-684)
struct FQ4_0 {
    static constexpr int CPB = 1;
    static constexpr bool MINS = false;
    using Act = ActQ80;
    using Ld = LdW;
    static __device__ __forceinline__ Ld load(const KArgs &a, size_t row, int q) {
        Ld l;
        l.w = ldg_stream(a.qs + row * a.qs_row + 16 * (size_t)q);
        l.d = ldg_u16(a.d + row * a.nb + q);
        return l;
    }
    static __device__ __forceinline__ int2 dot(const KArgs &a, const uint8_t *s, const Ld &l, int q) {
        const int8_t *x = Act::xq(s) + 32 * q;
        int4 xl = lds_v4(x), xh = lds_v4(x + 16);
        int lo = 0, hi = 0;
        lo = dp4a_ss(l.w.x & 0x0F0F0F0F, xl.x, lo);
        lo = dp4a_ss(l.w.y & 0x0F0F0F0F, xl.y, lo);
        lo = dp4a_ss(l.w.z & 0x0F0F0F0F, xl.z, lo);
        lo = dp4a_ss(l.w.w & 0x0F0F0F0F, xl.w, lo);
        hi = dp4a_us(l.w.x & 0xF0F0F0F0u, xh.x, hi);
        hi = dp4a_us(l.w.y & 0xF0F0F0F0u, xh.y, hi);
        hi = dp4a_us(l.w.z & 0xF0F0F0F0u, xh.z, hi);
        hi = dp4a_us(l.w.w & 0xF0F0F0F0u, xh.w, hi);
        // sum (n - 8) * x = sum n * x - 8 * sum x; the high nibbles were kept in place (x16).
        return make_int2(lo + (hi >> 4) - 8 * Act::xs(s, a.K)[q], 0);
    }
    static __device__ __forceinline__ float finish(const KArgs &a, const uint8_t *s, const Ld &l,
                                                   int b, int2 v) {
        float dw = f16_finite(l.d), xd = Act::xd(s, a.K)[b];
        if (dw == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn((float)v.x, __fmul_rn(dw, xd));
    }
};

// Q8_0 x Q8_0 (quant_q8.rs:707-717); also the Q8_0 BitLinear weight (ime.rs:840-853).
template <class A>
struct FQ8_0 {
    static constexpr int CPB = 2;
    static constexpr bool MINS = false;
    using Act = A;
    using Ld = LdW;
    static __device__ __forceinline__ Ld load(const KArgs &a, size_t row, int q) {
        Ld l;
        l.w = ldg_stream(a.qs + row * a.qs_row + 16 * (size_t)q);
        l.d = ldg_u16(a.d + row * a.nb + (q >> 1));
        return l;
    }
    static __device__ __forceinline__ int2 dot(const KArgs &a, const uint8_t *s, const Ld &l, int q) {
        int4 x = lds_v4(Act::xq(s) + 16 * q);
        int t = 0;
        t = dp4a_ss((int)l.w.x, x.x, t);
        t = dp4a_ss((int)l.w.y, x.y, t);
        t = dp4a_ss((int)l.w.z, x.z, t);
        t = dp4a_ss((int)l.w.w, x.w, t);
        return make_int2(t, 0);
    }
    static __device__ __forceinline__ float finish(const KArgs &a, const uint8_t *s, const Ld &l,
                                                   int b, int2 v);
};
template <>
__device__ __forceinline__ float FQ8_0<ActQ80>::finish(const KArgs &a, const uint8_t *s,
                                                        const Ld &l, int b, int2 v) {
    float dw = f16_finite(l.d), xd = ActQ80::xd(s, a.K)[b];
    if (dw == 0.0f || xd == 0.0f) return 0.0f;
    return __fmul_rn((float)v.x, __fmul_rn(dw, xd));
}
// BitLinear (ime.rs:918-929): (f32)dot * (block_scale * act_scale), no zero shortcut.
template <>
__device__ __forceinline__ float FQ8_0<ActI8>::finish(const KArgs &a, const uint8_t *s,
                                                       const Ld &l, int b, int2 v) {
    return __fmul_rn((float)v.x, __fmul_rn(f16_finite(l.d), a.act_scale));
}

// Q4_K x Q8_K (quant_q8.rs:1834-1862). Chunk q: superblock q/8, part p = q%8 covers
// qs[16p..16p+16] of the superblock = chunk c = p/2, half h = p%2: low nibbles pair with
// x[64c+16h..], high nibbles with x[64c+32+16h..]; sub-block scales 2c and 2c+1.
struct FQ4_K {
    static constexpr int CPB = 8;
    static constexpr bool MINS = true;
    using Act = ActQ8K;
    struct Ld {
        uint4 w, s;
    };
    static __device__ __forceinline__ Ld load(const KArgs &a, size_t row, int q) {
        Ld l;
        l.w = ldg_stream(a.qs + row * a.qs_row + 16 * (size_t)q);
        l.s = __ldg(reinterpret_cast<const uint4 *>(a.sc + row * a.sc_row + 16 * (size_t)(q >> 3)));
        return l;
    }
    static __device__ __forceinline__ int2 dot(const KArgs &a, const uint8_t *s, const Ld &l, int q) {
        const int sb = q >> 3, p = q & 7, c = p >> 1, h = p & 1;
        const int8_t *x = Act::xq(s) + 256 * sb + 64 * c + 16 * h;
        int4 xl = lds_v4(x), xh = lds_v4(x + 32);
        int lo = 0, hi = 0;
        lo = dp4a_ss(l.w.x & 0x0F0F0F0F, xl.x, lo);
        lo = dp4a_ss(l.w.y & 0x0F0F0F0F, xl.y, lo);
        lo = dp4a_ss(l.w.z & 0x0F0F0F0F, xl.z, lo);
        lo = dp4a_ss(l.w.w & 0x0F0F0F0F, xl.w, lo);
        hi = dp4a_us(l.w.x & 0xF0F0F0F0u, xh.x, hi);
        hi = dp4a_us(l.w.y & 0xF0F0F0F0u, xh.y, hi);
        hi = dp4a_us(l.w.z & 0xF0F0F0F0u, xh.z, hi);
        hi = dp4a_us(l.w.w & 0xF0F0F0F0u, xh.w, hi);
        hi >>= 4;
        // 6-bit scales/mins j = 2c, 2c+1 (unpack_q4_q5_k_scales_mins, quant_q8.rs:1817-1830)
        const int sh = 16 * (c & 1);
        uint32_t scp, mp;
        if (c < 2) {
            scp = (l.s.y >> sh) & 0x3F3F;
            mp = (l.s.z >> sh) & 0x3F3F;
        } else {
            scp = ((l.s.w >> sh) & 0x0F0F) | (((l.s.y >> sh) >> 2) & 0x3030);
            mp = (((l.s.w >> sh) >> 4) & 0x0F0F) | (((l.s.z >> sh) >> 2) & 0x3030);
        }
        const int16_t *bs = Act::bs(s, a.K) + 16 * sb + 4 * c + h;
        int sumi = (int)(scp & 0xFF) * lo + (int)(scp >> 8) * hi;
        int mins = (int)(mp & 0xFF) * (int)bs[0] + (int)(mp >> 8) * (int)bs[2];
        return make_int2(sumi, mins);
    }
    static __device__ __forceinline__ float finish(const KArgs &a, const uint8_t *s, const Ld &l,
                                                   int b, int2 v) {
        float d = f16_finite(l.s.x & 0xFFFF), dmin = f16_finite(l.s.x >> 16);
        float xd = Act::xd(s, a.K)[b];
        if ((d == 0.0f && dmin == 0.0f) || xd == 0.0f) return 0.0f;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, xd), (float)v.x),
                         __fmul_rn(__fmul_rn(dmin, xd), (float)v.y));
    }
};

// Q6_K x Q8_K (quant_q8.rs:1903-1942). Chunk q: superblock q/4, item t = q%4 (h = t/2,
// i = t%2) holds 16 l-values: A = ql[64h+16i..], B = ql[64h+32+16i..], H = qh[32h+16i..];
// values (6-bit, unsigned) pair with x[128h+16i + 32*k] for k = 0..3 and scales
// sc[8h+i+2k]; the -32 offset is applied as -32 * bsum of the same 16 elements.
struct FQ6_K {
    static constexpr int CPB = 4;
    static constexpr bool MINS = false;
    using Act = ActQ8K;
    struct Ld {
        uint4 A, B, H;
        uint2 sc;
        uint32_t d;
    };
    static __device__ __forceinline__ Ld load(const KArgs &a, size_t row, int q) {
        const int sb = q >> 2, t = q & 3, h = t >> 1;
        const uint8_t *base = a.qs + row * a.qs_row + 192 * (size_t)sb + 16 * t;
        Ld l;
        l.A = ldg_stream(base);
        l.B = ldg_stream(base + 64);
        l.H = ldg_stream(base + 128);
        l.sc = __ldg(reinterpret_cast<const uint2 *>(a.sc + row * a.sc_row + 16 * (size_t)sb + 8 * h));
        l.d = ldg_u16(a.d + row * a.nb + sb);
        return l;
    }
    static __device__ __forceinline__ int dot16(uint4 A, uint4 B, uint4 H, const int8_t *x,
                                                int4 &S) {
        int4 x1 = lds_v4(x), x2 = lds_v4(x + 32), x3 = lds_v4(x + 64), x4 = lds_v4(x + 96);
        const uint32_t a_[4] = {A.x, A.y, A.z, A.w}, b_[4] = {B.x, B.y, B.z, B.w},
                       h_[4] = {H.x, H.y, H.z, H.w};
        const int x1_[4] = {x1.x, x1.y, x1.z, x1.w}, x2_[4] = {x2.x, x2.y, x2.z, x2.w},
                  x3_[4] = {x3.x, x3.y, x3.z, x3.w}, x4_[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t u1 = (a_[j] & 0x0F0F0F0F) | ((h_[j] << 4) & 0x30303030);
            uint32_t u2 = (b_[j] & 0x0F0F0F0F) | ((h_[j] << 2) & 0x30303030);
            uint32_t u3 = ((a_[j] >> 4) & 0x0F0F0F0F) | (h_[j] & 0x30303030);
            uint32_t u4 = ((b_[j] >> 4) & 0x0F0F0F0F) | ((h_[j] >> 2) & 0x30303030);
            S.x = dp4a_ss((int)u1, x1_[j], S.x);
            S.y = dp4a_ss((int)u2, x2_[j], S.y);
            S.z = dp4a_ss((int)u3, x3_[j], S.z);
            S.w = dp4a_ss((int)u4, x4_[j], S.w);
        }
        return 0;
    }
    static __device__ __forceinline__ int2 dot(const KArgs &a, const uint8_t *s, const Ld &l, int q) {
        const int sb = q >> 2, t = q & 3, h = t >> 1, i = t & 1;
        const int e0 = 256 * sb + 128 * h + 16 * i;
        int4 S = make_int4(0, 0, 0, 0);
        dot16(l.A, l.B, l.H, Act::xq(s) + e0, S);
        const int16_t *bs = Act::bs(s, a.K) + (e0 >> 4);
        const int sc0 = (int)(int8_t)(l.sc.x >> (8 * i)), sc1 = (int)(int8_t)(l.sc.x >> (8 * i + 16));
        const int sc2 = (int)(int8_t)(l.sc.y >> (8 * i)), sc3 = (int)(int8_t)(l.sc.y >> (8 * i + 16));
        int sumi = sc0 * (S.x - 32 * (int)bs[0]) + sc1 * (S.y - 32 * (int)bs[2]) +
                   sc2 * (S.z - 32 * (int)bs[4]) + sc3 * (S.w - 32 * (int)bs[6]);
        return make_int2(sumi, 0);
    }
    static __device__ __forceinline__ float finish(const KArgs &a, const uint8_t *s, const Ld &l,
                                                   int b, int2 v) {
        float d = f16_finite(l.d), xd = Act::xd(s, a.K)[b];
        if (d == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn(__fmul_rn(d, xd), (float)v.x);
    }
};

// TQ2_0 x Q8_K (quant_q8.rs:1992-2003) and TQ2_0/TQ1_0 BitLinear (ime.rs:918-929). Chunk q
// covers elements 64q..64q+63 of the row; in the GPU layout word W, bit pair j, byte b holds
// the 2-bit code of element 64q + 16W + 4j + b, so (w >> 2j) & 0x03030303 lines up with four
// consecutive activations. Codes are value + 1; the +1 is removed as -sum(x).
template <class A>
struct FTQ2 {
    static constexpr int CPB = 4;
    static constexpr bool MINS = false;
    using Act = A;
    using Ld = LdW;
    static __device__ __forceinline__ Ld load(const KArgs &a, size_t row, int q) {
        Ld l;
        l.w = ldg_stream(a.qs + row * a.qs_row + 16 * (size_t)q);
        l.d = ldg_u16(a.d + row * a.nb + (q >> 2));
        return l;
    }
    static __device__ __forceinline__ int sum_codes(const Ld &l, const int8_t *x) {
        const uint32_t w_[4] = {l.w.x, l.w.y, l.w.z, l.w.w};
        int t = 0;
#pragma unroll
        for (int W = 0; W < 4; W++) {
            int4 xv = lds_v4(x + 16 * W);
            t = dp4a_ss((int)(w_[W] & 0x03030303), xv.x, t);
            t = dp4a_ss((int)((w_[W] >> 2) & 0x03030303), xv.y, t);
            t = dp4a_ss((int)((w_[W] >> 4) & 0x03030303), xv.z, t);
            t = dp4a_ss((int)((w_[W] >> 6) & 0x03030303), xv.w, t);
        }
        return t;
    }
    static __device__ __forceinline__ int2 dot(const KArgs &a, const uint8_t *s, const Ld &l, int q);
    static __device__ __forceinline__ float finish(const KArgs &a, const uint8_t *s, const Ld &l,
                                                   int b, int2 v);
};
template <>
__device__ __forceinline__ int2 FTQ2<ActQ8K>::dot(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int q) {
    int t = sum_codes(l, ActQ8K::xq(s) + 64 * q);
    const int16_t *bs = ActQ8K::bs(s, a.K) + 4 * q;
    return make_int2(t - ((int)bs[0] + (int)bs[1] + (int)bs[2] + (int)bs[3]), 0);
}
template <>
__device__ __forceinline__ float FTQ2<ActQ8K>::finish(const KArgs &a, const uint8_t *s,
                                                      const Ld &l, int b, int2 v) {
    float xd = ActQ8K::xd(s, a.K)[b];
    float dw = f16_finite(l.d);
    if (xd == 0.0f || dw == 0.0f) return 0.0f;
    return __fmul_rn((float)v.x, __fmul_rn(dw, xd));
}
template <>
__device__ __forceinline__ int2 FTQ2<ActI8>::dot(const KArgs &a, const uint8_t *s, const Ld &l,
                                                 int q) {
    int t = sum_codes(l, ActI8::xq(s) + 64 * q);
    const int *g = ActI8::g16(s, a.K) + 4 * q;
    return make_int2(t - (g[0] + g[1] + g[2] + g[3]), 0);
}
template <>
__device__ __forceinline__ float FTQ2<ActI8>::finish(const KArgs &a, const uint8_t *s,
                                                     const Ld &l, int b, int2 v) {
    return __fmul_rn((float)v.x, __fmul_rn(f16_finite(l.d), a.act_scale));
}

// I2_S BitLinear (quant.rs:370-377, ime.rs:918-929). Chunk q = half h of block q/2: byte g in
// [16h, 16h+16) carries elements g, 32+g, 64+g, 96+g in bits [7:6], [5:4], [3:2], [1:0].
struct FI2S {
    static constexpr int CPB = 2;
    static constexpr bool MINS = false;
    using Act = ActI8;
    struct Ld {
        uint4 w;
    };
    static __device__ __forceinline__ Ld load(const KArgs &a, size_t row, int q) {
        Ld l;
        l.w = ldg_stream(a.qs + row * a.qs_row + 16 * (size_t)q);
        return l;
    }
    static __device__ __forceinline__ int2 dot(const KArgs &a, const uint8_t *s, const Ld &l, int q) {
        const int b = q >> 1, h = q & 1;
        const int8_t *x = Act::xq(s) + 128 * b + 16 * h;
        int4 x0 = lds_v4(x), x1 = lds_v4(x + 32), x2 = lds_v4(x + 64), x3 = lds_v4(x + 96);
        const uint32_t w_[4] = {l.w.x, l.w.y, l.w.z, l.w.w};
        const int x0_[4] = {x0.x, x0.y, x0.z, x0.w}, x1_[4] = {x1.x, x1.y, x1.z, x1.w},
                  x2_[4] = {x2.x, x2.y, x2.z, x2.w}, x3_[4] = {x3.x, x3.y, x3.z, x3.w};
        int t = 0;
#pragma unroll
        for (int W = 0; W < 4; W++) {
            t = dp4a_ss((int)((w_[W] >> 6) & 0x03030303), x0_[W], t);
            t = dp4a_ss((int)((w_[W] >> 4) & 0x03030303), x1_[W], t);
            t = dp4a_ss((int)((w_[W] >> 2) & 0x03030303), x2_[W], t);
            t = dp4a_ss((int)(w_[W] & 0x03030303), x3_[W], t);
        }
        const int *g = Act::g16(s, a.K) + 8 * b + h;
        return make_int2(t - (g[0] + g[2] + g[4] + g[6]), 0);
    }
    static __device__ __forceinline__ float finish(const KArgs &a, const uint8_t *s, const Ld &l,
                                                   int b, int2 v) {
        return __fmul_rn((float)v.x, __fmul_rn(a.i2s_scale, a.act_scale));
    }
};

// ---------------------------------------------------------------- the kernel

constexpr int WARPS = 8;

template <class F, int U, bool DIAG>
__global__ void __launch_bounds__(WARPS * 32, 2) gemv_kernel(KArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int tok = blockIdx.y;
    KArgs args = a;
    if (a.act_scales) args.act_scale = a.act_scales[tok];
    F::Act::stage(args, a.x + (size_t)tok * a.x_row_stride, smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunks = a.nb * F::CPB;
    float *out = a.out + (size_t)tok * a.out_ld;
    for (size_t row = a.row_begin + (size_t)blockIdx.x * WARPS + warp; row < a.row_end;
         row += (size_t)gridDim.x * WARPS) {
        float acc = 0.0f;
        for (int base = 0; base < nchunks; base += 32 * U) {
            typename F::Ld ld[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                int q = base + 32 * u + lane;
                if (q < nchunks) ld[u] = F::load(args, row, q);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int q = base + 32 * u + lane;
                const bool valid = q < nchunks;
                if (base + 32 * u >= nchunks) break;  // warp-uniform
                int2 v = valid ? F::dot(args, smem, ld[u], q) : make_int2(0, 0);
#pragma unroll
                for (int m = 1; m < F::CPB; m <<= 1) {
                    v.x += __shfl_xor_sync(0xffffffffu, v.x, m);
                    if (F::MINS) v.y += __shfl_xor_sync(0xffffffffu, v.y, m);
                }
                if (valid && (q % F::CPB) == 0) {
                    const int b = q / F::CPB;
                    float val = F::finish(args, smem, ld[u], b, v);
                    if (DIAG) {
                        size_t o = (row - a.row_begin) * (size_t)a.nb + b;
                        a.dbg_sumi[o] = v.x;
                        if (a.dbg_mins) a.dbg_mins[o] = v.y;
                        a.dbg_val[o] = val;
                    } else {
                        acc = __fadd_rn(acc, val);
                    }
                }
            }
        }
        if (!DIAG) {
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
            if (lane == 0) out[row - a.row_begin] = acc;
        }
    }
}

// ---------------------------------------------------------------- launch

template <class F, int U, bool DIAG>
static int launch_t(const KArgs &a, size_t m, cudaStream_t st, const char *name) {
    const size_t smem = F::Act::bytes(a.K);
    auto kern = gemv_kernel<F, U, DIAG>;
    static int occ = -1;  // per template instance; the device set is homogeneous (B200)
    if (occ < 0) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        occ = 0;
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, WARPS * 32, smem);
    if (per_sm < 1) per_sm = 1;
    size_t rows = a.row_end - a.row_begin;
    size_t want = (rows + WARPS - 1) / WARPS;
    size_t cap = (size_t)num_sms() * per_sm;
    size_t gx = want;
    if (m * gx > cap) gx = (cap + m - 1) / m;
    if (gx < 1) gx = 1;
    dim3 grid((unsigned)gx, (unsigned)m);
    kern<<<grid, WARPS * 32, smem, st>>>(a);
    return check_launch(name);
}

static size_t smem_limit_k(int act_kind) {
    // shared bytes per element ~1.2; keep well inside the 160 KiB opt-in set above
    (void)act_kind;
    return 120 * 1024;
}

int launch_gemv(const GemvLaunch &L, cudaStream_t st) {
    const jkb_weight *w = L.w;
    KArgs a;
    a.qs = w->p.qs;
    a.qs_row = w->p.qs_row;
    a.sc = w->p.sc;
    a.sc_row = w->p.sc_row;
    a.d = w->p.d;
    a.x = (const uint8_t *)L.x;
    a.x_row_stride = L.x_row_stride;
    a.act_scales = L.act_scales;
    a.act_scale = L.act_scale;
    a.i2s_scale = w->p.i2s_scale;
    a.out = L.out;
    a.out_ld = L.out_ld;
    a.row_begin = L.row_begin;
    a.row_end = L.row_end;
    a.nb = (int)w->nb;
    a.K = (int)w->cols;
    a.dbg_sumi = L.dbg_sumi;
    a.dbg_mins = L.dbg_mins;
    a.dbg_val = L.dbg_val;
    if (w->cols > smem_limit_k(L.act_kind))
        return fail(JKB_E_BOUNDS, w->name, w->offset, w->cols, smem_limit_k(L.act_kind),
                    "input length %zu exceeds the %zu-element activation limit of the GEMV "
                    "kernels",
                    w->cols, smem_limit_k(L.act_kind));
    if (L.row_end <= L.row_begin) return JKB_OK;
    const bool diag = L.dbg_sumi != nullptr;
    const size_t m = L.m ? L.m : 1;
#define JKB_LAUNCH(F, U)                                                                  \
    return diag ? launch_t<F, U, true>(a, m, st, "gemv_kernel<diag>")                     \
                : launch_t<F, U, false>(a, m, st, "gemv_kernel")
    switch (w->gpu_format) {
    case GF_Q4_0:
        if (L.act_kind == ACT_Q8_0) JKB_LAUNCH(FQ4_0, 4);
        break;
    case GF_Q8_0:
        if (L.act_kind == ACT_Q8_0) JKB_LAUNCH(FQ8_0<ActQ80>, 4);
        if (L.act_kind == ACT_I8) JKB_LAUNCH(FQ8_0<ActI8>, 4);
        break;
    case GF_Q4_K:
        if (L.act_kind == ACT_Q8_K) JKB_LAUNCH(FQ4_K, 4);
        break;
    case GF_Q6_K:
        if (L.act_kind == ACT_Q8_K) JKB_LAUNCH(FQ6_K, 2);
        break;
    case GF_TQ2_0:
        if (L.act_kind == ACT_Q8_K) JKB_LAUNCH(FTQ2<ActQ8K>, 4);
        if (L.act_kind == ACT_I8) JKB_LAUNCH(FTQ2<ActI8>, 4);
        break;
    case GF_I2_S:
        if (L.act_kind == ACT_I8) JKB_LAUNCH(FI2S, 4);
        break;
    }
#undef JKB_LAUNCH
    return fail(JKB_E_CAPABILITY, w->name, w->offset, w->byte_len, w->gguf_bytes,
                "no GEMV kernel for %s weights with activation kind %d", quant_name(w->quant),
                L.act_kind);
}

// ---------------------------------------------------------------- ABI glue

static int act_kind_for(int quant) {
    return (quant == JKB_Q4_0 || quant == JKB_Q8_0) ? ACT_Q8_0 : ACT_Q8_K;
}

// gemv_* validation order (quant_q8.rs:1586-1603 and twins): quant + shape validator, then
// check_q8_block_len (:1562-1578).
static int gemv_call(const char *fn, int quant, float *out, size_t out_len, const jkb_weight *w,
                     const void *x, size_t x_len, void *stream) {
    int rc = check_weight(w);
    if (rc) return rc;
    const Fmt *f = fmt_of(quant);
    size_t cols = x_len * (size_t)f->block_elems;
    rc = validate_weight_call(fn, w, quant, out_len, cols);
    if (rc) return rc;
    if (x_len != w->nb)
        return fail(JKB_E_BOUNDS, w->name, w->offset, x_len, w->nb,
                    "%s: x_blocks len %zu != expected %zu", fn, x_len, w->nb);
    if (!out || !x) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    if ((rc = check_align(out, 4, fn, "output")) || (rc = check_align(x, 4, fn, "x_blocks")))
        return rc;
    GemvLaunch L{};
    L.w = w;
    L.x = x;
    L.act_kind = act_kind_for(quant);
    L.out = out;
    L.row_begin = 0;
    L.row_end = w->rows;
    L.m = 1;
    return launch_gemv(L, as_stream(stream));
}

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_gemv_q4_0_q8_0(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_0 *x,
                       size_t x_len, void *stream) {
    return gemv_call("gemv_q4_0_q8_0", JKB_Q4_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_q4_0_q8_0_4x(float *out, size_t out_len, const jkb_weight *w,
                          const jkb_block_q8_0 *x, size_t x_len, void *stream) {
    return gemv_call("gemv_q4_0_q8_0", JKB_Q4_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_q8_0_q8_0(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_0 *x,
                       size_t x_len, void *stream) {
    return gemv_call("gemv_q8_0_q8_0", JKB_Q8_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_q8_0_q8_0_4x(float *out, size_t out_len, const jkb_weight *w,
                          const jkb_block_q8_0 *x, size_t x_len, void *stream) {
    return gemv_call("gemv_q8_0_q8_0", JKB_Q8_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_q4_k_q8_k(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_k *x,
                       size_t x_len, void *stream) {
    return gemv_call("gemv_q4_k_q8_k", JKB_Q4_K_M, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_q6_k_q8_k(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_k *x,
                       size_t x_len, void *stream) {
    return gemv_call("gemv_q6_k_q8_k", JKB_Q6_K, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_tq1_0_q8_k(float *out, size_t out_len, const jkb_weight *w,
                        const jkb_block_q8_k *x, size_t x_len, void *stream) {
    return gemv_call("gemv_tq1_0_q8_k", JKB_TQ1_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_tq2_0_q8_k(float *out, size_t out_len, const jkb_weight *w,
                        const jkb_block_q8_k *x, size_t x_len, void *stream) {
    return gemv_call("gemv_tq2_0_q8_k", JKB_TQ2_0, out, out_len, w, x, x_len, stream);
}

int jkb_gemv_rows(float *out, size_t out_len, const jkb_weight *w, const void *x, size_t x_len,
                  size_t row_begin, size_t row_end, void *stream) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->quant == JKB_I2_S)
        return fail(JKB_E_CAPABILITY, w->name, w->offset, w->byte_len, w->gguf_bytes,
                    "I2_S weights have no Q8 GEMV in the reference; use jkb_bitlinear_i8");
    if (x_len != w->nb)
        return fail(JKB_E_BOUNDS, w->name, w->offset, x_len, w->nb,
                    "gemv_rows: x_blocks len %zu != expected %zu", x_len, w->nb);
    if (row_begin > row_end || row_end > w->rows)
        return fail(JKB_E_BOUNDS, "gemv_rows", row_begin, row_end - row_begin, w->rows,
                    "row range %zu..%zu out of bounds for %zu rows", row_begin, row_end,
                    w->rows);
    if (out_len != row_end - row_begin)
        return fail(JKB_E_BOUNDS, "gemv_rows", 0, out_len * 4, (row_end - row_begin) * 4,
                    "output length %zu != row range length %zu", out_len, row_end - row_begin);
    if ((!out && out_len) || !x) return fail(JKB_E_INVALID, "gemv_rows", 0, 0, 0, "null pointer");
    if ((rc = check_align(out, 4, "gemv_rows", "output")) ||
        (rc = check_align(x, 4, "gemv_rows", "x_blocks")))
        return rc;
    GemvLaunch L{};
    L.w = w;
    L.x = x;
    L.act_kind = act_kind_for(w->quant);
    L.out = out;
    L.row_begin = row_begin;
    L.row_end = row_end;
    L.m = 1;
    return launch_gemv(L, as_stream(stream));
}

int jkb_gemv_block_dots(const jkb_weight *w, const void *x, size_t x_len, int32_t *sumi,
                        int32_t *summins, float *block_values, void *stream) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->quant == JKB_I2_S)
        return fail(JKB_E_CAPABILITY, w->name, 0, 0, 0, "I2_S has no Q8 block dot");
    if (x_len != w->nb)
        return fail(JKB_E_BOUNDS, w->name, w->offset, x_len, w->nb,
                    "gemv_block_dots: x_blocks len %zu != expected %zu", x_len, w->nb);
    if (!x || !sumi || !block_values)
        return fail(JKB_E_INVALID, "gemv_block_dots", 0, 0, 0, "null pointer");
    if ((rc = check_align(x, 4, "gemv_block_dots", "x_blocks")) ||
        (rc = check_align(sumi, 4, "gemv_block_dots", "sumi")) ||
        (rc = check_align(block_values, 4, "gemv_block_dots", "block_values")) ||
        (summins && (rc = check_align(summins, 4, "gemv_block_dots", "summins"))))
        return rc;
    GemvLaunch L{};
    L.w = w;
    L.x = x;
    L.act_kind = act_kind_for(w->quant);
    L.row_begin = 0;
    L.row_end = w->rows;
    L.m = 1;
    L.dbg_sumi = sumi;
    L.dbg_mins = summins;
    L.dbg_val = block_values;
    return launch_gemv(L, as_stream(stream));
}

}  // extern "C"
