// Memory-bound decode GEMV / BitLinear kernels over the jkb_weight GPU layout.
//
// Work split: one lane owns one whole block (32, 128 or 256 elements) of one weight row.
// A row with nb blocks gets LPR = min(32, pow2ceil(nb)) lanes (so one warp covers 1, 2, 4 ...
// rows at a time), and lane i of the row walks blocks i, i+LPR, ... Persistent CTAs of 8 warps
// stride over rows. The quant planes are lane-interleaved (gpu_layout.cuh), so the lanes' j-th
// 16-byte chunk loads form one contiguous span.
//
// Per block a lane forms the exact integer sums with dp4a against the activation staged in
// shared memory, and applies the offsets as integer corrections: -8 for Q4_0 and -1 for
// ternary codes through the block sum, -32 for Q6_K through the 16-element bsums. It then
// evaluates the reference's f32 block formula with separately rounded __fmul_rn/__fsub_rn, so
// integer sums and block values are bit-exact. Only the f32 sum of a row's block values runs in
// a different order than the reference's sequential row loop: in-lane, then a shuffle tree.
//
// Activation staging (shared memory, per CTA and token; chunk = 16 bytes, XOR-swizzled inside
// each block so that lanes reading the same chunk of different blocks hit different banks):
//   BlockQ8K rows : xq[K] | bsums i16[16] per superblock | xd f32 | block totals i32
//   BlockQ8_0 rows: xq[K] | xd f32 per block | block sums i32
//   i8 rows       : xq[K] | block totals i32 (block = the weight format's block)
#include <cooperative_groups.h>
#include <cstdio>
#include <cstdlib>
#include <type_traits>

#include "gpu_layout.cuh"
#include "jkb_internal.h"
#include "quant_math.cuh"

namespace jkb {

namespace cg = cooperative_groups;

// One weight matrix of a launch. The launch walks a virtual row range [row_begin, row_end);
// matrix i owns virtual rows [vbeg, next matrix's vbeg) and maps virtual row r to its own row
// r - vbeg + row0, writing out[r - vbeg].
struct MatArgs {
    const uint8_t *qs;
    const uint8_t *sc;
    const uint16_t *d;
    float *out;
    size_t vbeg, row0;
};

struct KArgs {
    MatArgs mat[GEMV_MAX_MATS];
    int nmat;
    size_t qs_row;  // identical for every matrix of a launch (same format and cols)
    size_t sc_row;
    const uint8_t *x;
    size_t x_row_stride;
    const float *act_scales;
    float act_scale;
    float i2s_scale;
    size_t out_ld;
    size_t row_begin, row_end;
    int nb;  // blocks per row
    int K;
    int lpr_shift;  // log2(lanes per row)
    int ntok;       // M_TOK: tokens of the launch
    int tpc;        // M_TOK: tokens per CTA (1..TOK_MAX), each staged in its own smem slot
    int stage16;    // ActI8: 16-byte staging copies when the activation is 16-byte aligned
    int32_t *dbg_sumi, *dbg_mins;
    float *dbg_val;
    // pushed outputs: every output element is also stored at these byte offsets from its
    // address (the same position in each peer's mapping of a pushing peer group's buffer)
    int npush;
    long long push_delta[JKB_PEER_MAX_RANKS - 1];
};

// Row pointers of one weight row: quant plane, scale plane, f16 block scales.
struct Row {
    const uint8_t *q;
    const uint8_t *s;
    const uint16_t *d;
};

// ---------------------------------------------------------------- device helpers

__device__ __forceinline__ uint4 ldg_stream(const uint8_t *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
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
// Programmatic dependent launch: wait for the preceding grid's memory to be visible / allow
// the next grid in the stream to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" :::);
}
__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ int4 lds4(const void *p) { return *reinterpret_cast<const int4 *>(p); }
__device__ __forceinline__ int sbyte(uint32_t w, int k) { return (int)(int8_t)(w >> (8 * k)); }

// ---------------------------------------------------------------- activation staging

// Copies `nwords` 32-bit words of x (4-byte aligned) into shared memory, word wi to dst(wi),
// with asynchronous global-to-shared copies: no registers hold the data, every copy of the
// thread is in flight at once, so staging costs one memory round trip whatever the CTA size.
// The caller synchronizes the CTA afterwards.
template <class Dst>
__device__ __forceinline__ void stage_words(const uint8_t *x, int nwords, Dst dst) {
    const uint32_t *src = reinterpret_cast<const uint32_t *>(x);
    for (int wi = threadIdx.x; wi < nwords; wi += blockDim.x) {
        const uint32_t sa = (uint32_t)__cvta_generic_to_shared(dst(wi));
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(src + wi)
                     : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// BlockQ8K activations (quant_q8.rs:62-71). Superblock s: 256 i8 at s*256 with chunk j at
// 16*(j ^ (s & 7)); its 16 bsums (two 16-byte halves, half h at 16*(h ^ ((s >> 2) & 1))).
struct ActQ8K {
    static constexpr bool kCluster = false;  // staged by each CTA alone
    static int units(int) { return 0; }
    static __host__ __device__ size_t bytes(int K) {
        return (size_t)K + (size_t)(K / 256) * 40 + 16;
    }
    static __device__ __forceinline__ const int8_t *chunk(const uint8_t *s, int sb, int j) {
        return (const int8_t *)(s + sb * 256 + 16 * (j ^ (sb & 7)));
    }
    static __device__ __forceinline__ int4 bsums_half(const uint8_t *s, int K, int sb, int h) {
        return lds4(s + K + sb * 32 + 16 * (h ^ ((sb >> 2) & 1)));
    }
    static __device__ __forceinline__ float xd(const uint8_t *s, int K, int sb) {
        return reinterpret_cast<const float *>(s + K + (K / 256) * 32)[sb];
    }
    static __device__ __forceinline__ int tot(const uint8_t *s, int K, int sb) {
        return reinterpret_cast<const int *>(s + K + (K / 256) * 36)[sb];
    }
    static __device__ void stage(const KArgs &a, const uint8_t *x, uint8_t *s) {
        const int nb = a.K / 256, K = a.K;  // 292-byte BlockQ8K = 73 words
        float *xd_ = (float *)(s + K + nb * 32);
        stage_words(x, nb * 73, [&](int wi) -> uint8_t * {
            const int blk = wi / 73, w = wi - blk * 73;
            if (w == 0) return reinterpret_cast<uint8_t *>(xd_ + blk);
            if (w <= 64) {
                const int ww = w - 1, j = ww >> 2;
                return s + blk * 256 + 16 * (j ^ (blk & 7)) + 4 * (ww & 3);
            }
            const int ww = w - 65, h = ww >> 2;
            return s + K + blk * 32 + 16 * (h ^ ((blk >> 2) & 1)) + 4 * (ww & 3);
        });
        __syncthreads();
        int *tot_ = (int *)(s + a.K + nb * 36);
        for (int blk = threadIdx.x; blk < nb; blk += blockDim.x) {
            const int16_t *b16 = (const int16_t *)(s + a.K + blk * 32);
            int t = 0;
            for (int k = 0; k < 16; k++) t += b16[k];
            tot_[blk] = t;
        }
        __syncthreads();
    }
};

// BlockQ8_0 activations (quant_q8.rs:37-44). Block b: 32 i8 at b*32 with chunk j at
// 16*(j ^ ((b >> 2) & 1)); f32 scale; integer sum of the 32 values.
struct ActQ80 {
    static constexpr bool kCluster = false;
    static int units(int) { return 0; }
    static __host__ __device__ size_t bytes(int K) {
        return (size_t)K + (size_t)(K / 32) * 8 + 16;
    }
    static __device__ __forceinline__ const int8_t *chunk(const uint8_t *s, int b, int j) {
        return (const int8_t *)(s + b * 32 + 16 * (j ^ ((b >> 2) & 1)));
    }
    static __device__ __forceinline__ float xd(const uint8_t *s, int K, int b) {
        return reinterpret_cast<const float *>(s + K)[b];
    }
    static __device__ __forceinline__ int tot(const uint8_t *s, int K, int b) {
        return reinterpret_cast<const int *>(s + K + (K / 32) * 4)[b];
    }
    static __device__ void stage(const KArgs &a, const uint8_t *x, uint8_t *s) {
        const int nb = a.K / 32;  // 36-byte BlockQ8_0 = 9 words
        float *xd_ = (float *)(s + a.K);
        stage_words(x, nb * 9, [&](int wi) -> uint8_t * {
            const int blk = wi / 9, w = wi - blk * 9;
            if (w == 0) return reinterpret_cast<uint8_t *>(xd_ + blk);
            const int ww = w - 1, j = ww >> 2;
            return s + blk * 32 + 16 * (j ^ ((blk >> 2) & 1)) + 4 * (ww & 3);
        });
        __syncthreads();
        int *tot_ = (int *)(s + a.K + nb * 4);
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            const int *q = (const int *)(s + b * 32);
            int t = 0;
#pragma unroll
            for (int w = 0; w < 8; w++) t = __dp4a(q[w], 0x01010101, t);
            tot_[b] = t;
        }
        __syncthreads();
    }
};

// JKB_GEMV_STAGE16=0 in the environment stages 16-byte aligned i8 activations with 4-byte
// copies too (for measuring the 16-byte copies against them); unset, 16-byte copies.
static bool stage16_host() {
    static const bool on = [] {
        const char *v = getenv("JKB_GEMV_STAGE16");
        return !(v && v[0] == '0' && v[1] == 0);
    }();
    return on;
}

// Plain i8 activations (BitLinear, ime.rs:882): blocks of the weight format's BE elements,
// chunk j at 16*(j ^ swz(b)); integer total per block.
template <int BE>
struct ActI8 {
    static constexpr bool kCluster = false;
    static int units(int) { return 0; }
    static __host__ __device__ size_t bytes(int K) {
        return (size_t)K + (size_t)(K / BE) * 4 + 16;
    }
    static __device__ __forceinline__ int swz(int b) { return BE >= 128 ? (b & 7) : ((b >> 2) & 1); }
    static __device__ __forceinline__ const int8_t *chunk(const uint8_t *s, int b, int j) {
        return (const int8_t *)(s + b * BE + 16 * (j ^ swz(b)));
    }
    static __device__ __forceinline__ int tot(const uint8_t *s, int K, int b) {
        return reinterpret_cast<const int *>(s + K)[b];
    }
    // the token's activation scale, stored after the block totals by stage()
    static __device__ __forceinline__ float scale(const KArgs &a, const uint8_t *s) {
        return *reinterpret_cast<const float *>(s + a.K + (a.K / BE) * 4);
    }
    static __device__ void stage(const KArgs &a, const uint8_t *x, uint8_t *s) {
        if (threadIdx.x == 0) *reinterpret_cast<float *>(s + a.K + (a.K / BE) * 4) = a.act_scale;
        auto at = [&](int wi) -> uint8_t * {
            const int e = 4 * wi, b = e / BE, off = e - b * BE, j = off >> 4;
            return s + b * BE + 16 * (j ^ swz(b)) + (off & 15);
        };
        if ((((uintptr_t)x) & 15) == 0 && a.stage16) {
            // 16-byte copies: a block's 16-byte chunk lands whole at its swizzled position, a
            // quarter of the 4-byte copies' requests
            for (int ci = threadIdx.x; ci < a.K / 16; ci += blockDim.x) {
                const int e = 16 * ci, b = e / BE, j = (e - b * BE) >> 4;
                const uint32_t sa =
                    (uint32_t)__cvta_generic_to_shared(s + b * BE + 16 * (j ^ swz(b)));
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(x + e)
                             : "memory");
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
        } else if ((((uintptr_t)x) & 3) == 0) {
            stage_words(x, a.K / 4, at);
        } else {
            for (int i = threadIdx.x; i < a.K / 4; i += blockDim.x)
                *(uint32_t *)at(i) = (uint32_t)x[4 * i] | ((uint32_t)x[4 * i + 1] << 8) |
                                     ((uint32_t)x[4 * i + 2] << 16) |
                                     ((uint32_t)x[4 * i + 3] << 24);
        }
        __syncthreads();
        int *tot_ = (int *)(s + a.K);
        for (int b = threadIdx.x; b < a.K / BE; b += blockDim.x) {
            const int *q = (const int *)(s + b * BE);
            int t = 0;
            for (int w = 0; w < BE / 4; w++) t = __dp4a(q[w], 0x01010101, t);
            tot_[b] = t;
        }
        __syncthreads();
    }
};

// Loads G consecutive f32 values at element e (a multiple of G) of x, as 16-byte vectors when x
// is 16-byte aligned.
template <int G>
__device__ __forceinline__ void load_group(const float *x, bool vec, int e, float (&v)[G]) {
    if (vec) {
#pragma unroll
        for (int i = 0; i < G; i += 4) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(x + e + i));
            v[i] = t.x;
            v[i + 1] = t.y;
            v[i + 2] = t.z;
            v[i + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < G; i++) v[i] = __ldg(x + e + i);
    }
}

// f32 input quantized while staging, once per thread-block cluster. The CTAs of a cluster
// split the quantization units (BlockQ8K superblocks / groups of four BlockQ8_0 blocks) among
// their warps; each warp quantizes a unit and writes the result into the staging buffer of every
// CTA of the cluster through distributed shared memory. Two cluster barriers bracket the writes:
// the first makes sure every CTA of the cluster is running, the second makes every CTA's buffer
// complete and visible. Every thread of every CTA reaches both.
//
// BlockQ8K (quantize_row_q8_k, quant_q8.rs:447-475), into the ActQ8K layout: lane l of the warp
// takes elements 8l..8l+8 of the superblock; absmax by shuffles; lane l writes its 8 bytes, even
// lanes the 16-element bsums, lane 0 the scale and the block total.
// Every CTA of the cluster has started, so its shared memory may be written through the
// cluster window. Only execution is ordered (nothing has been written yet), so the arrive is
// relaxed: a release here would wait for the weight loads already in flight. A CTA alone (C = 1)
// writes only its own shared memory and needs no barrier here.
__device__ __forceinline__ void cluster_started(unsigned C) {
    if (C > 1)
        asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" :::
                         "memory");
}
// The staged activation is complete in every CTA of the cluster. A CTA alone takes the CTA
// barrier, which (unlike the cluster barrier's release) does not wait for its weight loads.
__device__ __forceinline__ void cluster_staged(cg::cluster_group &cl, unsigned C) {
    if (C > 1)
        cl.sync();
    else
        __syncthreads();
}

struct ActQ8KF32 : ActQ8K {
    static constexpr bool kCluster = true;  // launched as thread-block clusters
    static int units(int K) { return K / 256; }
    static __device__ void stage(const KArgs &a, const uint8_t *xb, uint8_t *s) {
        cg::cluster_group cl = cg::this_cluster();
        const unsigned C = cl.num_blocks(), rank = cl.block_rank();
        const float *x = reinterpret_cast<const float *>(xb);
        const bool vec = (((uintptr_t)x) & 15) == 0;
        const int K = a.K, nsb = K / 256;
        const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
        const int gw = (int)rank * nw + (threadIdx.x >> 5), gstride = (int)C * nw;
        cluster_started(C);
        // two superblocks per warp and round: both loads are issued before the arithmetic
        for (int sb0 = gw; sb0 < nsb; sb0 += 2 * gstride) {  // warp-uniform
            float vv[2][8];
#pragma unroll
            for (int r = 0; r < 2; r++)
                if (sb0 + r * gstride < nsb)
                    load_group<8>(x, vec, (sb0 + r * gstride) * 256 + 8 * lane, vv[r]);
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int sb = sb0 + r * gstride;
                if (sb >= nsb) break;  // warp-uniform
                const float *v = vv[r];
                float am = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; i++)
                    if (finite_f(v[i])) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
                for (int m = 1; m < 32; m <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, m));
                float d, inv;
                q8_scale(am, d, inv);
                uint32_t p0 = 0, p1 = 0;
                int si = 0;
                if (am != 0.0f) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int q = round_scaled(v[i], inv);
                        si += q;
                        if (i < 4)
                            p0 |= ((uint32_t)(q & 0xFF)) << (8 * i);
                        else
                            p1 |= ((uint32_t)(q & 0xFF)) << (8 * (i - 4));
                    }
                }
                const int pair = si + __shfl_xor_sync(0xffffffffu, si, 1);
                // lanes of equal parity hold the 16 distinct pair sums: reduce over them
                int tot = pair;
#pragma unroll
                for (int m = 2; m < 32; m <<= 1) tot += __shfl_xor_sync(0xffffffffu, tot, m);
                const int j = lane >> 1;  // 16-element group = chunk index
                const uint32_t oq = sb * 256 + 16 * (j ^ (sb & 7)) + 8 * (lane & 1);
                const uint32_t ob = K + sb * 32 + 16 * ((j >> 3) ^ ((sb >> 2) & 1)) + 2 * (j & 7);
                const uint32_t od = K + nsb * 32 + 4 * sb, ot = K + nsb * 36 + 4 * sb;
                for (unsigned dst = 0; dst < C; dst++) {
                    uint8_t *rs = cl.map_shared_rank(s, dst);
                    *reinterpret_cast<uint2 *>(rs + oq) = make_uint2(p0, p1);
                    if ((lane & 1) == 0) *reinterpret_cast<int16_t *>(rs + ob) = (int16_t)pair;
                    if (lane == 0) {
                        *reinterpret_cast<float *>(rs + od) = d;
                        *reinterpret_cast<int *>(rs + ot) = tot;
                    }
                }
            }
        }
        cluster_staged(cl, C);
    }
};

// BlockQ8_0 (quantize_row_q8_0_f32, quant_q8.rs:203-219), into the ActQ80 layout: a unit is
// four consecutive 32-element blocks; lane l takes elements 4l..4l+4, so 8 lanes hold a block.
struct ActQ80F32 : ActQ80 {
    static constexpr bool kCluster = true;
    static int units(int K) { return (K / 32 + 3) / 4; }
    static __device__ void stage(const KArgs &a, const uint8_t *xb, uint8_t *s) {
        cg::cluster_group cl = cg::this_cluster();
        const unsigned C = cl.num_blocks(), rank = cl.block_rank();
        const float *x = reinterpret_cast<const float *>(xb);
        const bool vec = (((uintptr_t)x) & 15) == 0;
        const int K = a.K, nbk = K / 32, nunit = (nbk + 3) / 4;
        const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
        const int gw = (int)rank * nw + (threadIdx.x >> 5), gstride = (int)C * nw;
        cluster_started(C);
        const int sub = lane & 7;
        // two units per warp and round: both loads are issued before the arithmetic
        for (int u0 = gw; u0 < nunit; u0 += 2 * gstride) {  // warp-uniform
            float vv[2][4];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int b = 4 * (u0 + r * gstride) + (lane >> 3);
#pragma unroll
                for (int i = 0; i < 4; i++) vv[r][i] = 0.0f;
                if (u0 + r * gstride < nunit && b < nbk)
                    load_group<4>(x, vec, b * 32 + 4 * sub, vv[r]);
            }
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int u = u0 + r * gstride;
                if (u >= nunit) break;  // warp-uniform
                const int b = 4 * u + (lane >> 3);
                const bool valid = b < nbk;  // the last unit may hold fewer than four blocks
                const float *v = vv[r];
                float am = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (finite_f(v[i])) am = fmaxf(am, fabsf(v[i]));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
                am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
                float d, inv;
                q8_scale(am, d, inv);
                uint32_t pk = 0;
                int si = 0;
                if (am != 0.0f) {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int q = round_scaled(v[i], inv);
                        si += q;
                        pk |= ((uint32_t)(q & 0xFF)) << (8 * i);
                    }
                }
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                si += __shfl_xor_sync(0xffffffffu, si, 4);
                if (valid) {
                    const uint32_t oq = b * 32 + 16 * ((sub >> 2) ^ ((b >> 2) & 1)) + 4 * (sub & 3);
                    const uint32_t od = K + 4 * b, ot = K + nbk * 4 + 4 * b;
                    for (unsigned dst = 0; dst < C; dst++) {
                        uint8_t *rs = cl.map_shared_rank(s, dst);
                        *reinterpret_cast<uint32_t *>(rs + oq) = pk;
                        if (sub == 0) {
                            *reinterpret_cast<float *>(rs + od) = d;
                            *reinterpret_cast<int *>(rs + ot) = si;
                        }
                    }
                }
            }
        }
        cluster_staged(cl, C);
    }
};

// ---------------------------------------------------------------- formats
// load(): the block's registers; value(): exact integer sums (iv) and the f32 block value.

template <int QCH>
__device__ __forceinline__ void load_chunks(const KArgs &a, const Row &rp, int b, uint4 (&q)[QCH]) {
#pragma unroll
    for (int j = 0; j < QCH; j++) q[j] = ldg_stream(rp.q + qs_chunk_offset(a.nb, QCH, b, j));
}

template <int QCH>
__device__ __forceinline__ void prefetch_chunks(const KArgs &a, const Row &rp, int b) {
#pragma unroll
    for (int j = 0; j < QCH; j++) prefetch_l2(rp.q + qs_chunk_offset(a.nb, QCH, b, j));
}

// dot of the low (mask 0x0F) or in-place high (mask 0xF0, result x16) nibbles of 16 bytes
__device__ __forceinline__ int dot_lo(uint4 w, int4 x, int acc) {
    acc = dp4a_ss((int)(w.x & 0x0F0F0F0F), x.x, acc);
    acc = dp4a_ss((int)(w.y & 0x0F0F0F0F), x.y, acc);
    acc = dp4a_ss((int)(w.z & 0x0F0F0F0F), x.z, acc);
    return dp4a_ss((int)(w.w & 0x0F0F0F0F), x.w, acc);
}
__device__ __forceinline__ int dot_hi16(uint4 w, int4 x, int acc) {
    acc = dp4a_us(w.x & 0xF0F0F0F0u, x.x, acc);
    acc = dp4a_us(w.y & 0xF0F0F0F0u, x.y, acc);
    acc = dp4a_us(w.z & 0xF0F0F0F0u, x.z, acc);
    return dp4a_us(w.w & 0xF0F0F0F0u, x.w, acc);
}
__device__ __forceinline__ int dot_i8(uint4 w, int4 x, int acc) {
    acc = dp4a_ss((int)w.x, x.x, acc);
    acc = dp4a_ss((int)w.y, x.y, acc);
    acc = dp4a_ss((int)w.z, x.z, acc);
    return dp4a_ss((int)w.w, x.w, acc);
}

// Q4_0 x Q8_0 (quant_q8.rs:672-684): low nibble of byte j -> element j, high -> j+16, minus 8.
struct FQ4_0 {
    static constexpr int BE = 32;
    using Act = ActQ80;
    struct Ld {
        uint4 q[1];
        uint32_t d;
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<1>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<1>(a, rp, b, l.q);
        l.d = ldg_u16(rp.d + b);
        return l;
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv) {
        const int lo = dot_lo(l.q[0], lds4(Act::chunk(s, b, 0)), 0);
        const int hi = dot_hi16(l.q[0], lds4(Act::chunk(s, b, 1)), 0);
        const int sumi = lo + (hi >> 4) - 8 * Act::tot(s, a.K, b);
        iv = make_int2(sumi, 0);
        const float dw = f16_finite(l.d), xd = Act::xd(s, a.K, b);
        if (dw == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn((float)sumi, __fmul_rn(dw, xd));
    }
};

// Q8_0 weights: x Q8_0 activations (quant_q8.rs:707-717) or i8 BitLinear activations
// (ime.rs:840-853, :918-929).
template <class A>
struct FQ8_0 {
    static constexpr int BE = 32;
    using Act = A;
    struct Ld {
        uint4 q[2];
        uint32_t d;
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<2>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<2>(a, rp, b, l.q);
        l.d = ldg_u16(rp.d + b);
        return l;
    }
    static __device__ __forceinline__ int sum(const uint8_t *s, const Ld &l, int b) {
        return dot_i8(l.q[1], lds4(A::chunk(s, b, 1)), dot_i8(l.q[0], lds4(A::chunk(s, b, 0)), 0));
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv);
};
template <>
__device__ __forceinline__ float FQ8_0<ActQ80>::value(const KArgs &a, const uint8_t *s,
                                                       const Ld &l, int b, int2 &iv) {
    const int sumi = sum(s, l, b);
    iv = make_int2(sumi, 0);
    const float dw = f16_finite(l.d), xd = ActQ80::xd(s, a.K, b);
    if (dw == 0.0f || xd == 0.0f) return 0.0f;
    return __fmul_rn((float)sumi, __fmul_rn(dw, xd));
}
template <>
__device__ __forceinline__ float FQ8_0<ActI8<32>>::value(const KArgs &a, const uint8_t *s,
                                                          const Ld &l, int b, int2 &iv) {
    const int sumi = sum(s, l, b);
    iv = make_int2(sumi, 0);
    return __fmul_rn((float)sumi, __fmul_rn(f16_finite(l.d), ActI8<32>::scale(a, s)));
}

// Q4_K x Q8_K (quant_q8.rs:1817-1862). Chunk pair (2c, 2c+1) holds qs[32c..32c+32]: low
// nibbles pair with x[64c..64c+32] (activation chunks 4c, 4c+1), high nibbles with
// x[64c+32..64c+64] (chunks 4c+2, 4c+3), scaled by the 6-bit sc[2c], sc[2c+1]; the min term
// uses m[2c], m[2c+1] and the bsums of the same elements.
struct FQ4_K {
    static constexpr int BE = 256;
    using Act = ActQ8K;
    struct Ld {
        uint4 q[8];
        uint4 s;
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<8>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<8>(a, rp, b, l.q);
        l.s = __ldg(reinterpret_cast<const uint4 *>(rp.s + 16 * (size_t)b));
        return l;
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv) {
        // unpack_q4_q5_k_scales_mins: bytes of sc_lo/m_lo are sc[0..4]/m[0..4], of sc_hi/m_hi
        // are sc[4..8]/m[4..8]
        const uint32_t sc_lo = l.s.y & 0x3F3F3F3F, m_lo = l.s.z & 0x3F3F3F3F;
        const uint32_t sc_hi = (l.s.w & 0x0F0F0F0F) | ((l.s.y >> 2) & 0x30303030);
        const uint32_t m_hi = ((l.s.w >> 4) & 0x0F0F0F0F) | ((l.s.z >> 2) & 0x30303030);
        const int4 b0 = ActQ8K::bsums_half(s, a.K, b, 0), b1 = ActQ8K::bsums_half(s, a.K, b, 1);
        const int bs[16] = {(int)(int16_t)b0.x, b0.x >> 16, (int)(int16_t)b0.y, b0.y >> 16,
                            (int)(int16_t)b0.z, b0.z >> 16, (int)(int16_t)b0.w, b0.w >> 16,
                            (int)(int16_t)b1.x, b1.x >> 16, (int)(int16_t)b1.y, b1.y >> 16,
                            (int)(int16_t)b1.z, b1.z >> 16, (int)(int16_t)b1.w, b1.w >> 16};
        int sumi = 0, mins = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 qa = l.q[2 * c], qb = l.q[2 * c + 1];
            int slo = dot_lo(qa, lds4(ActQ8K::chunk(s, b, 4 * c)), 0);
            slo = dot_lo(qb, lds4(ActQ8K::chunk(s, b, 4 * c + 1)), slo);
            int shi = dot_hi16(qa, lds4(ActQ8K::chunk(s, b, 4 * c + 2)), 0);
            shi = dot_hi16(qb, lds4(ActQ8K::chunk(s, b, 4 * c + 3)), shi) >> 4;
            const uint32_t scw = c < 2 ? sc_lo : sc_hi, mw = c < 2 ? m_lo : m_hi;
            const int k = 2 * (c & 1);
            sumi += (int)((scw >> (8 * k)) & 0xFF) * slo + (int)((scw >> (8 * k + 8)) & 0xFF) * shi;
            mins += (int)((mw >> (8 * k)) & 0xFF) * (bs[4 * c] + bs[4 * c + 1]) +
                    (int)((mw >> (8 * k + 8)) & 0xFF) * (bs[4 * c + 2] + bs[4 * c + 3]);
        }
        iv = make_int2(sumi, mins);
        const float d = f16_finite(l.s.x & 0xFFFF), dmin = f16_finite(l.s.x >> 16);
        const float xd = ActQ8K::xd(s, a.K, b);
        if ((d == 0.0f && dmin == 0.0f) || xd == 0.0f) return 0.0f;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, xd), (float)sumi),
                         __fmul_rn(__fmul_rn(dmin, xd), (float)mins));
    }
};

// Bits 0..3 of v to the low bit of bytes 0..3 (v * 0x00204081 places bit i at 8i; the four
// shifted copies do not overlap, so nothing carries).
__device__ __forceinline__ uint32_t spread4(uint32_t v) {
    return ((v & 0xF) * 0x00204081u) & 0x01010101u;
}

// Q5_0 x Q8_0 (quant_q8.rs:688-703): element j = (low nibble of byte j | bit j of qh << 4) - 16,
// element j + 16 = (high nibble | bit j + 16 of qh << 4) - 16. The fifth bits enter as 0/1
// bytes dotted with the activations (times 16), the -16 through the block sum.
struct FQ5_0 {
    static constexpr int BE = 32;
    using Act = ActQ80;
    struct Ld {
        uint4 q[1];
        uint32_t h;
        uint32_t d;
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<1>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<1>(a, rp, b, l.q);
        l.h = __ldg(reinterpret_cast<const uint32_t *>(rp.s) + b);
        l.d = ldg_u16(rp.d + b);
        return l;
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv) {
        const int4 x0 = lds4(Act::chunk(s, b, 0)), x1 = lds4(Act::chunk(s, b, 1));
        const int lo = dot_lo(l.q[0], x0, 0);
        const int hi = dot_hi16(l.q[0], x1, 0) >> 4;
        int hb = dp4a_ss((int)spread4(l.h), x0.x, 0);
        hb = dp4a_ss((int)spread4(l.h >> 4), x0.y, hb);
        hb = dp4a_ss((int)spread4(l.h >> 8), x0.z, hb);
        hb = dp4a_ss((int)spread4(l.h >> 12), x0.w, hb);
        hb = dp4a_ss((int)spread4(l.h >> 16), x1.x, hb);
        hb = dp4a_ss((int)spread4(l.h >> 20), x1.y, hb);
        hb = dp4a_ss((int)spread4(l.h >> 24), x1.z, hb);
        hb = dp4a_ss((int)spread4(l.h >> 28), x1.w, hb);
        const int sumi = lo + hi + 16 * hb - 16 * Act::tot(s, a.K, b);
        iv = make_int2(sumi, 0);
        const float dw = f16_finite(l.d), xd = Act::xd(s, a.K, b);
        if (dw == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn((float)sumi, __fmul_rn(dw, xd));
    }
};

// Q5_K x Q8_K (quant_q8.rs:1866-1899): the Q4_K block plus a fifth bit per element from qh[32]
// (bit 2c of qh[l] for element 64c + l, bit 2c + 1 for element 64c + 32 + l). Chunks 0-7 are qs
// as for Q4_K, chunks 8 and 9 hold qh[0..16] and qh[16..32]; the 5-bit values (0..31) are
// formed per byte and dotted directly.
struct FQ5_K {
    static constexpr int BE = 256;
    using Act = ActQ8K;
    struct Ld {
        uint4 q[10];
        uint4 s;
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<10>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<10>(a, rp, b, l.q);
        l.s = __ldg(reinterpret_cast<const uint4 *>(rp.s + 16 * (size_t)b));
        return l;
    }
    // bit `bit` of every byte of h moved to bit 4 of the byte
    static __device__ __forceinline__ uint32_t bit4(uint32_t h, int bit) {
        return (bit <= 4 ? (h << (4 - bit)) : (h >> (bit - 4))) & 0x10101010u;
    }
    static __device__ __forceinline__ int dot5(uint4 q, uint4 h, int4 x, bool high, int bit) {
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w}, hw[4] = {h.x, h.y, h.z, h.w};
        const int xw[4] = {x.x, x.y, x.z, x.w};
        int acc = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t nib = (high ? (qw[k] >> 4) : qw[k]) & 0x0F0F0F0Fu;
            acc = dp4a_ss((int)(nib | bit4(hw[k], bit)), xw[k], acc);
        }
        return acc;
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv) {
        const uint32_t sc_lo = l.s.y & 0x3F3F3F3F, m_lo = l.s.z & 0x3F3F3F3F;
        const uint32_t sc_hi = (l.s.w & 0x0F0F0F0F) | ((l.s.y >> 2) & 0x30303030);
        const uint32_t m_hi = ((l.s.w >> 4) & 0x0F0F0F0F) | ((l.s.z >> 2) & 0x30303030);
        const int4 b0 = ActQ8K::bsums_half(s, a.K, b, 0), b1 = ActQ8K::bsums_half(s, a.K, b, 1);
        const int bs[16] = {(int)(int16_t)b0.x, b0.x >> 16, (int)(int16_t)b0.y, b0.y >> 16,
                            (int)(int16_t)b0.z, b0.z >> 16, (int)(int16_t)b0.w, b0.w >> 16,
                            (int)(int16_t)b1.x, b1.x >> 16, (int)(int16_t)b1.y, b1.y >> 16,
                            (int)(int16_t)b1.z, b1.z >> 16, (int)(int16_t)b1.w, b1.w >> 16};
        int sumi = 0, mins = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 qa = l.q[2 * c], qb = l.q[2 * c + 1];
            const int slo = dot5(qa, l.q[8], lds4(ActQ8K::chunk(s, b, 4 * c)), false, 2 * c) +
                            dot5(qb, l.q[9], lds4(ActQ8K::chunk(s, b, 4 * c + 1)), false, 2 * c);
            const int shi = dot5(qa, l.q[8], lds4(ActQ8K::chunk(s, b, 4 * c + 2)), true, 2 * c + 1) +
                            dot5(qb, l.q[9], lds4(ActQ8K::chunk(s, b, 4 * c + 3)), true, 2 * c + 1);
            const uint32_t scw = c < 2 ? sc_lo : sc_hi, mw = c < 2 ? m_lo : m_hi;
            const int k = 2 * (c & 1);
            sumi += (int)((scw >> (8 * k)) & 0xFF) * slo + (int)((scw >> (8 * k + 8)) & 0xFF) * shi;
            mins += (int)((mw >> (8 * k)) & 0xFF) * (bs[4 * c] + bs[4 * c + 1]) +
                    (int)((mw >> (8 * k + 8)) & 0xFF) * (bs[4 * c + 2] + bs[4 * c + 3]);
        }
        iv = make_int2(sumi, mins);
        const float d = f16_finite(l.s.x & 0xFFFF), dmin = f16_finite(l.s.x >> 16);
        const float xd = ActQ8K::xd(s, a.K, b);
        if ((d == 0.0f && dmin == 0.0f) || xd == 0.0f) return 0.0f;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, xd), (float)sumi),
                         __fmul_rn(__fmul_rn(dmin, xd), (float)mins));
    }
};

// Q6_K x Q8_K (quant_q8.rs:1903-1942). Chunks 0-7 are ql, 8-11 qh (GGUF order). For half h
// and is = i: A = ql[64h+16i..] (chunk 4h+i), B = ql[64h+32+16i..] (4h+2+i),
// H = qh[32h+16i..] (8+2h+i); the four 6-bit values pair with activation chunks 8h+i+{0,2,4,6}
// and scales sc[8h+i+{0,2,4,6}]; -32 is applied through the matching bsums.
struct FQ6_K {
    static constexpr int BE = 256;
    using Act = ActQ8K;
    struct Ld {
        uint4 q[12];
        uint4 s;
        uint32_t d;
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<12>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<12>(a, rp, b, l.q);
        l.s = __ldg(reinterpret_cast<const uint4 *>(rp.s + 16 * (size_t)b));
        l.d = ldg_u16(rp.d + b);
        return l;
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv) {
        const int4 b0 = ActQ8K::bsums_half(s, a.K, b, 0), b1 = ActQ8K::bsums_half(s, a.K, b, 1);
        const int bs[16] = {(int)(int16_t)b0.x, b0.x >> 16, (int)(int16_t)b0.y, b0.y >> 16,
                            (int)(int16_t)b0.z, b0.z >> 16, (int)(int16_t)b0.w, b0.w >> 16,
                            (int)(int16_t)b1.x, b1.x >> 16, (int)(int16_t)b1.y, b1.y >> 16,
                            (int)(int16_t)b1.z, b1.z >> 16, (int)(int16_t)b1.w, b1.w >> 16};
        const uint32_t scw[4] = {l.s.x, l.s.y, l.s.z, l.s.w};
        int sumi = 0;
#pragma unroll
        for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const uint4 A = l.q[4 * h + i], B = l.q[4 * h + 2 + i], H = l.q[8 + 2 * h + i];
                const int c0 = 8 * h + i;
                const int4 x1 = lds4(ActQ8K::chunk(s, b, c0)), x2 = lds4(ActQ8K::chunk(s, b, c0 + 2));
                const int4 x3 = lds4(ActQ8K::chunk(s, b, c0 + 4)), x4 = lds4(ActQ8K::chunk(s, b, c0 + 6));
                const uint32_t a_[4] = {A.x, A.y, A.z, A.w}, b_[4] = {B.x, B.y, B.z, B.w},
                               h_[4] = {H.x, H.y, H.z, H.w};
                const int x1_[4] = {x1.x, x1.y, x1.z, x1.w}, x2_[4] = {x2.x, x2.y, x2.z, x2.w},
                          x3_[4] = {x3.x, x3.y, x3.z, x3.w}, x4_[4] = {x4.x, x4.y, x4.z, x4.w};
                int S1 = 0, S2 = 0, S3 = 0, S4 = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t u1 = (a_[j] & 0x0F0F0F0F) | ((h_[j] << 4) & 0x30303030);
                    const uint32_t u2 = (b_[j] & 0x0F0F0F0F) | ((h_[j] << 2) & 0x30303030);
                    const uint32_t u3 = ((a_[j] >> 4) & 0x0F0F0F0F) | (h_[j] & 0x30303030);
                    const uint32_t u4 = ((b_[j] >> 4) & 0x0F0F0F0F) | ((h_[j] >> 2) & 0x30303030);
                    S1 = dp4a_ss((int)u1, x1_[j], S1);
                    S2 = dp4a_ss((int)u2, x2_[j], S2);
                    S3 = dp4a_ss((int)u3, x3_[j], S3);
                    S4 = dp4a_ss((int)u4, x4_[j], S4);
                }
                // scales sc[c0 + {0,2,4,6}]: byte (c0 & 3) + {0, 2} of words c0/4 and c0/4 + 1
                const uint32_t w0 = scw[c0 >> 2], w1 = scw[(c0 >> 2) + 1];
                const int k = c0 & 3;
                sumi += sbyte(w0, k) * (S1 - 32 * bs[c0]) + sbyte(w0, k + 2) * (S2 - 32 * bs[c0 + 2]) +
                        sbyte(w1, k) * (S3 - 32 * bs[c0 + 4]) + sbyte(w1, k + 2) * (S4 - 32 * bs[c0 + 6]);
            }
        }
        iv = make_int2(sumi, 0);
        const float d = f16_finite(l.d), xd = ActQ8K::xd(s, a.K, b);
        if (d == 0.0f || xd == 0.0f) return 0.0f;
        return __fmul_rn(__fmul_rn(d, xd), (float)sumi);
    }
};

// TQ2_0 / TQ1_0 x Q8_K (quant_q8.rs:1960-2003) and TQ2_0 / TQ1_0 BitLinear (ime.rs:918-929).
// Chunk p, word W, bit pair j holds the codes (value + 1) of elements 64p+16W+4j+{0..3}, i.e.
// word j of activation chunk 4p+W; the +1 is removed as -sum(x) over the block.
template <class A>
struct FTQ2 {
    static constexpr int BE = 256;
    using Act = A;
    struct Ld {
        uint4 q[4];
        uint32_t d;
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<4>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<4>(a, rp, b, l.q);
        l.d = ldg_u16(rp.d + b);
        return l;
    }
    static __device__ __forceinline__ int codes(const uint8_t *s, const Ld &l, int b) {
        int t = 0;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const uint32_t w_[4] = {l.q[p].x, l.q[p].y, l.q[p].z, l.q[p].w};
#pragma unroll
            for (int W = 0; W < 4; W++) {
                const int4 xv = lds4(A::chunk(s, b, 4 * p + W));
                t = dp4a_ss((int)(w_[W] & 0x03030303), xv.x, t);
                t = dp4a_ss((int)((w_[W] >> 2) & 0x03030303), xv.y, t);
                t = dp4a_ss((int)((w_[W] >> 4) & 0x03030303), xv.z, t);
                t = dp4a_ss((int)((w_[W] >> 6) & 0x03030303), xv.w, t);
            }
        }
        return t;
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv);
};
template <>
__device__ __forceinline__ float FTQ2<ActQ8K>::value(const KArgs &a, const uint8_t *s,
                                                     const Ld &l, int b, int2 &iv) {
    const int sumi = codes(s, l, b) - ActQ8K::tot(s, a.K, b);
    iv = make_int2(sumi, 0);
    const float xd = ActQ8K::xd(s, a.K, b);
    const float dw = f16_finite(l.d);
    if (xd == 0.0f || dw == 0.0f) return 0.0f;
    return __fmul_rn((float)sumi, __fmul_rn(dw, xd));
}
template <>
__device__ __forceinline__ float FTQ2<ActI8<256>>::value(const KArgs &a, const uint8_t *s,
                                                         const Ld &l, int b, int2 &iv) {
    const int sumi = codes(s, l, b) - ActI8<256>::tot(s, a.K, b);
    iv = make_int2(sumi, 0);
    return __fmul_rn((float)sumi, __fmul_rn(f16_finite(l.d), ActI8<256>::scale(a, s)));
}

// I2_S BitLinear (quant.rs:370-377, ime.rs:918-929). Chunk h holds bytes 16h..16h+16; byte g
// carries elements g, 32+g, 64+g, 96+g in bits [7:6], [5:4], [3:2], [1:0], so plane j of
// word W pairs with word W of activation chunk 2j+h.
struct FI2S {
    static constexpr int BE = 128;
    using Act = ActI8<128>;
    struct Ld {
        uint4 q[2];
    };
    static __device__ __forceinline__ void prefetch(const KArgs &a, const Row &rp, int b) {
        prefetch_chunks<2>(a, rp, b);
    }
    static __device__ __forceinline__ Ld load(const KArgs &a, const Row &rp, int b) {
        Ld l;
        load_chunks<2>(a, rp, b, l.q);
        return l;
    }
    static __device__ __forceinline__ float value(const KArgs &a, const uint8_t *s, const Ld &l,
                                                  int b, int2 &iv) {
        int t = 0;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t w_[4] = {l.q[h].x, l.q[h].y, l.q[h].z, l.q[h].w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int4 xv = lds4(Act::chunk(s, b, 2 * j + h));
                const int x_[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int W = 0; W < 4; W++)
                    t = dp4a_ss((int)((w_[W] >> (6 - 2 * j)) & 0x03030303), x_[W], t);
            }
        }
        const int sumi = t - Act::tot(s, a.K, b);
        iv = make_int2(sumi, 0);
        return __fmul_rn((float)sumi, __fmul_rn(a.i2s_scale, Act::scale(a, s)));
    }
};

// ---------------------------------------------------------------- the kernel

constexpr int MAX_WARPS = 8;

// M_SINGLE: one matrix, row sums to out. M_DIAG: one matrix, per-block integer sums and values
// to the diagnostic arrays. M_MULTI: several matrices over one activation (virtual rows).
// M_TOK: one matrix, several tokens per CTA -- every weight block is loaded once and dotted
// with up to TOK_MAX staged activations (token batches of pre-quantized input).
enum { M_SINGLE = 0, M_DIAG = 1, M_MULTI = 2, M_TOK = 3 };
constexpr int TOK_MAX = 8;

// Row pointers of virtual row r and its output slot (token 0).
template <int MODE>
__device__ __forceinline__ Row row_of(const KArgs &a, size_t r, float *&outp) {
    const uint8_t *qs = a.mat[0].qs, *sc = a.mat[0].sc;
    const uint16_t *d = a.mat[0].d;
    float *o = a.mat[0].out;
    size_t vbeg = a.mat[0].vbeg, row0 = a.mat[0].row0;
    if (MODE == M_MULTI) {
        // matrices are ordered by vbeg: the last one starting at or before r owns it
#pragma unroll
        for (int i = 1; i < GEMV_MAX_MATS; i++) {
            if (i < a.nmat && r >= a.mat[i].vbeg) {
                qs = a.mat[i].qs;
                sc = a.mat[i].sc;
                d = a.mat[i].d;
                o = a.mat[i].out;
                vbeg = a.mat[i].vbeg;
                row0 = a.mat[i].row0;
            }
        }
    }
    const size_t lr = r - vbeg + row0;
    outp = o + (r - vbeg);
    return Row{qs + lr * a.qs_row, sc + lr * a.sc_row, d + lr * (size_t)a.nb};
}

// Resident CTAs per SM the register allocation must allow (0: the compiler's choice). The
// single-matrix Q6_K kernel streams the lm_head, the largest matrix of a decode step: held to
// 64 registers it runs 4 CTAs of 8 warps per SM instead of 3 (74 registers), so each SM keeps
// a third more 16-byte loads in flight (measured: 86 % -> 90 % of HBM on the 4096 x 128256
// lm_head, for a 4-byte spill).
template <class F, int MODE>
constexpr int gemv_min_blocks() {
    return MODE == M_SINGLE && std::is_same<F, FQ6_K>::value ? 4 : 0;
}

// Blocks a lane loads before consuming the first of them (the unrolled main loop), per
// format: as many as keep the loads in registers, given the size of one block's load (Ld).
// A launch takes this unrolled variant when its warps would otherwise walk several blocks
// one DRAM round trip at a time (small matrices, or rows longer than 32 blocks).
template <class F> struct GemvUnroll { static constexpr int value = 1; };
template <> struct GemvUnroll<FQ4_0> { static constexpr int value = 4; };
template <> struct GemvUnroll<FQ5_0> { static constexpr int value = 4; };
template <> struct GemvUnroll<FQ8_0<ActQ80>> { static constexpr int value = 4; };
template <> struct GemvUnroll<FQ8_0<ActI8<32>>> { static constexpr int value = 4; };
template <> struct GemvUnroll<FI2S> { static constexpr int value = 4; };
template <> struct GemvUnroll<FTQ2<ActQ8K>> { static constexpr int value = 2; };
template <> struct GemvUnroll<FTQ2<ActI8<256>>> { static constexpr int value = 2; };
template <> struct GemvUnroll<FQ4_K> { static constexpr int value = 2; };

// F: weight format. S: activation stager (F::Act, or a stager that quantizes f32 input into
// the same shared-memory layout). U: blocks in flight per lane (1 or GemvUnroll<F>).
template <class F, class S, int MODE, int U>
__global__ void __launch_bounds__(MAX_WARPS * 32, (gemv_min_blocks<F, MODE>())) gemv_kernel(KArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int TB = MODE == M_TOK ? TOK_MAX : 1;  // token slots per CTA
    const int tok = MODE == M_TOK ? (int)blockIdx.y * a.tpc : (int)blockIdx.y;
    const int nt = MODE == M_TOK ? min(a.tpc, a.ntok - tok) : 1;
    const size_t slot = MODE == M_TOK ? (S::bytes(a.K) + 15) / 16 * 16 : 0;
    KArgs args = a;
    const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int lpr = 1 << a.lpr_shift, rpw = 32 >> a.lpr_shift;
    const int li = lane & (lpr - 1), rsub = lane >> a.lpr_shift;
    const size_t wid = (size_t)blockIdx.x * warps + (threadIdx.x >> 5);
    const size_t nwarps = (size_t)gridDim.x * warps;
    const size_t tok_off = (size_t)tok * a.out_ld;
    const size_t stride = nwarps * rpw;
    size_t r0 = a.row_begin + wid * rpw;  // warp-uniform position (r0, b0)
    int b0 = 0;
    float acc[TB];
#pragma unroll
    for (int t = 0; t < TB; t++) acc[t] = 0.0f;
    // Grouped launches keep the current row's pointers in registers (the owning matrix is
    // looked up once per row); single-matrix launches form them from the parameters at each
    // load, which keeps the register count of the long-running kernels down.
    float *outp = nullptr;
    Row rpm{};
    if (MODE == M_MULTI) rpm = row_of<MODE>(a, r0 + rsub, outp);
    auto row_ptrs = [&]() -> Row {
        if (MODE == M_MULTI) return rpm;
        const size_t r = r0 + rsub;
        return Row{a.mat[0].qs + r * a.qs_row, a.mat[0].sc + r * a.sc_row,
                   a.mat[0].d + r * (size_t)a.nb};
    };
    // one block of row r0 + rsub: the exact integer sums and the f32 block value
    auto consume = [&](const typename F::Ld &l, int b) {
#pragma unroll
        for (int t = 0; t < TB; t++) {
            if (t >= nt) break;
            int2 iv;
            const float v = F::value(args, smem + t * slot, l, b, iv);
            if (MODE == M_DIAG) {
                const size_t o = (r0 + rsub - a.row_begin) * (size_t)a.nb + b;
                a.dbg_sumi[o] = iv.x;
                if (a.dbg_mins) a.dbg_mins[o] = iv.y;
                a.dbg_val[o] = v;
            } else {
                acc[t] = __fadd_rn(acc[t], v);
            }
        }
    };
    // advance to the next block column; at the end of a row, reduce its lanes and store
    auto advance = [&]() {
        b0 += lpr;
        if (b0 >= a.nb) {
            if (MODE != M_DIAG) {
#pragma unroll
                for (int t = 0; t < TB; t++) {
                    if (t >= nt) break;
                    for (int m = lpr >> 1; m > 0; m >>= 1)
                        acc[t] = __fadd_rn(acc[t], __shfl_xor_sync(0xffffffffu, acc[t], m));
                    if (li == 0 && r0 + rsub < a.row_end) {
                        float *o =
                            MODE == M_MULTI ? outp : a.mat[0].out + (r0 + rsub - a.row_begin);
                        float *dst = o + tok_off + (size_t)t * a.out_ld;
                        *dst = acc[t];
#pragma unroll
                        for (int q = 0; q < JKB_PEER_MAX_RANKS - 1; q++)
                            if (q < a.npush)
                                *reinterpret_cast<float *>(reinterpret_cast<char *>(dst) +
                                                           a.push_delta[q]) = acc[t];
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < TB; t++) acc[t] = 0.0f;
            b0 = 0;
            r0 += stride;
            if (MODE == M_MULTI) rpm = row_of<MODE>(a, r0 + rsub, outp);
        }
    };
    // The unrolled variant's next U steps (the positions advance() will visit): their loads
    // are issued together and consumed in order, so U DRAM round trips overlap.
    typename F::Ld l[U];
    int bq[U];
    bool vq[U];
    auto issue = [&]() {
        size_t pr = r0;
        int pb = b0;
        Row rp = row_ptrs();
#pragma unroll
        for (int u = 0; u < U; u++) {
            bq[u] = pb + li;
            vq[u] = pr < a.row_end && pr + rsub < a.row_end && bq[u] < a.nb;
            if (vq[u]) l[u] = F::load(args, rp, bq[u]);
            pb += lpr;
            if (pb >= a.nb && u + 1 < U) {
                pb = 0;
                pr += stride;
                if (MODE == M_MULTI) {
                    float *unused;
                    rp = row_of<MODE>(a, pr + rsub, unused);
                } else {
                    rp = Row{a.mat[0].qs + (pr + rsub) * a.qs_row,
                             a.mat[0].sc + (pr + rsub) * a.sc_row,
                             a.mat[0].d + (pr + rsub) * (size_t)a.nb};
                }
            }
        }
    };
    // Weights never depend on the previous kernel in the stream; the activation may. Before
    // waiting for the previous grid (programmatic dependent launch), the unrolled variant
    // loads the warp's first U blocks into registers and the one-block loop pulls the first
    // block into L2; the activation is staged after the wait. (Weight handles are complete
    // when their upload returns, so no earlier kernel writes them.)
    if constexpr (U == 1) {
        if (r0 + rsub < a.row_end && li < a.nb) F::prefetch(args, row_ptrs(), li);
    } else {
        issue();
    }
    pdl_wait();
    pdl_launch_dependents();
    if (MODE == M_TOK) {
        for (int t = 0; t < nt; t++) {
            if (a.act_scales) args.act_scale = a.act_scales[tok + t];
            S::stage(args, a.x + (size_t)(tok + t) * a.x_row_stride, smem + t * slot);
        }
    } else {
        if (a.act_scales) args.act_scale = a.act_scales[tok];
        S::stage(args, a.x + (size_t)tok * a.x_row_stride, smem);
    }
    if constexpr (U == 1) {
        while (r0 < a.row_end) {
            const int b = b0 + li;
            if (r0 + rsub < a.row_end && b < a.nb) {
                const typename F::Ld ld = F::load(args, row_ptrs(), b);
                consume(ld, b);
            }
            advance();
        }
    } else {
        while (r0 < a.row_end) {
#pragma unroll
            for (int u = 0; u < U; u++) {
                if (r0 >= a.row_end) break;
                if (vq[u]) consume(l[u], bq[u]);
                advance();
            }
            if (r0 < a.row_end) issue();
        }
    }
    // pushed outputs are performed at system scope before the grid completes, so a peer that
    // sees the signal sent after it (jkb_peer_group_signal) sees them
    if (a.npush) __threadfence_system();
}

// ---------------------------------------------------------------- launch

// Largest cluster for stagers that quantize f32 input once per cluster. A launch uses the
// smallest power of two (at most this) that leaves each warp of the cluster at most two
// quantization units: larger clusters cut the repeated quantization of wide inputs and of
// small CTAs, smaller ones pack the device better.
constexpr unsigned GEMV_MAX_CLUSTER = 8;
// JKB_GEMV_MAX_CLUSTER=1, 2 or 4 in the environment caps the cluster of the f32-input stagers
// (for measuring the cluster-shared quantization against one per CTA); unset, up to 8.
static unsigned max_cluster() {
    static const unsigned c = [] {
        const char *v = getenv("JKB_GEMV_MAX_CLUSTER");
        const int n = v ? atoi(v) : 0;
        return (n == 1 || n == 2 || n == 4) ? (unsigned)n : GEMV_MAX_CLUSTER;
    }();
    return c;
}

// Smallest CTA (in warps) the launcher shrinks to for small matrices. Every CTA stages the
// whole activation (or, with f32 input, its cluster quantizes it), so small CTAs leave each
// thread several staging copies or quantization rounds: launches keep 8-warp CTAs even when
// fewer CTAs than SMs result (measured, Q4_K_M, 2-warp floor -> 8: f32 input 512 x 14336
// 6.91 -> 4.53 us, 512 x 4096 3.76 -> 3.20 us, 1024 x 14336 5.74 -> 5.22 us; pre-quantized
// 512 x 14336 9.26 -> 5.03 us, 1024 x 4096 4.22 -> 3.01 us; 2048 rows and up unchanged).
// JKB_GEMV_MIN_WARPS=2 or 4 in the environment lets the launcher shrink CTAs that far when a
// matrix has fewer rows than the SMs' 8-warp CTAs take (for measuring the launch shapes).
static int min_warps() {
    static const int w = [] {
        const char *v = getenv("JKB_GEMV_MIN_WARPS");
        const int n = v ? atoi(v) : 0;
        return (n == 2 || n == 4) ? n : 8;
    }();
    return w;
}

// Smallest cluster of the f32-input stagers: 2, so that even inputs one CTA's warps quantize in
// one round are quantized once per CTA pair (measured on the Llama-3-8B decode shapes, K = 4096:
// q/k/v 6.35 -> 5.94 us, o 4.55 -> 4.20 us, gate/up 14.77 -> 14.50 us; clusters of at least 4
// made gate/up slower, 18.6 us). JKB_GEMV_MIN_CLUSTER=1, 2 or 4 in the environment sets it (for
// measuring).
static unsigned min_cluster() {
    static const unsigned c = [] {
        const char *v = getenv("JKB_GEMV_MIN_CLUSTER");
        const int n = v ? atoi(v) : 0;
        return (n == 1 || n == 2 || n == 4) ? (unsigned)n : 2u;
    }();
    return c;
}

// Launch shape of one GEMV launch (plan_t) and the number of steps each warp walks with it.
struct GemvPlan {
    int warps;
    unsigned C;
    size_t gx, m, smem;
    size_t steps;  // block steps per warp (row steps x ceil(nb / lanes per row))
};

template <class F, class S, int MODE, int U>
static GemvPlan plan_t(KArgs &a, size_t m) {
    GemvPlan p{};
    size_t smem = S::bytes(a.K);
    if (MODE == M_TOK) {  // as many token slots per CTA as fit in 150 KB, at most TOK_MAX
        const size_t slot = (smem + 15) / 16 * 16;
        size_t tpc = (150 * 1024) / slot;
        tpc = tpc < (size_t)TOK_MAX ? tpc : (size_t)TOK_MAX;
        tpc = tpc < m ? tpc : m;
        if (tpc < 1) tpc = 1;
        a.tpc = (int)tpc;
        a.ntok = (int)m;
        smem = slot * tpc;
        m = (m + tpc - 1) / tpc;  // CTA rows of the grid
    }
    auto kern = gemv_kernel<F, S, MODE, U>;
    // resident CTAs on the device per CTA size (8, 4 or 2 warps) and cluster size (1, 2, 4,
    // 8; for cluster launches the resident clusters times the cluster size), cached per
    // template instance (B200 only)
    static int resident_cached[3][4] = {{-1, -1, -1, -1}, {-1, -1, -1, -1}, {-1, -1, -1, -1}};
    static size_t smem_cached = 0;
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        attr_set = true;
    }
    if (smem_cached != smem) {
        for (int i = 0; i < 3; i++)
            for (int j = 0; j < 4; j++) resident_cached[i][j] = -1;
        smem_cached = smem;
    }
    const int rpw = 32 >> a.lpr_shift;
    const size_t rows = a.row_end - a.row_begin;
    const size_t sms = (size_t)num_sms();
    // Fewer warps per CTA when the matrix is small, down to min_warps() (8 unless set).
    int warps = MAX_WARPS;
    while (warps > min_warps() &&
           m * ((rows + (size_t)warps * rpw - 1) / ((size_t)warps * rpw)) < sms)
        warps >>= 1;
    const int slot = warps == 8 ? 0 : warps == 4 ? 1 : 2;
    unsigned C = 1;
    int cs = 0;
    if (S::kCluster)
        while (C < max_cluster() &&
               (S::units(a.K) > 2 * warps * (int)C || C < min_cluster())) {
            C <<= 1;
            cs++;
        }
    int &resident = resident_cached[slot][cs];
    if (resident < 0) {
        int n = 0;
        if (C > 1) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(C);
            cfg.blockDim = dim3(warps * 32);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = C;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
            n *= (int)C;
        } else {
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, warps * 32, smem);
            n *= (int)sms;
        }
        resident = n < (int)C ? (int)C : n;
    }
    const size_t want = (rows + (size_t)warps * rpw - 1) / ((size_t)warps * rpw);
    const size_t cap = (size_t)resident;
    size_t gx = want;
    if (m * gx > cap) gx = (cap + m - 1) / m;
    gx = (gx + C - 1) / C * C;  // whole clusters
    if (gx < 1) gx = 1;
    const size_t lpr = (size_t)1 << a.lpr_shift;
    p.warps = warps;
    p.C = C;
    p.gx = gx;
    p.m = m;
    p.smem = smem;
    p.steps = (rows + gx * warps * rpw - 1) / (gx * warps * rpw) * ((a.nb + lpr - 1) / lpr);
    return p;
}

template <class F, class S, int MODE, int U>
static int launch_p(const KArgs &a, const GemvPlan &p, cudaStream_t st, const char *name) {
    cudaError_t e = launch_pdl_cluster(gemv_kernel<F, S, MODE, U>,
                                       dim3((unsigned)p.gx, (unsigned)p.m), dim3(p.warps * 32),
                                       p.smem, st, p.C, a);
    return e == cudaSuccess ? JKB_OK : fail_cuda(e, name);
}

// JKB_GEMV_UNROLL=1 in the environment keeps every launch on the one-block-at-a-time loop (for
// measuring the unrolled loop against it); unset, the launcher decides.
static bool unroll_allowed() {
    static const bool ok = [] {
        const char *v = getenv("JKB_GEMV_UNROLL");
        return !(v && v[0] == '1' && v[1] == 0);
    }();
    return ok;
}

// Single and grouped launches of the formats with GemvUnroll<F> > 1 take the unrolled loop
// (its first loads also go ahead of the programmatic-launch wait) when each warp walks at most
// UNROLL_MAX_STEPS block steps: the small and mid-size matrices of a decode step, whose
// launches are latency-bound. Longer walks keep the one-block loop, whose lower register count
// keeps more CTAs resident (measured: 14336 x 14336 Q4_K_M, 8 steps a warp, 25.7 us with it
// against 27.4 us unrolled). Q6_K / Q5_K, token batches and the diagnostic launch keep one
// block at a time.
constexpr size_t UNROLL_MAX_STEPS = 4;

template <class F, class S, int MODE>
static int launch_t(const KArgs &a_in, size_t m, cudaStream_t st, const char *name) {
    constexpr bool can = MODE == M_SINGLE || MODE == M_MULTI;
    constexpr int UF = can ? GemvUnroll<F>::value : 1;
    KArgs a = a_in;
    const GemvPlan p1 = plan_t<F, S, MODE, 1>(a, m);
    if (UF > 1 && p1.steps <= UNROLL_MAX_STEPS && unroll_allowed()) {
        KArgs au = a_in;
        const GemvPlan pu = plan_t<F, S, MODE, UF>(au, m);
        return launch_p<F, S, MODE, UF>(au, pu, st, name);
    }
    return launch_p<F, S, MODE, 1>(a, p1, st, name);
}

static const size_t MAX_K = 120 * 1024;

int launch_gemv(const GemvLaunch &L, cudaStream_t st) {
    const jkb_weight *w = L.w;
    const bool multi = L.nmat > 1;
    KArgs a = {};
    if (multi) {
        if (L.nmat > GEMV_MAX_MATS)
            return fail(JKB_E_BOUNDS, "gemv", 0, (size_t)L.nmat, GEMV_MAX_MATS,
                        "%d matrices in one launch (limit %d)", L.nmat, GEMV_MAX_MATS);
        size_t v = 0;
        for (int i = 0; i < L.nmat; i++) {
            const jkb_weight *wi = L.ws[i];
            if (wi->gpu_format != w->gpu_format || wi->cols != w->cols ||
                wi->p.qs_row != w->p.qs_row || wi->p.sc_row != w->p.sc_row ||
                wi->p.i2s_scale != w->p.i2s_scale)
                return fail(JKB_E_INVALID, wi->name, wi->offset, wi->byte_len, wi->gguf_bytes,
                            "grouped GEMV: %s [%zu, %zu] does not share the format and width "
                            "of %s [%zu, %zu]",
                            wi->name, wi->rows, wi->cols, w->name, w->rows, w->cols);
            a.mat[i] = MatArgs{wi->p.qs, wi->p.sc, wi->p.d, L.outs[i], v, 0};
            v += wi->rows;
        }
        a.nmat = L.nmat;
        a.row_begin = 0;
        a.row_end = v;
    } else {
        a.mat[0] = MatArgs{w->p.qs, w->p.sc, w->p.d, L.out, L.row_begin, L.row_begin};
        a.nmat = 1;
        a.row_begin = L.row_begin;
        a.row_end = L.row_end;
    }
    a.qs_row = w->p.qs_row;
    a.sc_row = w->p.sc_row;
    a.stage16 = stage16_host() ? 1 : 0;
    a.x = (const uint8_t *)L.x;
    a.x_row_stride = L.x_row_stride;
    a.act_scales = L.act_scales;
    a.act_scale = L.act_scale;
    a.i2s_scale = w->p.i2s_scale;
    a.out_ld = L.out_ld;
    a.nb = (int)w->nb;
    a.K = (int)w->cols;
    int sh = 0;
    while ((1 << sh) < a.nb && sh < 5) sh++;
    a.lpr_shift = sh;
    a.dbg_sumi = L.dbg_sumi;
    a.dbg_mins = L.dbg_mins;
    a.dbg_val = L.dbg_val;
    if (w->cols > MAX_K)
        return fail(JKB_E_BOUNDS, w->name, w->offset, w->cols, MAX_K,
                    "input length %zu exceeds the %zu-element activation limit of the GEMV "
                    "kernels",
                    w->cols, MAX_K);
    if (a.row_end <= a.row_begin) return JKB_OK;
    const bool diag = L.dbg_sumi != nullptr;
    // token batches of pre-quantized input (Q8 blocks, or i8 with per-token scales) share
    // weight loads
    const bool tokb = !multi && !diag && (L.m ? L.m : 1) > 1 &&
                      (L.act_kind == ACT_I8 ||
                       (L.act_scales == nullptr &&
                        (L.act_kind == ACT_Q8_0 || L.act_kind == ACT_Q8_K)));
    // grouped launches: f32 input (one token), or i8 BitLinear activations (m tokens, every
    // matrix writing [m][out_ld])
    const bool multi_i8 = multi && L.act_kind == ACT_I8;
    const size_t m = multi && !multi_i8 ? 1 : (L.m ? L.m : 1);
    const bool f32_in = L.act_kind == ACT_F32_Q8_0 || L.act_kind == ACT_F32_Q8_K;
    if ((multi && ((!f32_in && !multi_i8) || diag)) || (diag && f32_in))
        return fail(JKB_E_CAPABILITY, w->name, w->offset, w->byte_len, w->gguf_bytes,
                    "no GEMV kernel for this combination of grouped/diagnostic launch and "
                    "activation kind %d",
                    L.act_kind);
    if (!diag) {
        // outputs in a pushing peer group's buffer: every matrix of the launch in the same one
        PushTarget pt;
        for (int i = 0; i < a.nmat; i++) {
            const size_t n = multi ? L.ws[i]->rows : a.row_end - a.row_begin;
            const float *lo = a.mat[i].out;
            PushTarget ti;
            const int rc = push_lookup(lo, lo + (m - 1) * a.out_ld + n, &ti, w->name);
            if (rc) return rc;
            if (i == 0)
                pt = ti;
            else if (ti.group != pt.group)
                return fail(JKB_E_INVALID, w->name, 0, (size_t)i, (size_t)a.nmat,
                            "grouped GEMV: outputs 0 and %d are not in the same pushing peer "
                            "group's buffer (one launch pushes to one group or none)",
                            i);
        }
        a.npush = pt.n;
        for (int q = 0; q < pt.n; q++) a.push_delta[q] = pt.delta[q];
    }
    // pre-quantized or i8 activations: single or diagnostic launches
#define JKB_LAUNCH(F)                                                                   \
    return diag  ? launch_t<F, F::Act, M_DIAG>(a, m, st, "gemv_kernel<diag>")           \
           : tokb ? launch_t<F, F::Act, M_TOK>(a, m, st, "gemv_kernel<tokens>")          \
                  : launch_t<F, F::Act, M_SINGLE>(a, m, st, "gemv_kernel")
    // i8 activations over several matrices (the BitNet gate and up projections)
#define JKB_LAUNCH_I8(F)                                                                \
    if (multi) return launch_t<F, F::Act, M_MULTI>(a, m, st, "gemv_kernel<grouped i8>"); \
    JKB_LAUNCH(F)
    // f32 activations quantized by the stager S: single or grouped launches
#define JKB_LAUNCH_F32(F, S)                                                            \
    return multi ? launch_t<F, S, M_MULTI>(a, m, st, "gemv_kernel<grouped>")            \
                 : launch_t<F, S, M_SINGLE>(a, m, st, "gemv_kernel<f32>")
    switch (w->gpu_format) {
    case GF_Q4_0:
        if (L.act_kind == ACT_Q8_0) JKB_LAUNCH(FQ4_0);
        if (L.act_kind == ACT_F32_Q8_0) JKB_LAUNCH_F32(FQ4_0, ActQ80F32);
        break;
    case GF_Q8_0:
        if (L.act_kind == ACT_Q8_0) JKB_LAUNCH(FQ8_0<ActQ80>);
        if (L.act_kind == ACT_I8) { JKB_LAUNCH_I8(FQ8_0<ActI8<32>>); }
        if (L.act_kind == ACT_F32_Q8_0) JKB_LAUNCH_F32(FQ8_0<ActQ80>, ActQ80F32);
        break;
    case GF_Q4_K:
        if (L.act_kind == ACT_Q8_K) JKB_LAUNCH(FQ4_K);
        if (L.act_kind == ACT_F32_Q8_K) JKB_LAUNCH_F32(FQ4_K, ActQ8KF32);
        break;
    case GF_Q6_K:
        if (L.act_kind == ACT_Q8_K) JKB_LAUNCH(FQ6_K);
        if (L.act_kind == ACT_F32_Q8_K) JKB_LAUNCH_F32(FQ6_K, ActQ8KF32);
        break;
    case GF_Q5_0:
        if (L.act_kind == ACT_Q8_0) JKB_LAUNCH(FQ5_0);
        if (L.act_kind == ACT_F32_Q8_0) JKB_LAUNCH_F32(FQ5_0, ActQ80F32);
        break;
    case GF_Q5_K:
        if (L.act_kind == ACT_Q8_K) JKB_LAUNCH(FQ5_K);
        if (L.act_kind == ACT_F32_Q8_K) JKB_LAUNCH_F32(FQ5_K, ActQ8KF32);
        break;
    case GF_TQ2_0:
        if (L.act_kind == ACT_Q8_K) JKB_LAUNCH(FTQ2<ActQ8K>);
        if (L.act_kind == ACT_I8) { JKB_LAUNCH_I8(FTQ2<ActI8<256>>); }
        break;
    case GF_I2_S:
        if (L.act_kind == ACT_I8) { JKB_LAUNCH_I8(FI2S); }
        break;
    }
#undef JKB_LAUNCH
#undef JKB_LAUNCH_I8
#undef JKB_LAUNCH_F32
    return fail(JKB_E_CAPABILITY, w->name, w->offset, w->byte_len, w->gguf_bytes,
                "no GEMV kernel for %s weights with activation kind %d", quant_name(w->quant),
                L.act_kind);
}

// ---------------------------------------------------------------- ABI glue

static int act_kind_for(int quant) {
    return (quant == JKB_Q4_0 || quant == JKB_Q8_0 || quant == JKB_Q5_0) ? ACT_Q8_0 : ACT_Q8_K;
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

// vec_dot_*_rvv (lib.rs:1312-1319, quant.rs:999-1005, :1056-1062, :1445-1451): the scalar
// vec_dot_* validation (validate_*_dimensions), then the input quantized to BlockQ8_0 / BlockQ8K
// and the integer Q8 GEMV (vec_dot_q8_0_chunked_rvv / vec_dot_q8_k_chunked_rvv,
// quant_q8.rs:1712-1750, :3280-3317). The reference quantizes into a stack chunk per 32 / 128
// blocks; here every CTA quantizes the whole input into shared memory.
static int rvv_act_kind(int quant) {
    return (quant == JKB_Q4_0 || quant == JKB_Q8_0 || quant == JKB_Q5_0) ? ACT_F32_Q8_0
                                                                        : ACT_F32_Q8_K;
}

static int vec_dot_rvv_call(const char *fn, int quant, float *out, size_t out_len,
                            const jkb_weight *w, const float *input, size_t in_len,
                            void *stream) {
    int rc = validate_weight_call(fn, w, quant, out_len, in_len);
    if (rc) return rc;
    if (!out || !input) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    if ((rc = check_align(out, 4, fn, "output")) || (rc = check_align(input, 4, fn, "input")))
        return rc;
    GemvLaunch L{};
    L.w = w;
    L.x = input;
    L.act_kind = rvv_act_kind(quant);
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
int jkb_gemv_q5_0_q8_0(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_0 *x,
                       size_t x_len, void *stream) {
    return gemv_call("gemv_q5_0_q8_0", JKB_Q5_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_q5_0_q8_0_4x(float *out, size_t out_len, const jkb_weight *w,
                          const jkb_block_q8_0 *x, size_t x_len, void *stream) {
    return gemv_call("gemv_q5_0_q8_0", JKB_Q5_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_q5_k_q8_k(float *out, size_t out_len, const jkb_weight *w, const jkb_block_q8_k *x,
                       size_t x_len, void *stream) {
    return gemv_call("gemv_q5_k_q8_k", JKB_Q5_K, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_tq1_0_q8_k(float *out, size_t out_len, const jkb_weight *w,
                        const jkb_block_q8_k *x, size_t x_len, void *stream) {
    return gemv_call("gemv_tq1_0_q8_k", JKB_TQ1_0, out, out_len, w, x, x_len, stream);
}
int jkb_gemv_tq2_0_q8_k(float *out, size_t out_len, const jkb_weight *w,
                        const jkb_block_q8_k *x, size_t x_len, void *stream) {
    return gemv_call("gemv_tq2_0_q8_k", JKB_TQ2_0, out, out_len, w, x, x_len, stream);
}

int jkb_vec_dot_q4_k_m_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                           size_t in_len, void *stream) {
    return vec_dot_rvv_call("vec_dot_q4_k_m", JKB_Q4_K_M, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q6_k_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream) {
    return vec_dot_rvv_call("vec_dot_q6_k", JKB_Q6_K, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q8_0_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream) {
    return vec_dot_rvv_call("vec_dot_q8_0", JKB_Q8_0, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q4_0_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream) {
    return vec_dot_rvv_call("vec_dot_q4_0", JKB_Q4_0, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q5_0_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream) {
    return vec_dot_rvv_call("vec_dot_q5_0", JKB_Q5_0, out, out_len, w, input, in_len, stream);
}
int jkb_vec_dot_q5_k_rvv(float *out, size_t out_len, const jkb_weight *w, const float *input,
                         size_t in_len, void *stream) {
    return vec_dot_rvv_call("vec_dot_q5_k", JKB_Q5_K, out, out_len, w, input, in_len, stream);
}

int jkb_vec_dot_grouped_rvv(const jkb_vec_dot_item *items, size_t n_items, const float *input,
                            size_t in_len, void *stream) {
    static const char *fn = "vec_dot_grouped_rvv";
    if (!items || !input) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    if (n_items == 0 || n_items > (size_t)GEMV_MAX_MATS)
        return fail(JKB_E_BOUNDS, fn, 0, n_items, GEMV_MAX_MATS,
                    "%zu items (expected 1..%d)", n_items, GEMV_MAX_MATS);
    int rc = check_weight(items[0].w);
    if (rc) return rc;
    const int quant = items[0].w->quant;
    if (quant != JKB_Q4_0 && quant != JKB_Q8_0 && quant != JKB_Q4_K_M && quant != JKB_Q6_K &&
        quant != JKB_Q5_0 && quant != JKB_Q5_K)
        return fail(JKB_E_CAPABILITY, items[0].w->name, items[0].w->offset, items[0].w->byte_len,
                    items[0].w->gguf_bytes,
                    "%s: no vec_dot_*_rvv path for %s weights (Q4_0, Q8_0, Q4_K_M, Q6_K, Q5_0, "
                    "Q5_K)",
                    fn, quant_name(quant));
    if ((rc = check_align(input, 4, fn, "input"))) return rc;
    GemvLaunch L{};
    for (size_t i = 0; i < n_items; i++) {
        const jkb_vec_dot_item &it = items[i];
        if ((rc = validate_weight_call(fn, it.w, quant, it.out_len, in_len))) return rc;
        if (!it.out) return fail(JKB_E_INVALID, fn, i, 0, 0, "null output of item %zu", i);
        if ((rc = check_align(it.out, 4, fn, "output"))) return rc;
        L.ws[i] = it.w;
        L.outs[i] = it.out;
    }
    L.w = items[0].w;
    L.nmat = (int)n_items;
    L.x = input;
    L.act_kind = rvv_act_kind(quant);
    L.m = 1;
    if (n_items == 1) {  // one matrix: the single-matrix kernel
        L.nmat = 0;
        L.out = items[0].out;
        L.row_begin = 0;
        L.row_end = items[0].w->rows;
    }
    return launch_gemv(L, as_stream(stream));
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

int jkb_gemv_batch(float *out, size_t out_len, const jkb_weight *w, const void *x, size_t x_len,
                   size_t m, void *stream) {
    static const char *fn = "gemv_batch";
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->quant == JKB_I2_S)
        return fail(JKB_E_CAPABILITY, w->name, w->offset, w->byte_len, w->gguf_bytes,
                    "I2_S weights have no Q8 GEMV in the reference; use jkb_bitlinear_i8_batch");
    if (m == 0 || x_len != m * w->nb)
        return fail(JKB_E_BOUNDS, w->name, w->offset, x_len, m * w->nb,
                    "%s: x_blocks len %zu != m (%zu) * %zu blocks", fn, x_len, m, w->nb);
    if (out_len != m * w->rows)
        return fail(JKB_E_BOUNDS, fn, 0, out_len * 4, m * w->rows * 4,
                    "output length %zu != m (%zu) * rows (%zu)", out_len, m, w->rows);
    if (!out || !x) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    if ((rc = check_align(out, 4, fn, "output")) || (rc = check_align(x, 4, fn, "x_blocks")))
        return rc;
    const int kind = act_kind_for(w->quant);
    GemvLaunch L{};
    L.w = w;
    L.x = x;
    L.x_row_stride = w->nb * (kind == ACT_Q8_0 ? sizeof(jkb_block_q8_0) : sizeof(jkb_block_q8_k));
    L.act_kind = kind;
    L.out = out;
    L.out_ld = w->rows;
    L.row_begin = 0;
    L.row_end = w->rows;
    L.m = m;
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
