// tcgen05 tensor-core path of the repacked block-scaled GEMM for 32-element scale groups without
// mins (Q8_0 / Q4_0 / TQ2_0 weights), bit-exact with accumulate_scaled_tile_scalar
// (repack.rs:3045-3093):
//     acc = 0; for g in K order: acc += (f32)c_g * (xs[m][g] * ws[n][g]),  c_g = sum_{k in g} xq*wq
//
// One persistent CTA per SM walks 128 x 128 output tiles (m fastest, so the CTAs working at the
// same time share weight tiles in L2). Warp roles:
//   warp 0      TMA producer: 128-byte K slices (4 groups) of the activation tile (128 rows) and
//               the weight tile (128 rows) into a 4-stage shared-memory ring, 128-byte swizzle.
//   warp 1      TMEM owner and MMA issuer: per 32-element group one tcgen05.mma.kind::i8
//               (M=128, N=128, K=32) into one of four int32 TMEM accumulators (4 x 128 columns);
//               tcgen05.commit signals the epilogue per group and frees the smem stage after its
//               four groups.
//   warps 2-9   epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 output rows), warps 2-5
//               columns 0-63 and warps 6-9 columns 64-127. Each thread converts its 64 int32 sums
//               to f32 exactly, forms xs*ws, the product and the running f32 sum in the
//               reference's order and rounding, group after group.
// The per-group scale epilogue is CUDA-core work (5 instructions per output per group) and
// bounds the kernel: the 32 int8 MACs of tensor work per output per group cost far less.
//
// Every mbarrier wait is bounded (about 2 s of globaltimer). On expiry the thread raises the
// device error word and the abort flag; the roles leave their loops, the producer waits (bounded)
// for its copies in flight, the MMA thread for its MMAs, and the CTA frees its TMEM and returns.
#include <cuda.h>

#include <cstdio>

#include "jkb_internal.h"

namespace jkb {

namespace {

constexpr int BM = 128, BN = 128, BK = 128;  // tile rows (tokens), tile columns, K bytes/stage
constexpr int STAGES = 4;
constexpr int NBUF = 4;                       // TMEM group accumulators
constexpr int TMEM_COLS = NBUF * BN;          // 512
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr int STAGE_A = BM * BK, STAGE_B = BN * BK;  // bytes
constexpr uint32_t STAGE_TX = STAGE_A + STAGE_B;
constexpr unsigned long long WAIT_NS = 2000000000ull;  // bounded waits: 2 s

struct Smem {
    uint8_t a[STAGES][STAGE_A];  // 1024-byte aligned (swizzle atoms)
    uint8_t b[STAGES][STAGE_B];
    float ws[EPI_WARPS][2][4][64];  // per epilogue warp: its 64 columns' scales of 4 groups,
                                    // transposed, double-buffered
    uint64_t full[STAGES], empty[STAGES], tfull[NBUF], tempty[NBUF], done;
    uint32_t tmem_base;
    int abort_flag;
};

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of parity `parity` to complete; false after WAIT_NS or when another role
// has aborted. The first try is inline; the polling loop is a call.
__device__ __forceinline__ bool mbar_wait_slow(uint64_t *b, uint32_t parity,
                                            volatile int *abort_flag, int *err) {
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; i++) {
        if (mbar_try(b, parity)) return true;
        if ((i & 255) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > WAIT_NS) {
                *abort_flag = 1;
                atomicOr(err, 1);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag,
                                          int *err) {
    return mbar_try(b, parity) || mbar_wait_slow(b, parity, abort_flag, err);
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
// 2-D TMA tile load (no multicast) completing on mbarrier b.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, uint64_t *b, int x,
                                            int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(b)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(b))
                 : "memory");
}
// D[tmem] (=|+=) A[smem desc] x B[smem desc]^T, int8 x int8 -> int32
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 consecutive TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// K-major operand tile of 128-byte rows with the 128-byte swizzle: 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(const void *p) {
    const uint64_t addr = smem_u32(p);
    return ((addr >> 4) & 0x3FFFull)           // start address
           | (1ull << 16)                      // leading byte offset (unused with swizzle)
           | ((uint64_t)(1024 >> 4) << 32)     // stride byte offset: next 8-row atom
           | (1ull << 46)                      // descriptor version (sm_100)
           | (2ull << 61);                     // SWIZZLE_128B
}
// kind::i8 instruction descriptor: D s32, A s8, B s8, both K-major, N = BN, M = BM.
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

__global__ void __launch_bounds__(THREADS)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const float *__restrict__ xs, const float *__restrict__ ws, int M, int G,
                      size_t row_begin, size_t sub_n, int tiles_m, int tiles_n,
                      float *__restrict__ out, int *err) {
    extern __shared__ uint8_t smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>((((uintptr_t)smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kstages = G / 4;
    const int ntiles = tiles_m * tiles_n;
    volatile int *abort_flag = &sm.abort_flag;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < NBUF; i++) {
            mbar_init(&sm.tfull[i], 1);
            mbar_init(&sm.tempty[i], EPI_WARPS);
        }
        mbar_init(&sm.done, 1);
        sm.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {  // TMEM: 512 columns for the four group accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int tm = t % tiles_m, tn = t / tiles_m;
                for (int ks = 0; ks < kstages; ks++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&sm.empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_tx(&sm.full[s], STAGE_TX);
                    tma_load_2d(sm.a[s], &tmA, &sm.full[s], ks * BK, tm * BM);
                    tma_load_2d(sm.b[s], &tmB, &sm.full[s], ks * BK, (int)(row_begin + tn * BN));
                }
            }
            if (!ok) {
                // abort: wait (bounded) until the copies already issued have landed
                for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; j++) {
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try(&sm.full[j % STAGES], (j / STAGES) & 1) &&
                           globaltimer() - t0 < WAIT_NS) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t it = 0, gc = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                for (int ks = 0; ks < kstages && ok; ks++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&sm.full[s], (it / STAGES) & 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = smem_desc(sm.a[s]), bd = smem_desc(sm.b[s]);
                    for (int j = 0; j < 4; j++, gc++) {
                        const int buf = gc % NBUF;
                        if (!mbar_wait(&sm.tempty[buf], ((gc / NBUF) & 1) ^ 1, abort_flag, err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // K step j: 32 bytes further along the 128-byte rows
                        mma_i8(tmem + buf * BN, ad + (uint64_t)(2 * j), bd + (uint64_t)(2 * j),
                               IDESC, 0u);
                        tc_commit(&sm.tfull[buf]);
                    }
                    tc_commit(&sm.empty[s]);
                }
            }
            // every MMA issued by this thread has completed before TMEM is released
            tc_commit(&sm.done);
            const uint64_t t0 = globaltimer();
            while (!mbar_try(&sm.done, 0) && globaltimer() - t0 < WAIT_NS) {
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        const int ew = warp - 2;                 // 0..7
        const int quarter = warp & 3;            // TMEM lane quarter this warp may access
        const int half = ew >> 2;                // column half: 0 -> 0..63, 1 -> 64..127
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t taddr_lane = tmem + ((uint32_t)(quarter * 32) << 16) + half * 64;
        uint32_t gc = 0;
        int blk = 0;  // scale block counter (4 groups) for the ws double buffer
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            const int tm = t % tiles_m, tn = t / tiles_m;
            const int m = tm * BM + row_in_tile;
            const size_t n0 = (size_t)tn * BN, c0n = n0 + half * 64;  // first column of the warp
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; i++) acc[i] = 0.0f;
            for (int gb = 0; gb < G && ok; gb += 4, blk++) {
                // this warp's copy of the weight scales of groups gb..gb+3 for its 64 columns:
                // lane l loads columns l and l + 32 (four groups each) and stores them transposed
                float (*wsb)[64] = sm.ws[ew][blk & 1];
                __syncwarp();  // the buffer's previous use (two blocks ago) is finished
#pragma unroll
                for (int h2 = 0; h2 < 2; h2++) {
                    const int col = lane + 32 * h2;
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (c0n + col < sub_n)
                        v = __ldg(reinterpret_cast<const float4 *>(
                            ws + (row_begin + c0n + col) * (size_t)G + gb));
                    wsb[0][col] = v.x;
                    wsb[1][col] = v.y;
                    wsb[2][col] = v.z;
                    wsb[3][col] = v.w;
                }
                float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
                if (m < M) xv = __ldg(reinterpret_cast<const float4 *>(xs + (size_t)m * G + gb));
                __syncwarp();
                for (int j = 0; j < 4; j++, gc++) {
                    const int buf = gc % NBUF;
                    if (!mbar_wait(&sm.tfull[buf], (gc / NBUF) & 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const float xj = j == 0 ? xv.x : j == 1 ? xv.y : j == 2 ? xv.z : xv.w;
#pragma unroll
                    for (int hc = 0; hc < 2; hc++) {  // 32 columns at a time
                        uint32_t c[32];
                        tmem_ld32(taddr_lane + buf * BN + 32 * hc, c);
                        tmem_ld_wait();
                        if (hc == 1) {  // the whole accumulator is in registers: release it
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&sm.tempty[buf]);
                        }
                        // exact i32 -> f32 (|c| < 2^22): bits(c + 0x4B400000) - 12582912.0f,
                        // then the reference's separately rounded products and sum (the
                        // intrinsics keep the compiler from contracting them into an FMA)
                        const float *wsj = wsb[j] + 32 * hc;
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            const float cf =
                                __fadd_rn(__int_as_float((int)c[i] + 0x4B400000), -12582912.0f);
                            const float sc = __fmul_rn(xj, wsj[i]);
                            acc[32 * hc + i] = __fadd_rn(acc[32 * hc + i], __fmul_rn(cf, sc));
                        }
                    }
                }
            }
            if (!ok) break;
            if (m < M && sub_n > c0n) {
                float *orow = out + (size_t)m * sub_n + c0n;
                const size_t nrem = sub_n - c0n;  // columns left from the warp's first one
                if (nrem >= 64 && (((uintptr_t)orow) & 15) == 0) {
#pragma unroll
                    for (int i = 0; i < 64; i += 4)
                        *reinterpret_cast<float4 *>(orow + i) =
                            make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
                } else {
#pragma unroll
                    for (int i = 0; i < 64; i++)
                        if ((size_t)i < nrem) orow[i] = acc[i];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS));
    }
}

// ---------------------------------------------------------------- host side

__device__ int g_tc_error;  // device error word of this kernel (bit 0: a bounded wait expired)

int *tc_error_word() {
    static int *ptr_by_device[128] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return nullptr;
    if (!ptr_by_device[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_tc_error) != cudaSuccess) return nullptr;
        ptr_by_device[dev] = (int *)p;
    }
    return ptr_by_device[dev];
}

// cuTensorMapEncodeTiled, resolved through the runtime's driver entry point so that the library
// does not link the driver library (it still loads on machines without a GPU driver).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

bool encode_2d(CUtensorMap *tm, const void *base, uint64_t inner, uint64_t outer, uint32_t box_in,
               uint32_t box_out) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner};  // bytes between rows (uint8 elements)
    const cuuint32_t box[2] = {box_in, box_out};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

// Smallest batch the tensor-core path takes (one 128-row MMA tile is mostly padding below it).
constexpr size_t TC_MIN_M = 32;

int gemm_tc_launch(const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                   size_t row_begin, size_t row_end, cudaStream_t st, bool *used) {
    *used = false;
    const size_t kp = w->k_pad;
    if (w->group_elems != 32 || w->mins != nullptr || kp % BK != 0 || act->m < TC_MIN_M ||
        act->k_pad != kp || (kp / 32) % 4 != 0 || act->m > (size_t)INT32_MAX)
        return JKB_OK;
    if ((((uintptr_t)w->q) & 15) || (((uintptr_t)act->q) & 15) || (((uintptr_t)w->scales) & 15) ||
        (((uintptr_t)act->x_scales) & 15))
        return JKB_OK;
    int *err = tc_error_word();
    if (!err) return JKB_OK;
    CUtensorMap tmA, tmB;
    if (!encode_2d(&tmA, act->q, kp, act->m, BK, BM) || !encode_2d(&tmB, w->q, kp, w->rows, BK, BN))
        return fail(JKB_E_CUDA, "gemm_repacked", 0, 0, 0, "cuTensorMapEncodeTiled failed");
    const size_t sub_n = row_end - row_begin;
    const int tiles_m = (int)((act->m + BM - 1) / BM), tiles_n = (int)((sub_n + BN - 1) / BN);
    const size_t ntiles = (size_t)tiles_m * tiles_n;
    const size_t smem = sizeof(Smem) + 1024;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_tc_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return fail_cuda(e, "gemm_repacked (tensor-core kernel attribute)");
        attr_set = true;
    }
    const size_t grid = ntiles < (size_t)num_sms() ? ntiles : (size_t)num_sms();
    gemm_q8_tc_kernel<<<(unsigned)grid, THREADS, smem, st>>>(
        tmA, tmB, act->x_scales, w->scales, (int)act->m, (int)(kp / 32), row_begin, sub_n, tiles_m,
        tiles_n, out, err);
    *used = true;
    return check_launch("gemm_q8_tc_kernel");
}

}  // namespace jkb

extern "C" int jkb_device_status(int32_t *flags, void *stream) {
    using namespace jkb;
    if (!flags) return fail(JKB_E_INVALID, "device_status", 0, 0, 0, "null pointer");
    int *err = tc_error_word();
    if (!err) return fail(JKB_E_CUDA, "device_status", 0, 0, 0, "no device error word");
    int v = 0;
    cudaStream_t st = as_stream(stream);
    cudaError_t e = cudaMemcpyAsync(&v, err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && v) e = cudaMemsetAsync(err, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda(e, "device_status");
    *flags = v;
    return v ? fail(JKB_E_TIMEOUT, "device_status", 0, 0, 0,
                    "a bounded wait in a tensor-core GEMM expired (flags %d)", v)
             : JKB_OK;
}
