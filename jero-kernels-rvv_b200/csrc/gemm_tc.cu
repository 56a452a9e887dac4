// tcgen05 tensor-core path of the repacked block-scaled GEMM: 32-element scale groups (Q8_0 /
// Q4_0 / TQ2_0 / I2_S weights, and Q4_K_M with its min terms) and 16-element groups (Q6_K). Per
// output (m, n), as in accumulate_scaled_tile_scalar (repack.rs:3045-3093):
//     acc = 0; for g in K order: acc += (f32)c_g * (xs[m][b] * ws[n][g]) [- xsum[m][g] * wm[n][g]]
// with c_g = sum_{k in g} xq*wq and b the 32-element activation block of g. The integer group sums c_g are exact (int8 MMA into int32). Two
// epilogues:
//   EXACT = true   the reference's roundings: p = (f32)c * (xs*ws) rounded, [p - xsum*wm rounded,]
//                  then acc + p rounded, so every output is bit-identical to the scalar reference;
//   EXACT = false  acc = fma((f32)c, xs*ws, acc) [then fma(-xsum, wm, acc)]: one rounding fewer
//                  per product, each output within one rounding per group of the reference (far
//                  inside 1e-5 relative).
//
// The per-group f32 epilogue, not the tensor core, bounds this GEMM: per output and group the
// MMA does 32 int8 MACs (about 1/256 of an SM-clock at the int8 rate), while the epilogue needs
// an int32 -> f32 conversion, the scale product and the accumulation on CUDA cores. Per SM and
// clock a B200 issues 4 warp instructions and has 128 FMA-pipe lanes (a packed f32x2 operation
// takes two) and 64 ALU lanes. The epilogue is shaped for that budget:
//   * the conversion is cvt.rn.f32.s32, which runs on the ALU pipe (exact: |c| < 2^24);
//   * the scale product and the accumulation are packed f32x2 operations (one issue slot per
//     two outputs) on the FMA pipe;
//   * TMEM is read with the 16x256b shape, which gives each thread 4 weight rows and, per
//     8-column repeat, one adjacent token pair: a thread needs 4 weight-row scales and COLS/4
//     token scales per group, the latter as f32x2 pairs, two pairs per 16-byte shared load
//     (the quantizer stores the transposed token scales permuted within 32-token blocks).
//
// Layout. The MMA's M side is 128 weight rows (TMEM lane = weight row), its N side BN tokens
// (TMEM column = token); one persistent CTA per SM walks (weight tile, token tile) pairs, token
// tiles fastest. The 32-token tile of small batches also runs at two CTAs per SM (more tiles
// than SMs) or, in the FMA epilogue, with each tile's K stages split over a cluster of 2 or 4
// CTAs (few tiles; see KSPLIT_MAX). Warp roles:
//   warp 0     TMA producer: per stage 128 bytes of K (4 groups) of the weight tile and of the
//              token tile (128-byte swizzle), the weight scales [128 rows][4 groups] and the
//              token scales [4 groups][BN tokens] (from the transposed activation-scale plane);
//              with mins also the weight mins and the negated token group sums, laid out alike.
//   warp 1     TMEM owner and MMA issuer: one tcgen05.mma.kind::i8 (M=128, N=BN, K=32) per group
//              into its own TMEM accumulator. Groups go in rounds of GPR (two round buffers of
//              GPR accumulators alternate); one tcgen05.commit per round signals the epilogue,
//              one per stage releases the stage's operands.
//   warps 2..  epilogue, WPQ warps per TMEM lane quarter: warp w reads lanes 32*(w%4).. (its 32
//              weight rows) and COLS = BN / WPQ token columns, per round one barrier wait and,
//              per 16-lane x 32-column chunk, the GPR groups' loads in flight together before
//              one wait; it converts, scales and accumulates in registers, releases the round
//              buffer, and at the end of a tile stores out[m][n].
//
// Every mbarrier wait is bounded (about 2 s of globaltimer). On expiry the thread raises the
// device error word and the abort flag; the roles leave their loops, the producer waits (bounded)
// for its copies in flight, the MMA thread for its MMAs, and the CTA frees its TMEM and returns.
#include <cuda.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>

#include "jkb_internal.h"
#include "nibble.cuh"

namespace jkb {

namespace {

constexpr int BMW = 128;  // weight rows per tile (MMA M, TMEM lanes)
constexpr int BK = 128;   // K bytes per stage
constexpr int GPS = 4;    // scale groups per stage
constexpr unsigned long long WAIT_NS = 2000000000ull;  // bounded waits: 2 s

template <int BN_, int WPQ_, int GPR_, bool EXACT_, bool MINS_ = false, bool H16_ = false,
          int NIB_ = NIB_NONE, int AB_ = 1, int CTAS_ = 1>
struct TcCfg {
    static constexpr int BN = BN_, WPQ = WPQ_, GPR = GPR_;
    // CTAS: resident CTAs per SM. Two halve each CTA's TMEM and shared memory so that an SM runs
    // two tiles' pipelines and twice the epilogue warps at once.
    static constexpr int CTAS = CTAS_;
    static constexpr bool EXACT = EXACT_;
    // MINS: groups carry a min term (Q4_K_M, Q4_1): acc += c * (xs * ws) - x_sum * wm
    static constexpr bool MINS = MINS_;
    // H16: 16-element weight scale groups (Q6_K). The int8 MMA sums 32 elements, so a masking
    // warp writes two copies of each token tile with alternate 16-byte halves of K zeroed, and
    // every 32-element slice takes two MMAs (even and odd half-groups) into two accumulators.
    static constexpr bool H16 = H16_;
    // NIB: the weight tile arrives as 4-bit codes (a jkb_nibble_matrix, format NibFmt);
    // converter warps write its int8 values into the MMA's operand tile and its scales (and
    // mins) into the scale tiles. Two warps for the formats whose codes expand in a few integer
    // operations; IQ4_NL's code-book lookups take four, one on each SM sub-partition.
    static constexpr int NIB = NIB_;
    static constexpr int CONV = NIB == NIB_IQ4_NL ? 4 : NIB ? 2 : 0;  // converter warps
    // Q4_K_M in the fused multiply-add epilogue: the odd groups of a 256-element block (the
    // high nibbles of its bytes) enter the MMA in place as 16 * code (unsigned A) and their
    // scales carry the 1/16. Powers of two scale exactly, so the products equal the plain
    // expansion's unless a scale product falls below the normal range; the exact epilogue keeps
    // the plain expansion.
    static constexpr bool HI16 = NIB == NIB_Q4_K && !EXACT;
    // Q4_0: the codes enter the MMA as they are (unsigned A, 0..15) and a second MMA per group
    // adds a constant -8 tile times the same activations into the same accumulator: the exact
    // integer sum of (code - 8) * x without per-element offsets in the conversion.
    static constexpr bool NEG8 = NIB == NIB_Q4_0;
    // AB: K steps (32 elements each) summed into one accumulator before the epilogue scales
    // it. 1: the 32-element scale groups. 4 / 8: BitLinear over the blocks of I2_S (128
    // elements) and TQ1_0 / TQ2_0 (256), whose value is (f32)c_block * (d * s) with the block's
    // weight scale d and the token's activation scale s (ime.rs:918-929); the accumulator of a
    // block spans AB / 4 stages and every 32-element group of the block carries the same d and
    // s, so the epilogue reads group 0's.
    static constexpr int AB = AB_;
    static_assert(AB == 1 || ((AB == 4 || AB == 8) && GPR == 1 && !H16 && !MINS && !NIB),
                  "BitLinear blocks: one accumulator per round, plain int8 weights");
    static constexpr int SPL = H16 ? 2 : 1;    // accumulators per 32-element slice
    static constexpr int NA = GPR * SPL;       // accumulators per round
    static constexpr int NG = GPS * SPL;       // weight-scale groups per stage
    static constexpr int COLS = BN / WPQ;  // token columns per epilogue thread
    static constexpr int EPI = 4 * WPQ;    // epilogue warps
    static constexpr int THREADS = (2 + EPI + (H16 ? 1 : 0) + CONV) * 32;
    // TMEM: two round buffers of GPR group accumulators (BN int32 columns each)
    static constexpr int TMEM_COLS = 512 / CTAS_;
    static constexpr int SA = BMW * BK, SB = BN * BK;  // operand bytes per stage
    static constexpr int SAN = NIB ? BMW * BK / 2 : 0;  // 4-bit weight tile bytes per stage
    static constexpr int SMT = NIB ? BMW * 16 : 0;       // scale words: 16 bytes per row
    // bytes the TMA brings per stage (weight tile or its 4-bit codes, token tile, scale tiles
    // the TMA loads) and the stage's shared-memory footprint
    static constexpr int STAGE_TX =
        NIB ? SAN + SMT + SB + GPS * BN * 4 + (MINS ? GPS * BN * 4 : 0)
            : SA + SB + BMW * NG * 4 + GPS * BN * 4 + (MINS ? BMW * NG * 4 + NG * BN * 4 : 0);
    static constexpr int STAGE_SMEM =
        STAGE_TX + (H16 ? 2 * SB : 0) + (NIB ? SA + BMW * NG * 4 + (MINS ? BMW * GPS * 4 : 0) : 0);
    static constexpr int STAGES_FIT = ((NEG8 ? 184 : 200) * 1024) / CTAS_ / STAGE_SMEM;
    // BitLinear blocks run on small batches, where a CTA's time is its stages' load latency:
    // they keep up to eight stages in flight, the block-scaled GEMM six
    static constexpr int STAGES_MAX = AB_ > 1 ? 8 : 6;
    static constexpr int STAGES = STAGES_FIT > STAGES_MAX ? STAGES_MAX : STAGES_FIT;
    // KSPLIT_MAX: the most CTAs (a cluster) that may share one tile by splitting its K stages,
    // for launches with few tiles. The 32-token tile of the FMA epilogue only: its accumulators
    // (16 KB a CTA) fit beside the stages for the partial sums' exchange, and the exact
    // epilogue's single sequential sum per output cannot be split.
    static constexpr int KSPLIT_MAX =
        (BN == 32 && CTAS_ == 1 && !EXACT_ && !H16_ && NIB_ == NIB_NONE && AB_ == 1) ? 4 : 1;
    static_assert((COLS == 32 || COLS == 64) && BN % 32 == 0 && BN <= 256, "tile shape");
    static_assert(KSPLIT_MAX == 1 || COLS == 32, "K split: one 32-token column block a thread");
    static_assert(GPS % GPR == 0 && 2 * NA * BN <= TMEM_COLS, "two rounds of NA buffers");
    static_assert(!(H16 && NIB), "nibble formats use 32-element groups");
    static_assert((BMW * NG * 4) % 128 == 0 && (GPS * BN * 4) % 128 == 0 &&
                      (BMW * GPS * 4) % 128 == 0 && SAN % 128 == 0 && SMT % 128 == 0,
                  "per-stage TMA destinations stay 128-byte aligned");
    static_assert(!NIB || MINS == (NIB == NIB_Q4_1 || NIB == NIB_Q4_K), "nibble min terms");
    static_assert(EPI % 4 == 0, "four converter warps 2 + EPI .. + 3 cover the 4 sub-partitions");
};

// Every TMA destination starts on a 128-byte boundary, the 128-byte-swizzled operand tiles on
// 1024-byte boundaries (the struct itself is placed 1024-byte aligned).
template <class C>
struct TcSmem {
    alignas(1024) uint8_t a[C::STAGES][C::SA];  // weight tiles (swizzle atoms)
    alignas(1024) uint8_t b[C::STAGES][C::SB];  // token tiles
    alignas(1024) uint8_t blo[C::H16 ? C::STAGES : 1][C::H16 ? C::SB : 1024];  // H16: odd halves zeroed
    alignas(1024) uint8_t bhi[C::H16 ? C::STAGES : 1][C::H16 ? C::SB : 1024];  // H16: even halves zeroed
    alignas(128) uint8_t an[C::NIB ? C::STAGES : 1][C::NIB ? C::SAN : 128];  // NIB: codes [128][64]
    alignas(128) uint8_t mt[C::NIB ? C::STAGES : 1][C::NIB ? C::SMT : 128];  // NIB: scale words
    alignas(128) float ws[C::STAGES][BMW][C::NG];
    alignas(128) float xs[C::STAGES][GPS][C::BN];
    alignas(128) float wm[C::MINS ? C::STAGES : 1][BMW][C::NG];    // weight mins (MINS)
    // -x_sums (-x_sums_16 for 16-element groups), permuted like xs
    alignas(128) float xn[C::MINS ? C::STAGES : 1][C::NG][C::BN];
    alignas(1024) uint8_t neg8[C::NEG8 ? C::SA : 1024];  // NEG8: a weight tile of -8
    // K split: the other CTAs' accumulators, [CTA rank - 1][f32 pair][epilogue thread]
    alignas(16) uint64_t xch[C::KSPLIT_MAX > 1 ? C::KSPLIT_MAX - 1 : 1]
                            [C::KSPLIT_MAX > 1 ? C::EPI * 32 * 16 : 1];
    uint64_t full[C::STAGES], empty[C::STAGES], masked[C::STAGES], tfull[2], tempty[2], done;
    uint64_t xfull;  // K split: the other CTAs' partial sums have landed in xch
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
// has aborted.
__device__ __forceinline__ bool mbar_wait_slow(uint64_t *b, uint32_t parity, volatile int *abort_flag,
                                               int *err) {
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
// Bounded like mbar_wait_slow, with a short sleep between polls: for warps that run ahead of
// the MMA and would otherwise take issue slots from the epilogue warps.
__device__ __forceinline__ bool mbar_wait_sleepy(uint64_t *b, uint32_t parity,
                                                 volatile int *abort_flag, int *err) {
    if (mbar_try(b, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        __nanosleep(256);
        if (mbar_try(b, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > WAIT_NS) {
            *abort_flag = 1;
            atomicOr(err, 1);
            return false;
        }
    }
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
// D[tmem] = A[smem desc] x B[smem desc]^T, int8 x int8 -> int32 (D is overwritten)
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc)
        : "memory");
}
// D[tmem] += A x B^T
__device__ __forceinline__ void mma_i8_acc(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, 1, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc)
        : "memory");
}
// 16x256b.x4: 16 TMEM lanes x 32 columns; lane t gets rows t/4 and t/4 + 8 of the 16 and, per
// 8-column repeat r, registers 4r..4r+3 = (row t/4, columns 8r + 2(t%4) + {0,1}), then the same
// columns of row t/4 + 8.
__device__ __forceinline__ void tmem_ld16x256(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
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
// kind::i8 instruction descriptor: D s32, A s8, B s8, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t idesc_i8(int bn) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) |
           ((uint32_t)(BMW >> 4) << 24);
}

// Packed f32 pairs (two outputs per instruction).
__device__ __forceinline__ uint64_t pk2(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Distributed shared memory of a thread-block cluster: the address of this CTA's shared
// location p in CTA `rank` of the cluster, a store there, and a release arrival (cluster
// scope) on an mbarrier there; and a wait on a local mbarrier that acquires at cluster scope.
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_u64(uint32_t addr, uint64_t v) {
    asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_cluster(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded like mbar_wait_slow (about 2 s; false on expiry or when another role has aborted).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *b, uint32_t parity,
                                                  volatile int *abort_flag, int *err) {
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_cluster(b, parity)) return true;
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

// NIB: converts stage s (K stage ks of its tile): the 4-bit codes in an[s] to int8 values in
// a[s], in the layout the TMA's 128-byte swizzle gives (16-byte unit u of row r at
// 16 * (u ^ (r & 7))), and the scale words in mt[s] to the f32 scales (and mins) in ws[s] /
// wm[s]. Thread e of the 32 * CONV converter threads takes rows e, e + 32 * CONV, ... of the
// scales and 16-byte code chunks e, e + 32 * CONV, ... (4 per row; a chunk's low nibbles fill
// one 16-byte unit of the row, its high nibbles another).
template <class C>
__device__ __forceinline__ void nib_convert(TcSmem<C> &sm, int s, int ks, int e) {
    constexpr int F = C::NIB, N = 32 * (C::CONV ? C::CONV : 1);
#pragma unroll
    for (int i = 0; i < (BMW + N - 1) / N; i++) {
        const int r = e + i * N;
        if (r >= BMW) break;
        const uint4 v = *reinterpret_cast<const uint4 *>(&sm.mt[C::NIB ? s : 0][16 * r]);
        float4 w4, n4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (F == NIB_Q4_K) {
            // the header of the 256-element block; this stage holds its groups 4h..4h+3,
            // h = ks & 1. Their 6-bit scales and mins, one per byte (unpack_q4_q5_k_scales_mins,
            // quant_q8.rs:1818-1830; v.y, v.z, v.w = scales[0..4], [4..8], [8..12]):
            //   h = 0: sc = scales[g] & 63, m = scales[g + 4] & 63
            //   h = 1: sc = scales[g + 8] & 15 | (scales[g] >> 6) << 4,
            //          m = scales[g + 8] >> 4 | (scales[g + 4] >> 6) << 4
            const float d = nib_f16_finite(v.x & 0xFFFF), dmin = nib_f16_finite(v.x >> 16);
            uint32_t scb, mnb;
            if (ks & 1) {
                scb = (v.w & 0x0F0F0F0Fu) | ((v.y >> 2) & 0x30303030u);
                mnb = ((v.w >> 4) & 0x0F0F0F0Fu) | ((v.z >> 2) & 0x30303030u);
            } else {
                scb = v.y & 0x3F3F3F3Fu;
                mnb = v.z & 0x3F3F3F3Fu;
            }
            // groups 1 and 3 are the high nibbles: with HI16 their scale carries 1/16
            const float dh = C::HI16 ? __fmul_rn(d, 0.0625f) : d;
            w4 = make_float4(__fmul_rn(d, nib_byte_f32<0>(scb)), __fmul_rn(dh, nib_byte_f32<1>(scb)),
                             __fmul_rn(d, nib_byte_f32<2>(scb)), __fmul_rn(dh, nib_byte_f32<3>(scb)));
            n4 = make_float4(__fmul_rn(dmin, nib_byte_f32<0>(mnb)), __fmul_rn(dmin, nib_byte_f32<1>(mnb)),
                             __fmul_rn(dmin, nib_byte_f32<2>(mnb)), __fmul_rn(dmin, nib_byte_f32<3>(mnb)));
        } else if (F == NIB_Q4_1) {
            // (d, m) of the stage's 4 blocks
            w4 = make_float4(nib_f16_finite(v.x), nib_f16_finite(v.y), nib_f16_finite(v.z),
                             nib_f16_finite(v.w));
            n4 = make_float4(nib_q4_1_min(v.x >> 16), nib_q4_1_min(v.y >> 16),
                             nib_q4_1_min(v.z >> 16), nib_q4_1_min(v.w >> 16));
        } else {
            // f16 d of 8 blocks; this stage's 4 are half ks & 1
            const uint32_t d01 = (ks & 1) ? v.z : v.x, d23 = (ks & 1) ? v.w : v.y;
            w4 = make_float4(nib_d_scale(d01), nib_d_scale(d01 >> 16), nib_d_scale(d23),
                             nib_d_scale(d23 >> 16));
        }
        *reinterpret_cast<float4 *>(&sm.ws[s][r][0]) = w4;
        if (C::MINS) *reinterpret_cast<float4 *>(&sm.wm[C::MINS ? s : 0][r][0]) = n4;
    }
    static_assert((BMW * 4) % N == 0, "code chunks split evenly");
#pragma unroll
    for (int i = 0; i < BMW * 4 / N; i++) {
        const int q = e + i * N;
        const int r = q >> 2, j = q & 3;
        const uint4 c = *reinterpret_cast<const uint4 *>(&sm.an[C::NIB ? s : 0][r * 64 + 16 * j]);
        // NEG8: Q4_0 codes as they are (the -8 comes from the second MMA)
        constexpr int FV = C::NEG8 ? NIB_Q4_1 : F;
        const uint4 lo = make_uint4(
            nib_values4<FV>(c.x & 0x0F0F0F0Fu), nib_values4<FV>(c.y & 0x0F0F0F0Fu),
            nib_values4<FV>(c.z & 0x0F0F0F0Fu), nib_values4<FV>(c.w & 0x0F0F0F0Fu));
        const uint4 hi = C::HI16
            ? make_uint4(c.x & 0xF0F0F0F0u, c.y & 0xF0F0F0F0u, c.z & 0xF0F0F0F0u, c.w & 0xF0F0F0F0u)
            : make_uint4(nib_values4<FV>((c.x >> 4) & 0x0F0F0F0Fu), nib_values4<FV>((c.y >> 4) & 0x0F0F0F0Fu),
                         nib_values4<FV>((c.z >> 4) & 0x0F0F0F0Fu), nib_values4<FV>((c.w >> 4) & 0x0F0F0F0Fu));
        // Q4_K_M chunk j holds elements 64(j/2) + 16(j&1) (low nibbles) and + 32 (high); the
        // other formats' chunk j is block j: elements 32j (low) and 32j + 16 (high)
        const int ulo = F == NIB_Q4_K ? 4 * (j >> 1) + (j & 1) : 2 * j;
        const int uhi = F == NIB_Q4_K ? ulo + 2 : ulo + 1;
        uint8_t *row = &sm.a[s][r * 128];
        const int x = r & 7;
        *reinterpret_cast<uint4 *>(row + 16 * (ulo ^ x)) = lo;
        *reinterpret_cast<uint4 *>(row + 16 * (uhi ^ x)) = hi;
    }
}

template <class C>
__global__ void __launch_bounds__(C::THREADS, C::CTAS)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ CUtensorMap tmWS, const __grid_constant__ CUtensorMap tmXS,
                   const __grid_constant__ CUtensorMap tmWM, const __grid_constant__ CUtensorMap tmXN,
                   int M, int G, int row_begin, int sub_n, int tiles_w, int tiles_t,
                   int ksplit, float *__restrict__ out, int *err) {
    constexpr int BN = C::BN, STAGES = C::STAGES, GPR = C::GPR, EPI = C::EPI, COLS = C::COLS;
    constexpr int NA = C::NA, SPL = C::SPL;
    extern __shared__ uint8_t smem_raw[];
    TcSmem<C> &sm =
        *reinterpret_cast<TcSmem<C> *>((((uintptr_t)smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kstages = G / GPS;
    const int ntiles = tiles_w * tiles_t;
    volatile int *abort_flag = &sm.abort_flag;
    // K split: a cluster of nsplit CTAs shares each tile, CTA rank r (= blockIdx.x % nsplit,
    // its rank in the one-dimensional cluster) taking K stages [k_begin, k_end); rank 0 adds
    // the others' accumulators to its own in rank order and stores the tile.
    const int nsplit = C::KSPLIT_MAX > 1 ? ksplit : 1;
    const int krank = (int)blockIdx.x % nsplit;
    const int tile0 = (int)blockIdx.x / nsplit, tstride = (int)gridDim.x / nsplit;
    const int k_begin = kstages * krank / nsplit, k_end = kstages * (krank + 1) / nsplit;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1 + EPI);  // the MMA commit and every epilogue warp
            // the masking warp (H16) or the converter warps (NIB)
            mbar_init(&sm.masked[i], C::CONV ? C::CONV : 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&sm.tfull[i], 1);
            mbar_init(&sm.tempty[i], EPI);
        }
        mbar_init(&sm.done, 1);
        // one arrival per epilogue thread of every other CTA of the cluster
        mbar_init(&sm.xfull, nsplit > 1 ? EPI * 32 * (nsplit - 1) : 1);
        sm.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)),
                     "r"(C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (C::NEG8) {
        // the constant -8 tile (every byte 0xF8), read by the tensor core (async proxy)
        for (int i = threadIdx.x; i < C::SA / 16; i += C::THREADS)
            reinterpret_cast<uint4 *>(sm.neg8)[i] = make_uint4(0xF8F8F8F8u, 0xF8F8F8F8u,
                                                                0xF8F8F8F8u, 0xF8F8F8F8u);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    if (nsplit > 1)  // every CTA of the cluster runs, barriers initialized, before any DSMEM access
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                         "memory");

    // epilogue geometry: TMEM lane quarter, token-column slice
    const int quarter = warp & 3, slice = (warp - 2) >> 2;
    const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(slice * COLS);
    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = tile0; t < ntiles && ok; t += tstride) {
                const int tt = t % tiles_t, tw = t / tiles_t;
                const int wrow = row_begin + tw * BMW, tok = tt * BN;
                for (int ks = k_begin; ks < k_end; ks++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&sm.empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_tx(&sm.full[s], C::STAGE_TX);
                    if (C::NIB) {
                        tma_load_2d(sm.an[C::NIB ? s : 0], &tmW, &sm.full[s], ks * (BK / 2), wrow);
                        // 16 bytes of scale words per row: Q4_0 / IQ4_NL the f16 d of 8 blocks
                        // (this stage's 4 are half ks & 1), Q4_1 the 4 (d, m) words, Q4_K_M the
                        // header of the 256-element block (half ks & 1 of its groups)
                        const int mx = C::NIB == NIB_Q4_1 ? 4 * ks
                                     : C::NIB == NIB_Q4_K ? 4 * (ks >> 1) : 8 * (ks >> 1);
                        tma_load_2d(sm.mt[C::NIB ? s : 0], &tmWS, &sm.full[s], mx, wrow);
                    } else
                        tma_load_2d(sm.a[s], &tmW, &sm.full[s], ks * BK, wrow);
                    tma_load_2d(sm.b[s], &tmX, &sm.full[s], ks * BK, tok);
                    if (!C::NIB)
                        tma_load_2d(&sm.ws[s][0][0], &tmWS, &sm.full[s], ks * C::NG, wrow);
                    tma_load_2d(&sm.xs[s][0][0], &tmXS, &sm.full[s], tok, ks * GPS);
                    if (C::MINS) {
                        if (!C::NIB)
                            tma_load_2d(&sm.wm[s][0][0], &tmWM, &sm.full[s], ks * C::NG, wrow);
                        tma_load_2d(&sm.xn[s][0][0], &tmXN, &sm.full[s], tok, ks * C::NG);
                    }
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
            // A unsigned for the in-place high nibbles (HI16) and the raw codes (NEG8)
            constexpr uint32_t IDESC = idesc_i8(BN) & ~((C::HI16 || C::NEG8) ? (1u << 7) : 0u);
            constexpr uint32_t IDESC_S = idesc_i8(BN);
            const uint64_t nd = smem_desc(sm.neg8);
            uint32_t it = 0, rc = 0;  // stage and round counters
            bool ok = true;
            for (int t = tile0; t < ntiles && ok; t += tstride) {
                for (int ks = k_begin; ks < k_end && ok; ks++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait((C::H16 || C::NIB) ? &sm.masked[s] : &sm.full[s],
                                   (it / STAGES) & 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = smem_desc(sm.a[s]), bd = smem_desc(sm.b[s]);
                    const uint64_t bdl = smem_desc(sm.blo[C::H16 ? s : 0]),
                                   bdh = smem_desc(sm.bhi[C::H16 ? s : 0]);
                    if constexpr (C::AB > 1) {
                        // BitLinear block: its AB K steps into one accumulator (the first one
                        // overwrites), one commit to the epilogue after the block's last stage
                        const int gs = ks * GPS;
                        const bool bfirst = gs % C::AB == 0, blast = (gs + GPS) % C::AB == 0;
                        const int rb = rc & 1;
                        if (bfirst) {
                            if (!mbar_wait(&sm.tempty[rb], ((rc >> 1) & 1) ^ 1, abort_flag, err)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
                        const uint32_t d = tmem + rb * BN;
                        for (int g = 0; g < GPS; g++) {
                            if (bfirst && g == 0)
                                mma_i8(d, ad + (uint64_t)(2 * g), bd + (uint64_t)(2 * g), IDESC);
                            else
                                mma_i8_acc(d, ad + (uint64_t)(2 * g), bd + (uint64_t)(2 * g), IDESC);
                        }
                        if (blast) {
                            tc_commit(&sm.tfull[rb]);
                            rc++;
                        }
                    } else
                    for (int r = 0; r < GPS / GPR; r++, rc++) {
                        const int rb = rc & 1;
                        if (!mbar_wait(&sm.tempty[rb], ((rc >> 1) & 1) ^ 1, abort_flag, err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        for (int j = 0; j < GPR; j++) {
                            const int g = r * GPR + j;  // K step g: 32 bytes along the rows
                            const uint32_t d = tmem + (rb * NA + SPL * j) * BN;
                            if (C::H16) {
                                mma_i8(d, ad + (uint64_t)(2 * g), bdl + (uint64_t)(2 * g), IDESC);
                                mma_i8(d + BN, ad + (uint64_t)(2 * g), bdh + (uint64_t)(2 * g),
                                       IDESC);
                            } else {
                                mma_i8(d, ad + (uint64_t)(2 * g), bd + (uint64_t)(2 * g), IDESC);
                                if (C::NEG8)
                                    mma_i8_acc(d, nd + (uint64_t)(2 * g), bd + (uint64_t)(2 * g),
                                               IDESC_S);
                            }
                        }
                        tc_commit(&sm.tfull[rb]);
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
    } else if (C::H16 && warp == 2 + EPI) {
        // ------------------------------------------------ masking warp (H16)
        // Two copies of each token tile, one with the odd and one with the even 16-byte halves
        // of every 32-byte K slice zeroed. In the 128-byte swizzle, the 16-byte unit at
        // position p of row r holds logical unit p ^ (r & 7).
        uint32_t it = 0;
        bool ok = true;
        for (int t = tile0; t < ntiles && ok; t += tstride) {
            for (int ks = k_begin; ks < k_end; ks++, it++) {
                const int s = it % STAGES;
                if (!mbar_wait(&sm.full[s], (it / STAGES) & 1, abort_flag, err)) {
                    ok = false;
                    break;
                }
                const uint4 z = make_uint4(0u, 0u, 0u, 0u);
                for (int idx = lane; idx < BN * 8; idx += 32) {
                    const int row = idx >> 3, logical = (idx & 7) ^ (row & 7);
                    const uint4 v = *reinterpret_cast<const uint4 *>(&sm.b[s][16 * idx]);
                    *reinterpret_cast<uint4 *>(&sm.blo[C::H16 ? s : 0][16 * idx]) = (logical & 1) ? z : v;
                    *reinterpret_cast<uint4 *>(&sm.bhi[C::H16 ? s : 0][16 * idx]) = (logical & 1) ? v : z;
                }
                // the copies are read by the tensor core (async proxy)
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.masked[s]);
            }
        }
    } else if (C::NIB && warp >= 2 + EPI) {
        // ------------------------------------------------ converter warps (NIB)
        // Each stage, once its TMA has landed: the codes and scale words to the operand and
        // scale tiles (nib_convert, an equal share per warp), then a signal on masked for the
        // MMA and the epilogue. Running ahead of the MMA, the warps sleep between polls instead
        // of taking issue slots from the epilogue warps.
        const int e = (warp - 2 - EPI) * 32 + lane;
        uint32_t it = 0;
        bool ok = true;
        for (int t = tile0; t < ntiles && ok; t += tstride) {
            for (int ks = k_begin; ks < k_end; ks++, it++) {
                const int s = it % STAGES;
                if (!mbar_wait_sleepy(&sm.full[s], (it / STAGES) & 1, abort_flag, err)) {
                    ok = false;
                    break;
                }
                if constexpr (C::NIB != NIB_NONE) nib_convert<C>(sm, s, ks, e);
                // the operand tile is read by the tensor core (async proxy)
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.masked[s]);
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        // TMEM is read with the 16x256b shape: per load, lane t holds weight rows t/4 and
        // t/4 + 8 of a 16-lane half and, per 8-column repeat r, the token pair 8r + 2(t%4) + {0,1}.
        // A thread thus owns 4 weight rows (R_i = 32*quarter + t/4 + 8i) and COLS/4 tokens, and
        // each token pair is one f32x2 operand.
        const int r0 = quarter * 32 + (lane >> 2), kq = lane & 3;
        uint32_t it = 0, rc = 0;
        [[maybe_unused]] uint32_t xphase = 0;
        bool ok = true;
        for (int t = tile0; t < ntiles && ok; t += tstride) {
            const int tt = t % tiles_t, tw = t / tiles_t;
            // acc[cb][h][r][i]: column block cb (32 tokens), half h, repeat r, row R_{2h+i}
            uint64_t acc[COLS / 32][2][4][2];
#pragma unroll
            for (int cb = 0; cb < COLS / 32; cb++)
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int r = 0; r < 4; r++) acc[cb][h][r][0] = acc[cb][h][r][1] = 0ull;
            for (int ks = k_begin; ks < k_end && ok; ks++, it++) {
                const int s = it % STAGES;
                // NIB: the token scales come with the TMA (full), the weight scales from the
                // converter warps (masked)
                if (!mbar_wait(&sm.full[s], (it / STAGES) & 1, abort_flag, err) ||
                    (C::NIB && !mbar_wait(&sm.masked[s], (it / STAGES) & 1, abort_flag, err))) {
                    ok = false;
                    break;
                }
                float4 w4[4][SPL], m4[4][SPL];
#pragma unroll
                for (int i = 0; i < 4; i++) {
#pragma unroll
                    for (int v = 0; v < SPL; v++) {
                        w4[i][v] = *reinterpret_cast<const float4 *>(&sm.ws[s][r0 + 8 * i][4 * v]);
                        if (C::MINS)
                            m4[i][v] = *reinterpret_cast<const float4 *>(
                                &sm.wm[C::MINS ? s : 0][r0 + 8 * i][4 * v]);
                    }
                }
                const float *xbase = &sm.xs[s][0][slice * COLS + 4 * kq];
                const float *nbase = &sm.xn[C::MINS ? s : 0][0][slice * COLS + 4 * kq];
                // BitLinear blocks: one round after the block's last stage, none before
                const bool blast = C::AB == 1 || (ks * GPS + GPS) % C::AB == 0;
#pragma unroll
                for (int rr = 0; rr < (C::AB > 1 ? 1 : GPS / GPR); rr++, rc++) {
                    if (!blast) break;  // (break skips the round counter's increment)
                    const int rb = rc & 1;
                    if (!mbar_wait(&sm.tfull[rb], (rc >> 1) & 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // the round's GPR group accumulators, chunk by chunk (cb, h): all GPR loads
                    // of a chunk in flight together, one wait, then their arithmetic
#pragma unroll
                    for (int ch = 0; ch < 2 * (COLS / 32); ch++) {
                        const int cb = ch >> 1, h = ch & 1;
                        uint32_t c[NA][16];
#pragma unroll
                        for (int j = 0; j < NA; j++)
                            tmem_ld16x256(tlane + (rb * NA + j) * BN + ((uint32_t)(16 * h) << 16) +
                                              32 * cb,
                                          c[j]);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < NA; j++) {
                            // accumulator j: 32-element slice g of the stage (token-scale group)
                            // and, with H16, its even or odd 16-element half (weight-scale group gw)
                            const int g = rr * GPR + j / SPL;
                            const int gw = C::H16 ? 2 * g + (j % SPL) : g;
                            // token scales of group g, permuted within 32-token blocks so that
                            // one 16-byte load holds the pairs of repeats 2p and 2p + 1
                            const float *xg = xbase + g * BN + 32 * cb;
                            const ulonglong2 xv0 = *reinterpret_cast<const ulonglong2 *>(xg);
                            const ulonglong2 xv1 = *reinterpret_cast<const ulonglong2 *>(xg + 16);
                            uint64_t ws2[2], wm2[2];
#pragma unroll
                            for (int i = 0; i < 2; i++) {
                                const float4 &wv4 = w4[2 * h + i][gw >> 2];
                                const int gq = gw & 3;
                                const float wv = gq == 0 ? wv4.x : gq == 1 ? wv4.y : gq == 2 ? wv4.z : wv4.w;
                                ws2[i] = pk2(__float_as_uint(wv), __float_as_uint(wv));
                                if (C::MINS) {
                                    // min group = weight-scale group gw (32 or 16 elements)
                                    const float4 &mv4 = m4[2 * h + i][gw >> 2];
                                    const float mv = gq == 0 ? mv4.x : gq == 1 ? mv4.y : gq == 2 ? mv4.z : mv4.w;
                                    wm2[i] = pk2(__float_as_uint(mv), __float_as_uint(mv));
                                }
                            }
                            ulonglong2 nv0 = make_ulonglong2(0ull, 0ull), nv1 = nv0;
                            if (C::MINS) {
                                const float *ng = nbase + gw * BN + 32 * cb;
                                nv0 = *reinterpret_cast<const ulonglong2 *>(ng);
                                nv1 = *reinterpret_cast<const ulonglong2 *>(ng + 16);
                            }
#pragma unroll
                            for (int r = 0; r < 4; r++) {
                                const uint64_t xp = r == 0 ? xv0.x : r == 1 ? xv0.y : r == 2 ? xv1.x : xv1.y;
                                const uint64_t np = r == 0 ? nv0.x : r == 1 ? nv0.y : r == 2 ? nv1.x : nv1.y;
#pragma unroll
                                for (int i = 0; i < 2; i++) {
                                    // exact: |c| <= 32 * 127 * 127 (BitLinear blocks:
                                    // 256 * 2 * 128) < 2^24
                                    const uint64_t cf = pk2(
                                        __float_as_uint(__int2float_rn((int)c[j][4 * r + 2 * i])),
                                        __float_as_uint(__int2float_rn((int)c[j][4 * r + 2 * i + 1])));
                                    const uint64_t sc = mul2(ws2[i], xp);
                                    uint64_t &a = acc[cb][h][r][i];
                                    if (C::EXACT) {
                                        // separately rounded products and sums, as the reference:
                                        // acc += c * s [- x_sum * wm]
                                        float c0, c1, s0, s1, a0, a1;
                                        upk2(cf, c0, c1);
                                        upk2(sc, s0, s1);
                                        upk2(a, a0, a1);
                                        float t0 = __fmul_rn(c0, s0), t1 = __fmul_rn(c1, s1);
                                        if (C::MINS) {
                                            float n0, n1, m0, m1;
                                            upk2(np, n0, n1);
                                            upk2(wm2[i], m0, m1);
                                            t0 = __fadd_rn(t0, __fmul_rn(n0, m0));
                                            t1 = __fadd_rn(t1, __fmul_rn(n1, m1));
                                        }
                                        a0 = __fadd_rn(a0, t0);
                                        a1 = __fadd_rn(a1, t1);
                                        a = pk2(__float_as_uint(a0), __float_as_uint(a1));
                                    } else {
                                        a = fma2(cf, sc, a);
                                        if (C::MINS) a = fma2(np, wm2[i], a);
                                    }
                                }
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.tempty[rb]);
                }
                __syncwarp();  // every lane's reads of this stage's scales are done
                if (lane == 0) mbar_arrive(&sm.empty[s]);
            }
            if (!ok) break;
            if constexpr (C::KSPLIT_MAX > 1) {
                if (nsplit > 1) {
                    // K split: ranks 1.. store their accumulators into rank 0's exchange slots
                    // (pair k of epilogue thread et at k * 32 * EPI + et) and every thread
                    // arrives on its barrier; rank 0 waits and adds them in rank order, then
                    // stores the tile.
                    constexpr int ET = 32 * EPI;
                    const int et = (warp - 2) * 32 + lane;
                    if (krank > 0) {
                        const uint32_t dst = cluster_addr(&sm.xch[krank - 1][et], 0);
#pragma unroll
                        for (int h = 0; h < 2; h++)
#pragma unroll
                            for (int r = 0; r < 4; r++)
#pragma unroll
                                for (int i = 0; i < 2; i++)
                                    st_cluster_u64(dst + 8u * (uint32_t)(((h * 4 + r) * 2 + i) * ET),
                                                   acc[0][h][r][i]);
                        // each thread's release arrival orders its own stores before it
                        mbar_arrive_cluster(cluster_addr(&sm.xfull, 0));
                        continue;
                    }
                    if (!mbar_wait_cluster(&sm.xfull, xphase, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    xphase ^= 1u;
                    for (int q = 0; q < nsplit - 1; q++)
#pragma unroll
                        for (int h = 0; h < 2; h++)
#pragma unroll
                            for (int r = 0; r < 4; r++)
#pragma unroll
                                for (int i = 0; i < 2; i++)
                                    acc[0][h][r][i] = add2(
                                        acc[0][h][r][i], sm.xch[q][((h * 4 + r) * 2 + i) * ET + et]);
                }
            }
            const int m0 = tt * BN + slice * COLS + 2 * kq;
#pragma unroll
            for (int h = 0; h < 2; h++)
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const int n = tw * BMW + r0 + 8 * (2 * h + i);
                    if (n >= sub_n) continue;
#pragma unroll
                    for (int cb = 0; cb < COLS / 32; cb++)
#pragma unroll
                        for (int r = 0; r < 4; r++) {
                            const int m = m0 + 32 * cb + 8 * r;
                            float lo, hi;
                            upk2(acc[cb][h][r][i], lo, hi);
                            if (m < M) out[(size_t)m * sub_n + n] = lo;
                            if (m + 1 < M) out[(size_t)(m + 1) * sub_n + n] = hi;
                        }
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(C::TMEM_COLS));
    }
}

// ---------------------------------------------------------------- host side

// JKB_GEMM_KSPLIT=0 in the environment keeps every tile on one CTA (for measuring the K split
// against it); unset, launches with few tiles split K.
static bool k_split_allowed() {
    static const bool on = [] {
        const char *v = getenv("JKB_GEMM_KSPLIT");
        return !(v && v[0] == '0' && v[1] == 0);
    }();
    return on;
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

// Row-major 2-D tensor map: `inner` elements per row (row pitch `pitch` bytes), `outer` rows.
bool encode_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t inner,
               uint64_t outer, uint64_t pitch, uint32_t box_in, uint32_t box_out,
               CUtensorMapSwizzle swz) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {box_in, box_out};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// The weight side of one launch: its tensor maps (nibble weights: codes, scale words).
struct TcWeight {
    CUtensorMap tmW, tmWS, tmWM;
    size_t rows = 0, k = 0;
};

template <class C>
int launch_tc_common(const TcWeight &wt, const jkb_act_q8 *act, float *out, size_t row_begin,
                     size_t row_end, cudaStream_t st, int *err) {
    const size_t kp = wt.k, G = kp / 32;
    CUtensorMap tmX, tmXS, tmXN;
    if (!encode_2d(&tmX, CU_TENSOR_MAP_DATA_TYPE_UINT8, act->q, kp, act->m, kp, BK, C::BN,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&tmXS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, act->x_scales_t,
                   (act->m + 31) / 32 * 32, G, act->xt_pitch * 4, C::BN, GPS,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(JKB_E_CUDA, "gemm_repacked", 0, 0, 0, "cuTensorMapEncodeTiled failed");
    tmXN = tmXS;
    // min terms: -x_sums per 32-element group, or -x_sums_16 per 16-element group (H16)
    if (C::MINS && !encode_2d(&tmXN, CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                              C::H16 ? act->x_nsums16_t : act->x_nsums_t,
                              (act->m + 31) / 32 * 32, G * C::SPL, act->xt_pitch * 4, C::BN,
                              C::NG, CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(JKB_E_CUDA, "gemm_repacked", 0, 0, 0, "cuTensorMapEncodeTiled failed");
    const size_t sub_n = row_end - row_begin;
    const int tiles_w = (int)((sub_n + BMW - 1) / BMW), tiles_t = (int)((act->m + C::BN - 1) / C::BN);
    const size_t ntiles = (size_t)tiles_w * tiles_t;
    const size_t smem = sizeof(TcSmem<C>) + 1024;
    static bool attr_set[128] = {};  // per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda(e, "gemm_repacked (cudaGetDevice)");
    if (dev < 0 || dev >= 128)
        return fail(JKB_E_INVALID, "gemm_repacked", 0, 0, 0, "device ordinal %d out of range", dev);
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(gemm_tc_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return fail_cuda(e, "gemm_repacked (tensor-core kernel attribute)");
        attr_set[dev] = true;
    }
    // K split: with few tiles, clusters of 2 or 4 CTAs share each tile (one tile a cluster, at
    // least two K stages a CTA), so that more SMs stream weights and run epilogues.
    int nsplit = 1;
    if (C::KSPLIT_MAX > 1 && k_split_allowed()) {
        for (int c = C::KSPLIT_MAX; c >= 2; c >>= 1)
            if ((size_t)c * ntiles <= (size_t)num_sms() && G / GPS >= (size_t)(2 * c)) {
                nsplit = c;
                break;
            }
    }
    if (nsplit > 1) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(nsplit * ntiles));
        cfg.blockDim = dim3(C::THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)nsplit;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, gemm_tc_kernel<C>, wt.tmW, tmX, wt.tmWS, tmXS, wt.tmWM, tmXN,
                               (int)act->m, (int)G, (int)row_begin, (int)sub_n, tiles_w, tiles_t,
                               nsplit, out, err);
        if (e != cudaSuccess) return fail_cuda(e, "gemm_tc_kernel (K-split cluster launch)");
        return check_launch("gemm_tc_kernel");
    }
    const size_t slots = (size_t)num_sms() * C::CTAS;
    const size_t grid = ntiles < slots ? ntiles : slots;
    gemm_tc_kernel<C><<<(unsigned)grid, C::THREADS, smem, st>>>(
        wt.tmW, tmX, wt.tmWS, tmXS, wt.tmWM, tmXN, (int)act->m, (int)G, (int)row_begin,
        (int)sub_n, tiles_w, tiles_t, 1, out, err);
    return check_launch("gemm_tc_kernel");
}

// i8 repacked weight: int8 tile, f32 scales (and mins) by TMA.
template <class C>
int launch_tc(const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out, size_t row_begin,
              size_t row_end, cudaStream_t st, int *err) {
    const size_t kp = w->k_pad, G = kp / 32;
    TcWeight wt;
    wt.rows = w->rows;
    wt.k = kp;
    if (!encode_2d(&wt.tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->q, kp, w->rows, kp, BK, BMW,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&wt.tmWS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->scales, G * C::SPL, w->rows,
                   G * C::SPL * 4, C::NG, BMW, CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(JKB_E_CUDA, "gemm_repacked", 0, 0, 0, "cuTensorMapEncodeTiled failed");
    wt.tmWM = wt.tmWS;
    if (C::MINS && !encode_2d(&wt.tmWM, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->mins, G * C::SPL,
                              w->rows, G * C::SPL * 4, C::NG, BMW, CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(JKB_E_CUDA, "gemm_repacked", 0, 0, 0, "cuTensorMapEncodeTiled failed");
    return launch_tc_common<C>(wt, act, out, row_begin, row_end, st, err);
}

// Nibble weight: by TMA, without swizzle, per stage 64 bytes of codes and 16 bytes of scale
// words of each of the tile's 128 rows.
template <class C>
int launch_tc_nib(const jkb_nibble_matrix *w, const jkb_act_q8 *act, float *out,
                  size_t row_begin, size_t row_end, cudaStream_t st, int *err) {
    TcWeight wt;
    wt.rows = w->rows;
    wt.k = w->cols;
    const bool f16 = C::NIB == NIB_Q4_0 || C::NIB == NIB_IQ4_NL;
    const size_t mpitch = w->nb * w->meta_bytes;  // scale bytes per row
    if (!encode_2d(&wt.tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs, w->cols / 2, w->rows,
                   w->cols / 2, BK / 2, BMW, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_2d(&wt.tmWS, f16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32,
                   w->meta, mpitch / (f16 ? 2 : 4), w->rows, mpitch, f16 ? 8 : 4, BMW,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(JKB_E_CUDA, "gemm_nibble", 0, 0, 0, "cuTensorMapEncodeTiled failed");
    wt.tmWM = wt.tmW;  // unused
    return launch_tc_common<C>(wt, act, out, row_begin, row_end, st, err);
}

}  // namespace

// Tile widths (tokens per tile). Measured on B200 with barrier rounds (2048 x 4096 x 14336,
// FMA epilogue, normalized to full waves) the three configurations reach the same throughput
// per SM within 1 %, so the choice is the number of waves times the tile width: the padding of
// a partial last token tile and the idle SMs of a partial last wave are what differ. Ties go to
// the wider tile (less operand traffic per output).
constexpr int TILE_BN[3] = {128, 96, 64};

// The tile width with the smallest estimated time: waves of (weight tile, token tile) pairs over
// the SMs, each wave as long as one tile's token columns.
// With min terms or 16-element groups the 128-token configuration runs out of registers (it
// spills), so it is not a candidate then.
int choose_tile(size_t m, size_t sub_n, bool mins) {
    const size_t tiles_w = (sub_n + BMW - 1) / BMW, sms = (size_t)num_sms();
    int best = TILE_BN[mins ? 1 : 0];
    size_t best_t = 0;
    for (int i = mins ? 1 : 0; i < 3; i++) {
        const size_t tiles = tiles_w * ((m + TILE_BN[i] - 1) / TILE_BN[i]);
        const size_t t = (tiles + sms - 1) / sms * (size_t)TILE_BN[i];
        if (i == (mins ? 1 : 0) || t < best_t) {
            best = TILE_BN[i];
            best_t = t;
        }
    }
    return best;
}

// The three configurations: (tokens per tile, epilogue warps per lane quarter, groups per
// barrier round).
template <bool E, bool MN, bool H> using TC64 = TcCfg<64, 2, H ? 2 : 4, E, MN, H>;
template <bool E, bool MN, bool H> using TC96 = TcCfg<96, 3, H ? 1 : 2, E, MN, H>;
template <bool E, bool MN, bool H> using TC128 = TcCfg<128, 2, H ? 1 : 2, E, MN, H>;
// Small batches (16 to 32 tokens): a 32-token tile with one epilogue warp per lane quarter.
template <bool E, bool MN, bool H> using TC32 = TcCfg<32, 1, H ? 2 : 4, E, MN, H>;
// The same tile at two CTAs per SM (256 TMEM columns and half the stages each), for launches
// with more tiles than SMs: an SM then runs two tiles' pipelines and twice the epilogue warps
// at once. Measured at 16 tokens (FMA epilogue): 28672 x 8192 Q4_K_M 98.2 -> 82.9 us, Q8_0
// 80.9 -> 58.1 us; 128256 x 8192 Q6_K (16-element groups, one group a round so that the
// masking warp's CTA fits two to an SM) 539.8 -> 421.5 us. With fewer tiles than SMs the halved
// stages only slow each tile (8192 x 28672 Q4_K_M, 64 tiles: 162.5 -> 188.0 us), so those keep
// one CTA per SM.
template <bool E, bool MN>
using TC32X2 = TcCfg<32, 1, 4, E, MN, false, NIB_NONE, 1, 2>;
template <bool E, bool MN>
using TC32X2H = TcCfg<32, 1, 1, E, MN, true, NIB_NONE, 1, 2>;
// JKB_GEMM_SMALL2=0 or 1 in the environment forces the 32-token tile to one or two CTAs per SM
// (for measuring one against the other); unset, the tile count decides.
static int small_two_cta() {
    static const int v = [] {
        const char *e = getenv("JKB_GEMM_SMALL2");
        return (e && (e[0] == '0' || e[0] == '1') && e[1] == 0) ? e[0] - '0' : -1;
    }();
    return v;
}

// The nibble GEMM's configurations: the repacked GEMM's three with two converter warps; with
// IQ4_NL's four (14 warps and more leave 144 registers a thread or fewer) only the 64-token
// tile, at two groups per round, stays clear of spills.
template <int NB> constexpr bool NMINS = NB == NIB_Q4_1 || NB == NIB_Q4_K;
template <bool E, int NB>
using TN64 = TcCfg<64, 2, NB == NIB_IQ4_NL ? 2 : 4, E, NMINS<NB>, false, NB>;
template <bool E, int NB> using TN96 = TcCfg<96, 3, 2, E, NMINS<NB>, false, NB>;
template <bool E, int NB> using TN128 = TcCfg<128, 2, 2, E, NMINS<NB>, false, NB>;

std::atomic<int> g_gemm_exact{0};

// Smallest batch the tensor-core path takes (one 128-row MMA tile is mostly padding below it);
// the repacked GEMM takes batches from TC_SMALL_M tokens on its 32-token tile (measured against
// the dp4a token-batch kernels at 16 tokens on the Llama-3-70B shapes).
constexpr size_t TC_MIN_M = 32;
constexpr size_t TC_SMALL_M = 16;

// 16-element groups with min terms (Q2_K): the 64-token tile at one group a round, the only
// configuration that keeps its scales, mins and token sums in registers without spilling.
template <bool E> using TC64_H16_MINS = TcCfg<64, 2, 1, E, true, true>;

template <bool EXACT, bool MINS, bool H16>
int launch_tc_bn(int bn, const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                 size_t row_begin, size_t row_end, cudaStream_t st, int *err) {
    if constexpr (MINS && H16) {
        return launch_tc<TC64_H16_MINS<EXACT>>(w, act, out, row_begin, row_end, st, err);
    } else {
        switch (bn) {
            case 32:
                {
                    const size_t tiles = (row_end - row_begin + BMW - 1) / BMW *
                                         ((act->m + 31) / 32);
                    const int forced = small_two_cta();
                    if (forced == 1 || (forced < 0 && tiles > (size_t)num_sms())) {
                        if constexpr (H16)
                            return launch_tc<TC32X2H<EXACT, MINS>>(w, act, out, row_begin,
                                                                   row_end, st, err);
                        else
                            return launch_tc<TC32X2<EXACT, MINS>>(w, act, out, row_begin,
                                                                  row_end, st, err);
                    }
                }
                return launch_tc<TC32<EXACT, MINS, H16>>(w, act, out, row_begin, row_end, st, err);
            case 64:
                return launch_tc<TC64<EXACT, MINS, H16>>(w, act, out, row_begin, row_end, st, err);
            case 128:
                return launch_tc<TC128<EXACT, MINS, H16>>(w, act, out, row_begin, row_end, st,
                                                          err);
            default:
                return launch_tc<TC96<EXACT, MINS, H16>>(w, act, out, row_begin, row_end, st, err);
        }
    }
}

int gemm_tc_launch(const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                   size_t row_begin, size_t row_end, cudaStream_t st, bool *used) {
    *used = false;
    const size_t kp = w->k_pad;
    const bool mins = w->mins != nullptr, h16 = w->group_elems == 16;
    const float *xn = h16 ? act->x_nsums16_t : act->x_nsums_t;  // min terms' token sums
    // the 16-element groups with min terms (Q2_K) have only the 64-token tile
    const size_t min_m = (h16 && mins) ? TC_MIN_M : TC_SMALL_M;
    if ((w->group_elems != 32 && !h16) || kp % BK != 0 || act->m < min_m ||
        act->k_pad != kp ||
        act->m > (size_t)INT32_MAX || w->rows > (size_t)INT32_MAX || act->x_scales_t == nullptr ||
        (mins && xn == nullptr))
        return JKB_OK;
    if ((((uintptr_t)w->q) & 15) || (((uintptr_t)act->q) & 15) || (((uintptr_t)w->scales) & 15) ||
        (((uintptr_t)act->x_scales_t) & 15) || (act->xt_pitch & 31) ||
        (mins && ((((uintptr_t)w->mins) & 15) || (((uintptr_t)xn) & 15))))
        return JKB_OK;
    int *err = device_error_word();
    if (!err) return JKB_OK;
    *used = true;
    const int bn = act->m <= 32 ? 32 : choose_tile(act->m, row_end - row_begin, mins || h16);
    const bool exact = g_gemm_exact.load(std::memory_order_relaxed);
    if (h16 && mins)  // Q2_K: 16-element groups with min terms
        return exact ? launch_tc_bn<true, true, true>(bn, w, act, out, row_begin, row_end, st, err)
                     : launch_tc_bn<false, true, true>(bn, w, act, out, row_begin, row_end, st, err);
    if (h16)
        return exact ? launch_tc_bn<true, false, true>(bn, w, act, out, row_begin, row_end, st, err)
                     : launch_tc_bn<false, false, true>(bn, w, act, out, row_begin, row_end, st, err);
    if (mins)
        return exact ? launch_tc_bn<true, true, false>(bn, w, act, out, row_begin, row_end, st, err)
                     : launch_tc_bn<false, true, false>(bn, w, act, out, row_begin, row_end, st, err);
    return exact ? launch_tc_bn<true, false, false>(bn, w, act, out, row_begin, row_end, st, err)
                 : launch_tc_bn<false, false, false>(bn, w, act, out, row_begin, row_end, st, err);
}


// BitLinear configurations: one accumulator per block (GPR = 1), AB K steps per block. The
// 32-token tile (one epilogue warp per lane quarter) serves matrices with few 128-row weight
// tiles, where the token tiles are what spreads the work over the SMs.
template <bool E, int AB> using TB32 = TcCfg<32, 1, 1, E, false, false, NIB_NONE, AB>;
template <bool E, int AB> using TB64 = TcCfg<64, 2, 1, E, false, false, NIB_NONE, AB>;
template <bool E, int AB> using TB96 = TcCfg<96, 3, 1, E, false, false, NIB_NONE, AB>;
template <bool E, int AB> using TB128 = TcCfg<128, 2, 1, E, false, false, NIB_NONE, AB>;

template <bool EXACT, int AB>
int launch_bl_bn(int bn, const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                 cudaStream_t st, int *err) {
    switch (bn) {
        case 32: return launch_tc<TB32<EXACT, AB>>(w, act, out, 0, w->rows, st, err);
        case 64: return launch_tc<TB64<EXACT, AB>>(w, act, out, 0, w->rows, st, err);
        case 128: return launch_tc<TB128<EXACT, AB>>(w, act, out, 0, w->rows, st, err);
        default: return launch_tc<TB96<EXACT, AB>>(w, act, out, 0, w->rows, st, err);
    }
}

// Tensor-core BitLinear over a token batch (bitlinear_i8 per token, ime.rs:882-938): a
// repacked TQ1_0 / TQ2_0 / I2_S / Q8_0 weight and i8 activations whose every 32-element group
// carries its token's scale (act_q8_from_i8). A TQ block's 8 K steps (I2_S: 4) sum into one
// accumulator and the epilogue adds (f32)c_block * (d * s) per block in K order, so with the
// exact epilogue each output is the reference's row sum bit for bit; Q8_0's 32-element blocks
// are the plain GEMM's groups. Conditions as gemm_tc_launch; *used reports whether it ran.
int gemm_tc_bitlinear_launch(const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                             cudaStream_t st, bool *used) {
    const int ab = (w->quant == JKB_TQ1_0 || w->quant == JKB_TQ2_0) ? 8
                   : w->quant == JKB_I2_S                          ? 4
                                                                   : 1;
    if (ab == 1) return gemm_tc_launch(w, act, out, 0, w->rows, st, used);
    *used = false;
    const size_t kp = w->k_pad;
    if (w->group_elems != 32 || w->mins || kp % (32 * (size_t)ab) != 0 || kp % BK != 0 ||
        act->m < TC_MIN_M || act->k_pad != kp || act->m > (size_t)INT32_MAX ||
        w->rows > (size_t)INT32_MAX || act->x_scales_t == nullptr)
        return JKB_OK;
    if ((((uintptr_t)w->q) & 15) || (((uintptr_t)act->q) & 15) || (((uintptr_t)w->scales) & 15) ||
        (((uintptr_t)act->x_scales_t) & 15) || (act->xt_pitch & 31))
        return JKB_OK;
    int *err = device_error_word();
    if (!err) return JKB_OK;
    *used = true;
    // the repacked GEMM's choice, or the 32-token tile when it takes fewer tile-widths of
    // waves (small weight matrices: BitNet's 2560-row down projection has 20 weight tiles)
    int bn = choose_tile(act->m, w->rows, false);
    {
        const size_t tiles_w = (w->rows + BMW - 1) / BMW, sms = (size_t)num_sms();
        auto cost = [&](size_t b) {
            const size_t tiles = tiles_w * ((act->m + b - 1) / b);
            return (tiles + sms - 1) / sms * b;
        };
        if (cost(32) < cost((size_t)bn)) bn = 32;
    }
    const bool exact = g_gemm_exact.load(std::memory_order_relaxed);
    if (ab == 8)
        return exact ? launch_bl_bn<true, 8>(bn, w, act, out, st, err)
                     : launch_bl_bn<false, 8>(bn, w, act, out, st, err);
    return exact ? launch_bl_bn<true, 4>(bn, w, act, out, st, err)
                 : launch_bl_bn<false, 4>(bn, w, act, out, st, err);
}

template <bool EXACT, int NB>
int launch_nib_bn(int bn, const jkb_nibble_matrix *w, const jkb_act_q8 *act, float *out,
                  size_t row_begin, size_t row_end, cudaStream_t st, int *err) {
    if constexpr (NB != NIB_IQ4_NL) {
        if (bn == 96)
            return launch_tc_nib<TN96<EXACT, NB>>(w, act, out, row_begin, row_end, st, err);
        if constexpr (!NMINS<NB>)
            if (bn == 128)
                return launch_tc_nib<TN128<EXACT, NB>>(w, act, out, row_begin, row_end, st, err);
    }
    return launch_tc_nib<TN64<EXACT, NB>>(w, act, out, row_begin, row_end, st, err);
}

template <int NB>
int launch_nib_fmt(bool exact, const jkb_nibble_matrix *w, const jkb_act_q8 *act, float *out,
                   size_t row_begin, size_t row_end, cudaStream_t st, int *err) {
    // IQ4_NL: the 64-token tile only; the others choose like the repacked GEMM
    const int bn = NB == NIB_IQ4_NL ? 64 : choose_tile(act->m, row_end - row_begin, NMINS<NB>);
    return exact ? launch_nib_bn<true, NB>(bn, w, act, out, row_begin, row_end, st, err)
                 : launch_nib_bn<false, NB>(bn, w, act, out, row_begin, row_end, st, err);
}

// Smallest batch for which the tensor-core path beats the nibble row kernel. Measured on B200:
// a row-kernel call costs about 2.85 ps per (weight row, 32-element block, token), a
// tensor-core call about 1.4 us per 128-element K stage per wave of 128-row weight tiles over
// the SMs, independent of the batch up to its 64-token tile. Equal at
// m = 1.4 us * waves / (4 * 2.85 ps * rows), about 122880 * waves / rows; never below 8 tokens,
// always from 32.
size_t nibble_tc_min_m(size_t rows) {
    const size_t tiles = (rows + BMW - 1) / BMW, sms = (size_t)num_sms();
    const size_t waves = (tiles + sms - 1) / sms;
    size_t m = (122880 * waves + rows - 1) / (rows ? rows : 1);
    return m < 8 ? 8 : m > TC_MIN_M ? TC_MIN_M : m;
}

// Tensor-core path of the compact nibble GEMM: taken for batches of at least nibble_tc_min_m
// tokens with K a multiple of 128 (the stage depth) and 16-byte scale rows; *used reports
// whether it ran.
int gemm_tc_nibble_launch(const jkb_nibble_matrix *w, const jkb_act_q8 *act, float *out,
                          size_t row_begin, size_t row_end, cudaStream_t st, bool *used) {
    *used = false;
    const size_t k = w->cols;
    const bool mins = w->quant == JKB_Q4_1 || w->quant == JKB_Q4_K_M;
    // the scale-word rows must be 16-byte multiples (the TMA's row pitch): Q4_0 / IQ4_NL need
    // cols % 256 == 0, the other formats hold already at cols % 128 == 0
    const size_t mpitch = w->nb * w->meta_bytes;
    if (k % BK != 0 || mpitch % 16 != 0 || act->m < nibble_tc_min_m(w->rows) ||
        act->k_pad != k ||
        act->m > (size_t)INT32_MAX ||
        w->rows > (size_t)INT32_MAX || act->x_scales_t == nullptr ||
        (mins && act->x_nsums_t == nullptr))
        return JKB_OK;
    if ((((uintptr_t)w->qs) & 15) || (((uintptr_t)w->meta) & 15) || (((uintptr_t)act->q) & 15) ||
        (((uintptr_t)act->x_scales_t) & 15) || (act->xt_pitch & 31) ||
        (mins && (((uintptr_t)act->x_nsums_t) & 15)))
        return JKB_OK;
    int *err = device_error_word();
    if (!err) return JKB_OK;
    *used = true;
    const bool exact = g_gemm_exact.load(std::memory_order_relaxed);
    switch (w->quant) {
        case JKB_Q4_0:
            return launch_nib_fmt<NIB_Q4_0>(exact, w, act, out, row_begin, row_end, st, err);
        case JKB_Q4_1:
            return launch_nib_fmt<NIB_Q4_1>(exact, w, act, out, row_begin, row_end, st, err);
        case JKB_IQ4_NL:
            return launch_nib_fmt<NIB_IQ4_NL>(exact, w, act, out, row_begin, row_end, st, err);
        default:
            return launch_nib_fmt<NIB_Q4_K>(exact, w, act, out, row_begin, row_end, st, err);
    }
}


}  // namespace jkb

extern "C" int jkb_gemm_set_exact(int exact) {
    jkb::g_gemm_exact.store(exact ? 1 : 0, std::memory_order_relaxed);
    return JKB_OK;
}

extern "C" int jkb_gemm_get_exact(void) { return jkb::g_gemm_exact.load(std::memory_order_relaxed); }
