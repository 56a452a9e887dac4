// Repacked block-scaled GEMM (repack.rs:2718-3093) over jkb_repacked_weight (i8 [rows][k_pad]
// plus per-group f32 scales / mins) and jkb_act_q8 (i8 [m][k_pad] plus per-32 scales / sums).
//
// Semantics per output (m, n), bit-exact with accumulate_scaled_tile_scalar
// (repack.rs:3045-3093): acc = 0.0; for each scale group g in K order:
//     c = sum_{k in g} xq[m][k] * wq[n][k]            (exact i32)
//     acc += (f32)c * (xs[m][b] * ws[n][g])  [- xsum[m][.] * wm[n][g]]
// with b = g for 32-element groups and g/2 for Q6_K's 16-element groups.
//
// gemm_tc.cu holds the tcgen05 tensor-core kernel used for 32-element groups; this file holds
// the dp4a tile kernel used for the other cases (16-element groups, mins, small M) and the
// ABI entry points.
#include <cstring>
#include <mutex>

#include "jkb_internal.h"

namespace jkb {

int gemm_tc_launch(const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                   size_t row_begin, size_t row_end, cudaStream_t st, bool *used);

namespace {

constexpr int TM = 64, TN = 64, TG = 32;  // tile M, tile N, K elements staged per step

// 256 threads; thread (ty, tx) owns outputs m = ty*4 + i, n = tx*4 + j (i, j < 4).
__global__ void __launch_bounds__(256) gemm_dp4a_kernel(
    const int8_t *__restrict__ xq, const float *__restrict__ xs, const float *__restrict__ xsum,
    const float *__restrict__ xs16, size_t m, size_t kp, const int8_t *__restrict__ wq,
    const float *__restrict__ ws, const float *__restrict__ wm, size_t groups, int gsz,
    size_t row_begin, size_t row_end, float *__restrict__ out) {
    // Row pitch TG + 8 keeps every 8-byte staging store aligned and spreads rows over banks.
    __shared__ __align__(16) int8_t sa[TM][TG + 8];
    __shared__ __align__(16) int8_t sb[TN][TG + 8];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const size_t m0 = (size_t)blockIdx.y * TM, n0 = row_begin + (size_t)blockIdx.x * TN;
    const size_t kb = kp / 32, kc = kp / 16;
    const size_t sub_n = row_end - row_begin;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    const int per_step = TG / gsz;  // scale groups per staged step (1 or 2)
    const size_t steps = kp / TG;
    for (size_t st = 0; st < steps; st++) {
        // stage 64 x 32 bytes of A and B (one 8-byte word per thread each)
        {
            int r = threadIdx.x >> 2, c = (threadIdx.x & 3) * 8;
            size_t gm = m0 + r, gn = n0 + r;
            uint2 va = make_uint2(0, 0), vb = make_uint2(0, 0);
            if (gm < m) va = *reinterpret_cast<const uint2 *>(xq + gm * kp + st * TG + c);
            if (gn < row_end) vb = *reinterpret_cast<const uint2 *>(wq + gn * kp + st * TG + c);
            *reinterpret_cast<uint2 *>(&sa[r][c]) = va;
            *reinterpret_cast<uint2 *>(&sb[r][c]) = vb;
        }
        __syncthreads();
        for (int gg = 0; gg < per_step; gg++) {
            const size_t g = st * per_step + gg;
            const int k0 = gg * gsz;
            int c[4][4];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) c[i][j] = 0;
            for (int k = k0; k < k0 + gsz; k += 4) {
                int a4[4], b4[4];
#pragma unroll
                for (int i = 0; i < 4; i++) a4[i] = *reinterpret_cast<const int *>(&sa[ty * 4 + i][k]);
#pragma unroll
                for (int j = 0; j < 4; j++) b4[j] = *reinterpret_cast<const int *>(&sb[tx * 4 + j][k]);
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) c[i][j] = __dp4a(a4[i], b4[j], c[i][j]);
            }
            const size_t b32 = gsz == 32 ? g : g / 2;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                size_t gm = m0 + ty * 4 + i;
                if (gm >= m) continue;
                float x_sc = xs[gm * kb + b32];
                float x_sm = 0.0f;
                if (wm) x_sm = gsz == 32 ? xsum[gm * kb + b32] : xs16[gm * kc + g];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    size_t gn = n0 + tx * 4 + j;
                    if (gn >= row_end) continue;
                    float t = __fmul_rn((float)c[i][j], __fmul_rn(x_sc, ws[gn * groups + g]));
                    if (wm) t = __fsub_rn(t, __fmul_rn(x_sm, wm[gn * groups + g]));
                    acc[i][j] = __fadd_rn(acc[i][j], t);
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        size_t gm = m0 + ty * 4 + i;
        if (gm >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            size_t gn = n0 + tx * 4 + j;
            if (gn < row_end) out[gm * sub_n + (gn - row_begin)] = acc[i][j];
        }
    }
}

}  // namespace

// execute_gemm_repacked_rows validation (repack.rs:2725-2779).
static int gemm_rows(const char *fn, float *out, size_t out_len, const jkb_repacked_weight *w,
                     const jkb_act_q8 *act, size_t row_begin, size_t row_end, bool gemv_only,
                     cudaStream_t st) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed repacked weight");
    if (!act || act->magic != ACT_MAGIC)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed activation handle");
    if (gemv_only && act->m != 1)
        return fail(JKB_E_BOUNDS, "gemv_repacked", 0, out_len * 4, w->device_bytes,
                    "gemv_repacked requires act.m() == 1, got %zu", act->m);
    if (act->k != w->cols)
        return fail(JKB_E_BOUNDS, "gemm_repacked", 0, out_len * 4, w->device_bytes,
                    "activation k %zu != weight cols %zu", act->k, w->cols);
    if (row_begin > row_end || row_end > w->rows)
        return fail(JKB_E_BOUNDS, "gemm_repacked", row_begin, row_end - row_begin, w->rows,
                    "row_range %zu..%zu out of bounds for %zu rows", row_begin, row_end, w->rows);
    size_t sub_n = row_end - row_begin;
    if (out_len != act->m * sub_n)
        return fail(JKB_E_BOUNDS, "gemm_repacked", 0, out_len * 4, act->m * sub_n * 4,
                    "output length %zu != m * row_range.len() = %zu", out_len, act->m * sub_n);
    if (sub_n == 0 || act->m == 0) return JKB_OK;
    if (!out) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null output");
    int arc = check_align(out, 4, fn, "output");
    if (!arc) arc = push_reject(out, out + out_len, fn);
    if (arc) return arc;
    bool used = false;
    int rc = gemm_tc_launch(w, act, out, row_begin, row_end, st, &used);
    if (rc || used) return rc;
    dim3 grid((unsigned)((sub_n + TN - 1) / TN), (unsigned)((act->m + TM - 1) / TM));
    gemm_dp4a_kernel<<<grid, 256, 0, st>>>(act->q, act->x_scales, act->x_sums, act->x_sums_16,
                                          act->m, act->k_pad, w->q, w->scales, w->mins,
                                          w->scale_groups, (int)w->group_elems, row_begin,
                                          row_end, out);
    return check_launch("gemm_dp4a_kernel");
}

// ---------------------------------------------------------------- allocation-free variant
// Scratch of jkb_gemm_repacked_f32_noalloc: the quantized activation batch lives in this
// file-scope device array instead of a caller-created jkb_act_q8. It holds batches with
// m * k_padded <= NOALLOC_MAX_ELEMS (2^21, e.g. 512 tokens x 4096). Every GPU that loads the
// library keeps these 4.25 MiB until process exit, and all calls share them.
constexpr size_t NOALLOC_MAX_ELEMS = size_t(1) << 21;
constexpr size_t NOALLOC_Q_BYTES = NOALLOC_MAX_ELEMS;             // i8 values [m][k_pad]
constexpr size_t NOALLOC_G32_BYTES = NOALLOC_MAX_ELEMS / 32 * 4;  // f32 per 32 elements
constexpr size_t NOALLOC_G16_BYTES = NOALLOC_MAX_ELEMS / 16 * 4;  // f32 per 16 elements
// regions, each 256-byte aligned: q | x_scales | x_sums | x_sums_16 | super_scales |
// x_scales_t | x_nsums_t (super_scales needs m * ceil(k/256) <= m * k_pad / 32 floats; the two
// transposed planes need k_pad / 32 * round_up(m, 32) floats each, under 2x x_scales when
// m >= 32, the smallest batch the tensor-core GEMM that reads them takes)
constexpr size_t NOALLOC_XT_BYTES = 2 * NOALLOC_G32_BYTES;
constexpr size_t NOALLOC_BYTES =
    NOALLOC_Q_BYTES + 3 * NOALLOC_G32_BYTES + NOALLOC_G16_BYTES + 2 * NOALLOC_XT_BYTES;
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_BYTES];

// Host code cannot use g_noalloc_scratch's name as a device address; the address comes from
// cudaGetSymbolAddress, once per device with that device current, and is cached here.
static uint8_t *noalloc_scratch(int *rc) {
    static std::mutex mu;
    static uint8_t *ptr_by_device[128] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *rc = fail_cuda(e, "gemm_repacked_f32_noalloc (cudaGetDevice)");
        return nullptr;
    }
    if (dev < 0 || dev >= 128) {
        *rc = fail(JKB_E_INVALID, "gemm_repacked_f32_noalloc", 0, 0, 0,
                   "device ordinal %d outside the supported range", dev);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!ptr_by_device[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            *rc = fail_cuda(e, "gemm_repacked_f32_noalloc (cudaGetSymbolAddress)");
            return nullptr;
        }
        ptr_by_device[dev] = static_cast<uint8_t *>(p);
    }
    return ptr_by_device[dev];
}

// A QuantizedActQ8View (caller-owned planes) as the activation record the GEMM reads. One
// token never takes the tensor-core path, so the transposed planes stay absent.
static int act_of_view(const char *fn, const jkb_act_q8_view *v, jkb_act_q8 *a) {
    if (!v) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null activation view");
    if (v->k == 0 || v->k_padded != (v->k + 31) / 32 * 32)
        return fail(JKB_E_BOUNDS, fn, 0, v->k, v->k_padded,
                    "activation view k %zu / k_padded %zu are inconsistent", v->k, v->k_padded);
    if (v->m && (!v->q || !v->x_scales || !v->x_sums || !v->x_sums_16))
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "activation view with a null plane");
    int rc;
    if ((rc = check_align(v->q, 16, fn, "view q")) ||
        (rc = check_align(v->x_scales, 4, fn, "view x_scales")) ||
        (rc = check_align(v->x_sums, 4, fn, "view x_sums")) ||
        (rc = check_align(v->x_sums_16, 4, fn, "view x_sums_16")))
        return rc;
    memset(a, 0, sizeof(*a));
    a->magic = ACT_MAGIC;
    a->m_cap = a->m = v->m;
    a->k = v->k;
    a->k_pad = v->k_padded;
    a->q = v->q;
    a->x_scales = v->x_scales;
    a->x_sums = v->x_sums;
    a->x_sums_16 = v->x_sums_16;
    a->super_scales = v->super_scales;
    a->xt_pitch = (v->m + 31) / 32 * 32;
    return JKB_OK;
}

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_gemm_repacked_f32_noalloc(float *out, size_t out_len, const jkb_repacked_weight *w,
                                  const float *input, size_t in_len, size_t m, void *stream) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "gemm_repacked_f32_noalloc", 0, 0, 0,
                    "null or destroyed weight");
    // gemm_repacked_f32_rows validation (repack.rs:4147-4161), then the scratch limit
    if (m == 0 || w->cols == 0 || in_len != m * w->cols)
        return fail(JKB_E_BOUNDS, "gemm_repacked_f32_noalloc", 0, in_len * 4, m * w->cols * 4,
                    "input length %zu != m (%zu) * cols (%zu)", in_len, m, w->cols);
    const size_t kp = (w->cols + 31) / 32 * 32;
    if (m > NOALLOC_MAX_ELEMS / kp)
        return fail(JKB_E_BOUNDS, "gemm_repacked_f32_noalloc", 0, in_len * 4,
                    NOALLOC_MAX_ELEMS,
                    "m (%zu) * k_padded (%zu) exceeds the %zu-element limit of the built-in "
                    "scratch; use jkb_gemm_repacked_f32 with a jkb_act_q8 handle",
                    m, kp, NOALLOC_MAX_ELEMS);
    int rc = JKB_OK;
    uint8_t *s = noalloc_scratch(&rc);
    if (!s) return rc;
    // A stack view over the static scratch, filled by the same quantizer and read by the same
    // GEMM as the handle-based path. Every value the GEMM reads (rows 0..m-1 of each region)
    // is written by this call's quantizer first, so nothing needs clearing.
    jkb_act_q8 view;
    memset(&view, 0, sizeof(view));
    view.magic = ACT_MAGIC;
    view.m_cap = NOALLOC_MAX_ELEMS / kp;
    view.k = w->cols;
    view.k_pad = kp;
    view.q = reinterpret_cast<int8_t *>(s);
    view.x_scales = reinterpret_cast<float *>(s + NOALLOC_Q_BYTES);
    view.x_sums = reinterpret_cast<float *>(s + NOALLOC_Q_BYTES + NOALLOC_G32_BYTES);
    view.x_sums_16 = reinterpret_cast<float *>(s + NOALLOC_Q_BYTES + 2 * NOALLOC_G32_BYTES);
    view.super_scales = reinterpret_cast<float *>(s + NOALLOC_Q_BYTES + 2 * NOALLOC_G32_BYTES +
                                                  NOALLOC_G16_BYTES);
    view.xt_pitch = (m + 31) / 32 * 32;
    const bool fits = kp / 32 * view.xt_pitch * 4 <= NOALLOC_XT_BYTES;
    uint8_t *xt = s + NOALLOC_Q_BYTES + 3 * NOALLOC_G32_BYTES + NOALLOC_G16_BYTES;
    view.x_scales_t = fits ? reinterpret_cast<float *>(xt) : nullptr;
    view.x_nsums_t = fits ? reinterpret_cast<float *>(xt + NOALLOC_XT_BYTES) : nullptr;
    view.x_nsums16_t = nullptr;  // 16-element min groups (Q2_K) take the dp4a kernel here
    rc = jkb_act_q8_quantize(&view, input, in_len, m, w->cols, stream);
    if (rc) return rc;
    return gemm_rows("gemm_repacked_f32_noalloc", out, out_len, w, &view, 0, w->rows, false,
                     as_stream(stream));
}

int jkb_gemm_repacked(float *out, size_t out_len, const jkb_repacked_weight *w,
                      const jkb_act_q8 *act, void *stream) {
    size_t rows = (w && w->magic == REPACKED_MAGIC) ? w->rows : 0;
    return gemm_rows("gemm_repacked", out, out_len, w, act, 0, rows, false, as_stream(stream));
}

int jkb_gemm_repacked_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                           const jkb_act_q8 *act, size_t row_begin, size_t row_end,
                           void *stream) {
    return gemm_rows("gemm_repacked_rows", out, out_len, w, act, row_begin, row_end, false,
                     as_stream(stream));
}

int jkb_gemv_repacked(float *out, size_t out_len, const jkb_repacked_weight *w,
                      const jkb_act_q8 *act, void *stream) {
    size_t rows = (w && w->magic == REPACKED_MAGIC) ? w->rows : 0;
    return gemm_rows("gemv_repacked", out, out_len, w, act, 0, rows, true, as_stream(stream));
}

int jkb_gemv_repacked_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                           const jkb_act_q8 *act, size_t row_begin, size_t row_end,
                           void *stream) {
    return gemm_rows("gemv_repacked_rows", out, out_len, w, act, row_begin, row_end, true,
                     as_stream(stream));
}

int jkb_bitlinear_i8_gemm(float *out, size_t out_len, const jkb_repacked_weight *w,
                          const int8_t *act_i8, size_t act_len, const float *act_scales,
                          size_t m, jkb_act_q8 *scratch, void *stream) {
    static const char *fn = "bitlinear_i8_gemm";
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed repacked weight");
    if (w->quant != JKB_TQ1_0 && w->quant != JKB_TQ2_0 && w->quant != JKB_Q8_0 &&
        w->quant != JKB_I2_S)
        return fail(JKB_E_BOUNDS, w->name, 0, w->device_bytes, w->device_bytes,
                    "unsupported quantization format for BitLinear: %s; expected TQ1_0, TQ2_0, "
                    "Q8_0, or I2_S",
                    quant_name(w->quant));
    if (!scratch || scratch->magic != ACT_MAGIC)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed activation handle");
    if (scratch->k != w->cols || scratch->k_pad != w->cols)
        return fail(JKB_E_BOUNDS, fn, 0, scratch->k, w->cols,
                    "activation handle k %zu != weight cols %zu", scratch->k, w->cols);
    if (m == 0 || m > scratch->m_cap || act_len != m * w->cols || out_len != m * w->rows)
        return fail(JKB_E_BOUNDS, w->name, 0, act_len, m * w->cols,
                    "bitlinear batch: act len %zu / out len %zu do not match m=%zu x [%zu, %zu] "
                    "(activation capacity %zu)",
                    act_len, out_len, m, w->rows, w->cols, scratch->m_cap);
    if (!out || !act_i8 || !act_scales) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    int rc;
    if ((rc = check_align(out, 4, fn, "output")) ||
        (rc = check_align(act_scales, 4, fn, "act_scales")) ||
        (rc = push_reject(out, out + out_len, fn)))
        return rc;
    cudaStream_t st = as_stream(stream);
    if ((rc = act_q8_from_i8(scratch, act_i8, act_scales, m, st))) return rc;
    bool used = false;
    rc = gemm_tc_bitlinear_launch(w, scratch, out, st, &used);
    if (rc || used) return rc;
    // small batches: the repacked GEMM over 32-element groups (within the 1e-5 contract)
    return gemm_rows(fn, out, out_len, w, scratch, 0, w->rows, false, st);
}

int jkb_gemv_repacked_view(float *out, size_t out_len, const jkb_repacked_weight *w,
                           const jkb_act_q8_view *act, void *stream) {
    size_t rows = (w && w->magic == REPACKED_MAGIC) ? w->rows : 0;
    return jkb_gemv_repacked_view_rows(out, out_len, w, act, 0, rows, stream);
}

int jkb_gemv_repacked_view_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                                const jkb_act_q8_view *act, size_t row_begin, size_t row_end,
                                void *stream) {
    jkb_act_q8 a;
    int rc = act_of_view("gemv_repacked_view_rows", act, &a);
    if (rc) return rc;
    return gemm_rows("gemv_repacked_view_rows", out, out_len, w, &a, row_begin, row_end, true,
                     as_stream(stream));
}

int jkb_gemv_repacked_f32(float *out, size_t out_len, const jkb_repacked_weight *w,
                          const float *input, size_t in_len, jkb_act_q8 *scratch, void *stream) {
    size_t rows = (w && w->magic == REPACKED_MAGIC) ? w->rows : 0;
    return jkb_gemv_repacked_f32_rows(out, out_len, w, input, in_len, 0, rows, scratch, stream);
}

int jkb_gemv_repacked_f32_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                               const float *input, size_t in_len, size_t row_begin,
                               size_t row_end, jkb_act_q8 *scratch, void *stream) {
    static const char *fn = "gemv_repacked_f32_rows";
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed weight");
    // QuantizedActQ8::quantize_row (repack.rs:531) then gemv_repacked_rows (:4014)
    if (in_len == 0)
        return fail(JKB_E_BOUNDS, "QuantizedActQ8", 0, 0, 0,
                    "activation length 0 does not match m (1) * k (0)");
    if (in_len != w->cols)
        return fail(JKB_E_BOUNDS, "gemm_repacked", 0, out_len * 4, w->device_bytes,
                    "activation k %zu != weight cols %zu", in_len, w->cols);
    int rc = jkb_act_q8_quantize(scratch, input, in_len, 1, in_len, stream);
    if (rc) return rc;
    return gemm_rows(fn, out, out_len, w, scratch, row_begin, row_end, true, as_stream(stream));
}

int jkb_gemm_repacked_f32_rows(float *out, size_t out_len, const jkb_repacked_weight *w,
                               const float *input, size_t in_len, size_t m, size_t row_begin,
                               size_t row_end, jkb_act_q8 *scratch, void *stream) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "gemm_repacked_f32", 0, 0, 0, "null or destroyed weight");
    // gemm_repacked_f32_rows validation (repack.rs:4150-4162)
    if (m == 0 || w->cols == 0 || in_len != m * w->cols)
        return fail(JKB_E_BOUNDS, "gemm_repacked_f32", 0, in_len * 4, m * w->cols * 4,
                    "input length %zu != m (%zu) * cols (%zu)", in_len, m, w->cols);
    int rc = jkb_act_q8_quantize(scratch, input, in_len, m, w->cols, stream);
    if (rc) return rc;
    return gemm_rows("gemm_repacked_f32_rows", out, out_len, w, scratch, row_begin, row_end,
                     false, as_stream(stream));
}

int jkb_gemm_repacked_f32(float *out, size_t out_len, const jkb_repacked_weight *w,
                          const float *input, size_t in_len, size_t m, jkb_act_q8 *scratch,
                          void *stream) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "gemm_repacked_f32", 0, 0, 0, "null or destroyed weight");
    // gemm_repacked_f32_rows validation (repack.rs:4147-4161)
    if (m == 0 || w->cols == 0 || in_len != m * w->cols)
        return fail(JKB_E_BOUNDS, "gemm_repacked_f32", 0, in_len * 4, m * w->cols * 4,
                    "input length %zu != m (%zu) * cols (%zu)", in_len, m, w->cols);
    int rc = jkb_act_q8_quantize(scratch, input, in_len, m, w->cols, stream);
    if (rc) return rc;
    return jkb_gemm_repacked(out, out_len, w, scratch, stream);
}

}  // extern "C"
