// The BitNet b1.58 feed-forward chain over device buffers:
//   act1, s1 = subln_quantize_absmax_i8(x, norm1)            (lib.rs:1042-1101)
//   gate = bitlinear_i8(W_gate, act1, s1); up = bitlinear_i8(W_up, act1, s1)   (ime.rs:882-938)
//   h = relu_squared_gate_f32(gate, up)                       (lib.rs:1111-1148)
//   act2, s2 = subln_quantize_absmax_i8(h, norm2)
//   out = bitlinear_i8(W_down, act2, s2)
// as the reference composes it (tests/empirical_challenge_m3_bitnet.rs:582-686), for m tokens.
//
// The kernels run in one stream, each launched with programmatic stream serialization so that
// the next one's weight prefetch overlaps the previous one's tail: the SubLN quantizer; the
// gate and up projections; ReLU^2 gating fused with the second SubLN quantizer (h leaves the
// CTA only as the copy kept for inspection); the down projection. The projections take the
// GEMV kernel (a single token: gate and up in one grouped launch sharing one activation
// staging per CTA; small batches: one launch per matrix, each CTA dotting every weight block
// it loads with up to eight staged tokens) or, for batches of at least 32 tokens when the
// handle holds RepackedWeights of the three matrices, the tensor-core BitLinear GEMM (one
// TMEM accumulator per BitLinear block). Every step is the single-call kernel
// of the corresponding reference function, so each intermediate equals what those calls
// produce.
#include "jkb_internal.h"

#include <cstdlib>
#include <cstring>

struct jkb_bitnet_ffn {
    uint32_t magic;
    const jkb_weight *gate, *up, *down;
    // optional RepackedWeights of the same tensors: batches of at least TC_BATCH tokens run the
    // three projections on the tensor cores (jkb_bitlinear_i8_gemm)
    const jkb_repacked_weight *rgate, *rup, *rdown;
    jkb_act_q8 *act_h, *act_i;  // their activation scratch (k = hidden, k = intermediate)
    const float *norm1, *norm2;
    float eps;
    size_t hidden, inter, m_cap;
    bool grouped;  // gate and up share one launch
    uint8_t *base;
    size_t device_bytes;
    int8_t *act1;    // [m_cap][hidden]
    float *scale1;   // [m_cap]
    float *gate_out; // [m_cap][inter]
    float *up_out;   // [m_cap][inter]
    float *relu;     // [m_cap][inter]
    int8_t *act2;    // [m_cap][inter]
    float *scale2;   // [m_cap]
};

namespace jkb {

constexpr uint32_t FFN_MAGIC = 0x4A4B4631u;  // "JKF1"

static bool check_ffn(const jkb_bitnet_ffn *f) { return f && f->magic == FFN_MAGIC; }

static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Smallest batch that takes the tensor-core projections (the GEMM's smallest token tile).
constexpr size_t TC_BATCH = 32;

static int check_repacked_pair(const jkb_repacked_weight *r, const jkb_weight *w) {
    if (!r || r->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "bitnet_ffn", 0, 0, 0, "null or destroyed repacked weight");
    if (r->quant != w->quant || r->rows != w->rows || r->cols != w->cols)
        return fail(JKB_E_BOUNDS, r->name, 0, r->rows, w->rows,
                    "repacked weight %s [%zu, %zu] does not match %s [%zu, %zu]", r->name,
                    r->rows, r->cols, w->name, w->rows, w->cols);
    return JKB_OK;
}

// The three BitLinear steps of m tokens (the activations and their scales on the device).
static int ffn_projections_up(const jkb_bitnet_ffn *f, size_t m, cudaStream_t st) {
    GemvLaunch L{};
    L.x = f->act1;
    L.x_row_stride = f->hidden;
    L.act_kind = ACT_I8;
    L.act_scales = f->scale1;
    L.out_ld = f->inter;
    L.m = m;
    if (f->grouped && m == 1) {
        L.w = f->gate;
        L.nmat = 2;
        L.ws[0] = f->gate;
        L.ws[1] = f->up;
        L.outs[0] = f->gate_out;
        L.outs[1] = f->up_out;
        return launch_gemv(L, st);
    }
    L.row_begin = 0;
    L.row_end = f->inter;
    L.w = f->gate;
    L.out = f->gate_out;
    int rc = launch_gemv(L, st);
    if (rc) return rc;
    L.w = f->up;
    L.out = f->up_out;
    return launch_gemv(L, st);
}

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_bitnet_ffn_create(const jkb_weight *w_gate, const jkb_weight *w_up,
                          const jkb_weight *w_down, const jkb_repacked_weight *r_gate,
                          const jkb_repacked_weight *r_up, const jkb_repacked_weight *r_down,
                          const float *norm1, size_t norm1_len, const float *norm2,
                          size_t norm2_len, float eps, size_t m_capacity, jkb_bitnet_ffn **out) {
    static const char *fn = "bitnet_ffn";
    if (!out) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null out");
    *out = nullptr;
    int rc;
    if ((rc = check_weight(w_gate)) || (rc = check_weight(w_up)) || (rc = check_weight(w_down)))
        return rc;
    const size_t inter = w_gate->rows, hidden = w_gate->cols;
    // each projection validated as its bitlinear_i8 call (ime.rs:660-763)
    if ((rc = validate_bitlinear(w_gate, inter, hidden)) ||
        (rc = validate_bitlinear(w_up, inter, hidden)) ||
        (rc = validate_bitlinear(w_down, hidden, inter)))
        return rc;
    if (norm1_len != hidden || norm2_len != inter)
        return fail(JKB_E_BOUNDS, "subln", 0, norm1_len, hidden,
                    "dimension mismatch: norm weights %zu / %zu for hidden %zu / intermediate %zu",
                    norm1_len, norm2_len, hidden, inter);
    if (!norm1 || !norm2) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null norm weight");
    if ((rc = check_align(norm1, 4, "subln", "norm_weight")) ||
        (rc = check_align(norm2, 4, "subln", "norm_weight")))
        return rc;
    if (m_capacity == 0) return fail(JKB_E_BOUNDS, fn, 0, 0, 0, "m_capacity must be positive");
    const bool tc = r_gate || r_up || r_down;
    if (tc && ((rc = check_repacked_pair(r_gate, w_gate)) ||
               (rc = check_repacked_pair(r_up, w_up)) ||
               (rc = check_repacked_pair(r_down, w_down))))
        return rc;
    if (inter > SUBLN_MAX_LEN || hidden > SUBLN_MAX_LEN)
        return fail(JKB_E_BOUNDS, "subln", 0, inter > hidden ? inter : hidden, SUBLN_MAX_LEN,
                    "row length exceeds the %zu-element limit of the GPU kernel", SUBLN_MAX_LEN);
    jkb_bitnet_ffn *f = (jkb_bitnet_ffn *)calloc(1, sizeof(jkb_bitnet_ffn));
    if (!f) return fail(JKB_E_INVALID, fn, 0, 0, 0, "host allocation failed");
    f->gate = w_gate;
    f->up = w_up;
    f->down = w_down;
    f->norm1 = norm1;
    f->norm2 = norm2;
    f->eps = eps;
    f->hidden = hidden;
    f->inter = inter;
    f->m_cap = m_capacity;
    f->grouped = w_gate->gpu_format == w_up->gpu_format && w_gate->p.qs_row == w_up->p.qs_row &&
                 w_gate->p.sc_row == w_up->p.sc_row && w_gate->p.i2s_scale == w_up->p.i2s_scale;
    const size_t A = 256, M = m_capacity;
    size_t off[7], o = 0;
    const size_t bytes[7] = {M * hidden, M * 4, M * inter * 4, M * inter * 4, M * inter * 4,
                             M * inter, M * 4};
    for (int i = 0; i < 7; i++) {
        off[i] = o;
        o = round_up(o + bytes[i], A);
    }
    cudaError_t e = cudaMalloc(&f->base, o);
    if (e != cudaSuccess) {
        free(f);
        return fail_cuda(e, "bitnet_ffn scratch");
    }
    f->device_bytes = o;
    f->act1 = (int8_t *)(f->base + off[0]);
    f->scale1 = (float *)(f->base + off[1]);
    f->gate_out = (float *)(f->base + off[2]);
    f->up_out = (float *)(f->base + off[3]);
    f->relu = (float *)(f->base + off[4]);
    f->act2 = (int8_t *)(f->base + off[5]);
    f->scale2 = (float *)(f->base + off[6]);
    if (tc && m_capacity >= TC_BATCH) {
        f->rgate = r_gate;
        f->rup = r_up;
        f->rdown = r_down;
        if ((rc = jkb_act_q8_create(m_capacity, hidden, &f->act_h)) ||
            (rc = jkb_act_q8_create(m_capacity, inter, &f->act_i))) {
            if (f->act_h) jkb_act_q8_destroy(f->act_h);
            cudaFree(f->base);
            free(f);
            return rc;
        }
    }
    f->magic = FFN_MAGIC;
    *out = f;
    return JKB_OK;
}

int jkb_bitnet_ffn_forward(jkb_bitnet_ffn *f, float *out, size_t out_len, const float *x,
                           size_t x_len, size_t m, void *stream) {
    static const char *fn = "bitnet_ffn";
    if (!check_ffn(f)) return fail(JKB_E_INVALID, fn, 0, 0, 0, "invalid bitnet_ffn handle");
    if (m == 0 || m > f->m_cap)
        return fail(JKB_E_BOUNDS, fn, 0, m, f->m_cap, "m=%zu outside 1..%zu (capacity)", m,
                    f->m_cap);
    if (x_len != m * f->hidden)
        return fail(JKB_E_BOUNDS, "subln", 0, x_len * 4, m * f->hidden * 4,
                    "dimension mismatch: input=%zu, expected m (%zu) * hidden (%zu)", x_len, m,
                    f->hidden);
    if (out_len != m * f->hidden)
        return fail(JKB_E_BOUNDS, f->down->name, 0, out_len * 4, m * f->hidden * 4,
                    "output length %zu != m (%zu) * hidden (%zu)", out_len, m, f->hidden);
    if (!out || !x) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null pointer");
    int rc;
    if ((rc = check_align(out, 4, fn, "output")) || (rc = check_align(x, 4, fn, "input")))
        return rc;
    cudaStream_t st = as_stream(stream);
    if ((rc = launch_subln(false, f->act1, nullptr, x, nullptr, f->norm1, m, f->hidden, f->eps,
                           f->scale1, st)))
        return rc;
    const bool tc = f->rgate && m >= TC_BATCH;
    if (tc) {
        if ((rc = jkb_bitlinear_i8_gemm(f->gate_out, m * f->inter, f->rgate, f->act1,
                                        m * f->hidden, f->scale1, m, f->act_h, stream)) ||
            (rc = jkb_bitlinear_i8_gemm(f->up_out, m * f->inter, f->rup, f->act1, m * f->hidden,
                                        f->scale1, m, f->act_h, stream)))
            return rc;
    } else if ((rc = ffn_projections_up(f, m, st))) {
        return rc;
    }
    if ((rc = launch_subln(true, f->act2, f->relu, f->gate_out, f->up_out, f->norm2, m, f->inter,
                           f->eps, f->scale2, st)))
        return rc;
    if (tc)
        return jkb_bitlinear_i8_gemm(out, out_len, f->rdown, f->act2, m * f->inter, f->scale2, m,
                                     f->act_i, stream);
    GemvLaunch L{};
    L.w = f->down;
    L.x = f->act2;
    L.x_row_stride = f->inter;
    L.act_kind = ACT_I8;
    L.act_scales = f->scale2;
    L.out = out;
    L.out_ld = f->hidden;
    L.row_begin = 0;
    L.row_end = f->hidden;
    L.m = m;
    return launch_gemv(L, st);
}

int jkb_bitnet_ffn_buffers(const jkb_bitnet_ffn *f, int8_t **act1, float **scale1,
                           float **gate, float **up, float **relu, int8_t **act2,
                           float **scale2) {
    if (!check_ffn(f))
        return fail(JKB_E_INVALID, "bitnet_ffn", 0, 0, 0, "invalid bitnet_ffn handle");
    if (act1) *act1 = f->act1;
    if (scale1) *scale1 = f->scale1;
    if (gate) *gate = f->gate_out;
    if (up) *up = f->up_out;
    if (relu) *relu = f->relu;
    if (act2) *act2 = f->act2;
    if (scale2) *scale2 = f->scale2;
    return JKB_OK;
}

int jkb_bitnet_ffn_destroy(jkb_bitnet_ffn *f) {
    if (!f) return JKB_OK;
    if (!check_ffn(f))
        return fail(JKB_E_INVALID, "bitnet_ffn", 0, 0, 0, "invalid bitnet_ffn handle");
    f->magic = 0;
    if (f->act_h) jkb_act_q8_destroy(f->act_h);
    if (f->act_i) jkb_act_q8_destroy(f->act_i);
    cudaFree(f->base);
    free(f);
    return JKB_OK;
}

}  // extern "C"
