// Device scratch arenas (the GPU counterpart of jero_core's ScratchWorkspace and ScratchScope),
// the in-scratch activation quantizers (quant_q8.rs:398-444, :598-641) and QuantizedActQ8View
// (repack.rs:806-1090): callers that quantize a decode row per token carve its Q8 blocks or its
// QuantizedActQ8 planes from one arena they set up once, so the per-token calls allocate
// nothing.
//
// An arena is a bump allocator over one device region: every carve starts at a 128-byte
// boundary (SCRATCH_ALIGNMENT) and advances the cursor; reset() rewinds to 0; a scope is a saved
// cursor that scope_end() rewinds to (what dropping a ScratchScope does). A failed call leaves
// the cursor where it was (fail closed, quant_q8.rs:3805-3819).
#include <cstring>

#include "jkb_internal.h"

struct jkb_scratch {
    uint32_t magic;
    uint8_t *base;
    size_t cap, used;
    bool owned;  // allocated by jkb_scratch_create (freed by destroy) or wrapped caller memory
};

namespace jkb {
namespace {

constexpr uint32_t SCRATCH_MAGIC = 0x5C7A7C4Bu;
constexpr size_t SCRATCH_ALIGN = JKB_SCRATCH_ALIGNMENT;

size_t align_up(size_t n) { return (n + SCRATCH_ALIGN - 1) / SCRATCH_ALIGN * SCRATCH_ALIGN; }

bool check_ws(const jkb_scratch *ws) { return ws && ws->magic == SCRATCH_MAGIC; }

// Carves `n` bytes (a 128-byte aligned start) or fails with the arena untouched.
int carve(jkb_scratch *ws, const char *fn, size_t n, uint8_t **out) {
    const size_t at = align_up(ws->used);
    if (at > ws->cap || n > ws->cap - at)
        return fail(JKB_E_BOUNDS, fn, at, n, ws->cap > ws->used ? ws->cap - ws->used : 0,
                    "%s: scratch exhausted: %zu bytes requested, %zu remaining", fn, n,
                    ws->cap > ws->used ? ws->cap - ws->used : 0);
    *out = ws->base + at;
    ws->used = at + n;
    return JKB_OK;
}

// quantize_row_q8_0_in_scratch / _in_scope and the Q8_K pair: validate, carve the blocks, then
// quantize into them; any failure rewinds the cursor.
int quantize_in_scratch(const char *fn, const float *x, size_t x_len, jkb_scratch *ws,
                        void **out, size_t block_elems, size_t block_bytes, void *stream) {
    if (!out) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null out");
    *out = nullptr;
    if (!check_ws(ws)) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed scratch");
    // validate_activation_input (quant_q8.rs:111-131)
    if (x_len == 0 || x_len % block_elems != 0)
        return fail(JKB_E_BOUNDS, fn, 0, x_len * 4, 0,
                    "%s: input length %zu must be a positive multiple of %zu", fn, x_len,
                    block_elems);
    if (!x) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null input");
    const size_t nb = x_len / block_elems, saved = ws->used;
    uint8_t *blocks = nullptr;
    int rc = carve(ws, fn, nb * block_bytes, &blocks);
    if (rc) return rc;
    rc = block_elems == 32
             ? jkb_quantize_row_q8_0_f32(x, x_len, (jkb_block_q8_0 *)blocks, nb, stream)
             : jkb_quantize_row_q8_k(x, x_len, (jkb_block_q8_k *)blocks, nb, stream);
    if (rc) {
        ws->used = saved;
        return rc;
    }
    *out = blocks;
    return JKB_OK;
}

// The planes of a one-row QuantizedActQ8View, each at a 128-byte boundary: q [k_pad],
// x_scales and x_sums [k_pad / 32], x_sums_16 [k_pad / 16], super_scales [ceil(k / 256)].
struct RowPlanes {
    size_t q, g32, g16, sup;
};
RowPlanes row_planes(size_t k) {
    const size_t kp = (k + 31) / 32 * 32;
    return {kp, kp / 32 * 4, kp / 16 * 4, (k + 255) / 256 * 4};
}

int view_in_scratch(const char *fn, const float *act, size_t k, jkb_scratch *ws,
                    jkb_act_q8_view *out, void *stream) {
    if (!out) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null out");
    memset(out, 0, sizeof(*out));
    if (!check_ws(ws)) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed scratch");
    if (k == 0)  // repack.rs:874-882
        return fail(JKB_E_BOUNDS, "QuantizedActQ8View", 0, 0, 0,
                    "activation length must be non-empty");
    if (!act) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null input");
    const RowPlanes p = row_planes(k);
    const size_t need = align_up(p.q) + 2 * align_up(p.g32) + align_up(p.g16) + p.sup;
    const size_t at = align_up(ws->used);
    if (at > ws->cap || need > ws->cap - at)
        return fail(JKB_E_BOUNDS, "QuantizedActQ8View", at, need,
                    ws->cap > ws->used ? ws->cap - ws->used : 0,
                    "%s: scratch exhausted: %zu bytes requested, %zu remaining", fn, need,
                    ws->cap > ws->used ? ws->cap - ws->used : 0);
    const size_t saved = ws->used;
    uint8_t *q, *xs, *xsum, *xs16, *sup;
    carve(ws, fn, p.q, &q);
    carve(ws, fn, p.g32, &xs);
    carve(ws, fn, p.g32, &xsum);
    carve(ws, fn, p.g16, &xs16);
    carve(ws, fn, p.sup, &sup);
    // the same quantizer as QuantizedActQ8::quantize_into, on a one-row view of these planes
    jkb_act_q8 a;
    memset(&a, 0, sizeof(a));
    a.magic = ACT_MAGIC;
    a.m_cap = 1;
    a.k = k;
    a.k_pad = p.q;
    a.q = (int8_t *)q;
    a.x_scales = (float *)xs;
    a.x_sums = (float *)xsum;
    a.x_sums_16 = (float *)xs16;
    a.super_scales = (float *)sup;
    a.xt_pitch = 32;  // no transposed planes: one token never takes the tensor-core GEMM
    int rc = jkb_act_q8_quantize(&a, act, k, 1, k, stream);
    if (rc) {
        ws->used = saved;
        return rc;
    }
    out->m = 1;
    out->k = k;
    out->k_padded = p.q;
    out->q = a.q;
    out->x_scales = a.x_scales;
    out->x_sums = a.x_sums;
    out->x_sums_16 = a.x_sums_16;
    out->super_scales = a.super_scales;
    return JKB_OK;
}

}  // namespace
}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_scratch_create(size_t bytes, jkb_scratch **out) {
    if (!out) return fail(JKB_E_INVALID, "ScratchWorkspace", 0, 0, 0, "null out");
    *out = nullptr;
    if (bytes == 0)
        return fail(JKB_E_BOUNDS, "ScratchWorkspace", 0, 0, 0, "capacity must be non-zero");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return fail_cuda(e, "ScratchWorkspace::new");
    *out = new jkb_scratch{SCRATCH_MAGIC, (uint8_t *)p, bytes, 0, true};
    return JKB_OK;
}

int jkb_scratch_wrap(void *device_base, size_t bytes, jkb_scratch **out) {
    if (!out) return fail(JKB_E_INVALID, "ScratchWorkspace", 0, 0, 0, "null out");
    *out = nullptr;
    if (!device_base || bytes == 0)
        return fail(JKB_E_BOUNDS, "ScratchWorkspace", 0, bytes, 0,
                    "a wrapped region needs a non-null base and a non-zero size");
    if (((uintptr_t)device_base) % SCRATCH_ALIGN)
        return fail(JKB_E_BOUNDS, "ScratchWorkspace", 0, bytes, 0,
                    "wrapped region base is not %zu-byte aligned", SCRATCH_ALIGN);
    *out = new jkb_scratch{SCRATCH_MAGIC, (uint8_t *)device_base, bytes, 0, false};
    return JKB_OK;
}

int jkb_scratch_destroy(jkb_scratch *ws) {
    if (!check_ws(ws)) return fail(JKB_E_INVALID, "ScratchWorkspace", 0, 0, 0, "null or destroyed");
    ws->magic = 0;
    if (ws->owned) cudaFree(ws->base);
    delete ws;
    return JKB_OK;
}

int jkb_scratch_reset(jkb_scratch *ws) {
    if (!check_ws(ws)) return fail(JKB_E_INVALID, "ScratchWorkspace", 0, 0, 0, "null or destroyed");
    ws->used = 0;
    return JKB_OK;
}

int jkb_scratch_used_bytes(const jkb_scratch *ws, size_t *used) {
    if (!check_ws(ws) || !used)
        return fail(JKB_E_INVALID, "ScratchWorkspace", 0, 0, 0, "null or destroyed");
    *used = ws->used;
    return JKB_OK;
}

int jkb_scratch_remaining_bytes(const jkb_scratch *ws, size_t *remaining) {
    if (!check_ws(ws) || !remaining)
        return fail(JKB_E_INVALID, "ScratchWorkspace", 0, 0, 0, "null or destroyed");
    *remaining = ws->cap - ws->used;
    return JKB_OK;
}

int jkb_scratch_alloc(jkb_scratch *ws, size_t bytes, void **out) {
    if (!check_ws(ws) || !out)
        return fail(JKB_E_INVALID, "ScratchWorkspace", 0, 0, 0, "null or destroyed");
    uint8_t *p = nullptr;
    int rc = carve(ws, "ScratchWorkspace::alloc", bytes, &p);
    *out = rc ? nullptr : p;
    return rc;
}

int jkb_scratch_scope_begin(const jkb_scratch *ws, size_t *mark) {
    if (!check_ws(ws) || !mark)
        return fail(JKB_E_INVALID, "ScratchScope", 0, 0, 0, "null or destroyed");
    *mark = ws->used;
    return JKB_OK;
}

int jkb_scratch_scope_end(jkb_scratch *ws, size_t mark) {
    if (!check_ws(ws)) return fail(JKB_E_INVALID, "ScratchScope", 0, 0, 0, "null or destroyed");
    if (mark > ws->used)
        return fail(JKB_E_BOUNDS, "ScratchScope", mark, 0, ws->used,
                    "scope mark %zu is past the cursor %zu", mark, ws->used);
    ws->used = mark;
    return JKB_OK;
}

int jkb_quantize_row_q8_0_in_scratch(const float *x, size_t x_len, jkb_scratch *ws,
                                     jkb_block_q8_0 **out, void *stream) {
    return quantize_in_scratch("quantize_row_q8_0_in_scratch", x, x_len, ws, (void **)out, 32,
                               sizeof(jkb_block_q8_0), stream);
}

int jkb_quantize_row_q8_0_in_scope(const float *x, size_t x_len, jkb_scratch *ws,
                                   jkb_block_q8_0 **out, void *stream) {
    return quantize_in_scratch("quantize_row_q8_0_in_scope", x, x_len, ws, (void **)out, 32,
                               sizeof(jkb_block_q8_0), stream);
}

int jkb_quantize_row_q8_k_in_scratch(const float *x, size_t x_len, jkb_scratch *ws,
                                     jkb_block_q8_k **out, void *stream) {
    return quantize_in_scratch("quantize_row_q8_k_in_scratch", x, x_len, ws, (void **)out, 256,
                               sizeof(jkb_block_q8_k), stream);
}

int jkb_quantize_row_q8_k_in_scope(const float *x, size_t x_len, jkb_scratch *ws,
                                   jkb_block_q8_k **out, void *stream) {
    return quantize_in_scratch("quantize_row_q8_k_in_scope", x, x_len, ws, (void **)out, 256,
                               sizeof(jkb_block_q8_k), stream);
}

size_t jkb_act_q8_view_scratch_bytes_for_row(size_t k) {
    if (k == 0) return 0;
    const RowPlanes p = row_planes(k);
    return SCRATCH_ALIGN + align_up(p.q) + 2 * align_up(p.g32) + align_up(p.g16) +
           align_up(p.sup);
}

int jkb_act_q8_view_quantize_row_in_scratch(const float *act, size_t k, jkb_scratch *ws,
                                            jkb_act_q8_view *out, void *stream) {
    return view_in_scratch("QuantizedActQ8View::quantize_row_in_scratch", act, k, ws, out,
                           stream);
}

int jkb_act_q8_view_quantize_row_in_scope(const float *act, size_t k, jkb_scratch *ws,
                                          jkb_act_q8_view *out, void *stream) {
    return view_in_scratch("QuantizedActQ8View::quantize_row_in_scope", act, k, ws, out, stream);
}

int jkb_act_q8_as_view(const jkb_act_q8 *act, jkb_act_q8_view *out) {
    if (!act || act->magic != ACT_MAGIC || !out)
        return fail(JKB_E_INVALID, "QuantizedActQ8::as_view", 0, 0, 0, "null or destroyed");
    out->m = act->m;
    out->k = act->k;
    out->k_padded = act->k_pad;
    out->q = act->q;
    out->x_scales = act->x_scales;
    out->x_sums = act->x_sums;
    out->x_sums_16 = act->x_sums_16;
    out->super_scales = act->super_scales;
    return JKB_OK;
}

}  // extern "C"
