// PackedNibbleMatrix (repack.rs:4188-5545) on the GPU: compact 4-bit Q4_0 / Q4_1 / IQ4_NL /
// Q4_K_M weights, their GEMM straight from the 4-bit codes, dequantize_row, the reference's
// tile-buffer constructors and its host tile packer.
//
// The reference keeps 128-byte tiles of 8 rows x 32 nibbles so that one RVV/IME instruction
// builds both 8x16 operand tiles. On the GPU the codes stay in GGUF order, row by row
// (nibble.cuh), which is what the tensor-core GEMM's TMA tiles want and what the tile-buffer
// constructors convert into. Device bytes equal the GGUF payload (1.00x, the reference's
// footprint contract, tests/wave3_prefill_gqa_and_gemm.rs:233-279).
//
// GEMM semantics (execute_nibble_gemm_rows, repack.rs:5181-5397, with accumulate_scaled_tile_
// scalar, :3045-3093): per output (m, n), acc = 0; for each 32-element block b in K order:
//     c = sum xq[m][k] * w[n][k]  (exact i32; w = code - 8 (Q4_0), KVALUES_IQ4NL[code], or code)
//     acc += (f32)c * (xs[m][b] * ws[n][b])  [- x_sum[m][b] * wm[n][b]  for Q4_1 / Q4_K_M]
// ws: Q4_0 / IQ4_NL d (blocks whose d decodes to zero hold +0.0 and zero codes in the
// reference; their contributions are +-0 either way), Q4_1 d with wm = -m (+0.0 when m == 0),
// Q4_K_M d * sc with wm = dmin * m.
// Batches of >= 32 tokens with cols a multiple of 128 run on the tcgen05 kernel (gemm_tc.cu,
// converter warps expand the codes); everything else runs nibble_rows_kernel below, which
// reproduces the reference's roundings exactly.
#include <cstdio>
#include <cstring>
#include <vector>

#include "jkb_internal.h"
#include "nibble.cuh"

namespace jkb {

int gemm_tc_nibble_launch(const jkb_nibble_matrix *w, const jkb_act_q8 *act, float *out,
                          size_t row_begin, size_t row_end, cudaStream_t st, bool *used);

namespace {

// Block geometry of the nibble formats (quant.rs:20-91, lib.rs:129-132).
const Fmt NIB_FMTS[] = {
    {JKB_Q4_0, "Q4_0", 32, 18, 0},
    {JKB_Q4_1, "Q4_1", 32, 20, 0},
    {JKB_IQ4_NL, "IQ4_NL", 32, 18, 0},
    {JKB_Q4_K_M, "Q4_K_M", 256, 144, 0},
};

const Fmt *nib_fmt(int quant) {
    for (const Fmt &f : NIB_FMTS)
        if (f.quant == quant) return &f;
    return nullptr;
}

size_t meta_bytes_of(int quant) {
    return quant == JKB_Q4_K_M ? 16 : quant == JKB_Q4_1 ? 4 : 2;
}

// validate_nibble_quant (repack.rs:4231-4236).
int check_nibble_quant(const char *op, const char *name, int quant, size_t offset,
                       size_t byte_len) {
    if (nib_fmt(quant)) return JKB_OK;
    return fail(JKB_E_CAPABILITY, name, offset, byte_len, byte_len,
                "%s: unsupported tensor quant %s", op, quant_name(quant));
}

int check_matrix(const jkb_nibble_matrix *w) {
    if (!w || w->magic != NIBBLE_MAGIC)
        return fail(JKB_E_INVALID, "PackedNibbleMatrix", 0, 0, 0, "null or destroyed handle");
    return JKB_OK;
}

// One thread per (row, block): the block's quant bytes to qs, its scale bytes to meta.
__global__ void nibble_relayout_kernel(int quant, const uint8_t *__restrict__ raw, size_t rows,
                                       size_t nb, int bb, uint8_t *__restrict__ qs,
                                       uint8_t *__restrict__ meta, int mb) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * nb) return;
    const size_t r = idx / nb, b = idx % nb;
    const uint8_t *blk = raw + idx * (size_t)bb;
    const int qb = quant == JKB_Q4_K_M ? 128 : 16;   // quant bytes per block
    const int off = quant == JKB_Q4_K_M ? 16 : quant == JKB_Q4_1 ? 4 : 2;
    uint8_t *q = qs + r * nb * (size_t)qb + b * (size_t)qb;
    for (int i = 0; i < qb; i++) q[i] = blk[off + i];
    uint8_t *m = meta + idx * (size_t)mb;
    for (int i = 0; i < mb; i++) m[i] = blk[i];
}

// Group g (32 elements) of `row`: int8 values (word i = elements 4i..4i+3), scale and min.
template <int F>
__device__ __forceinline__ void nib_load_group(const uint8_t *__restrict__ qs,
                                               const uint8_t *__restrict__ meta, size_t nb,
                                               size_t cols, size_t row, int g, uint32_t (&v)[8],
                                               float &ws, float &wm) {
    const uint8_t *qrow = qs + row * (cols / 2);
    wm = 0.0f;
    if (F == NIB_Q4_K) {
        const int l = g >> 3, is = g & 7, c = is >> 1, sh = 4 * (is & 1);
        const uint4 *p = reinterpret_cast<const uint4 *>(qrow + 128 * (size_t)l + 32 * c);
        const uint4 a = __ldg(p), b = __ldg(p + 1);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = (w[i] >> sh) & 0x0F0F0F0Fu;
        const uint4 h = __ldg(reinterpret_cast<const uint4 *>(meta) + row * nb + (size_t)l);
        int sc, mn;
        nib_k4_scale_min(h.y, h.z, h.w, is, sc, mn);
        ws = __fmul_rn(nib_f16_finite(h.x & 0xFFFF), (float)sc);
        wm = __fmul_rn(nib_f16_finite(h.x >> 16), (float)mn);
    } else {
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(qrow + 16 * (size_t)g));
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = nib_values4<F>(w[i] & 0x0F0F0F0Fu);
            v[4 + i] = nib_values4<F>((w[i] >> 4) & 0x0F0F0F0Fu);
        }
        if (F == NIB_Q4_1) {
            const uint32_t dm = __ldg(reinterpret_cast<const uint32_t *>(meta) + row * nb + g);
            ws = nib_f16_finite(dm & 0xFFFF);
            wm = nib_q4_1_min(dm >> 16);
        } else {
            ws = nib_d_scale(__ldg(reinterpret_cast<const unsigned short *>(meta) + row * nb + g));
        }
    }
}

// Row kernel (small batches, any cols): a CTA owns R rows x T tokens (R * T <= 256). Per chunk
// of 32 blocks, lane l of a warp computes block g0 + l of its rows for every token --
// p = (f32)c * (xs * ws) [- x_sum * wm] with the reference's roundings -- into shared memory;
// then thread (row, token) adds the chunk's 32 values to its accumulator in block order, so
// each output is the reference's sequential sum, bit for bit.
template <int F>
__global__ void __launch_bounds__(256) nibble_rows_kernel(
    const uint8_t *__restrict__ qs, const uint8_t *__restrict__ meta, size_t nb, size_t cols,
    const int8_t *__restrict__ xq, const float *__restrict__ xs, const float *__restrict__ xsum,
    size_t m, size_t kp, size_t row_begin, size_t row_end, int R, int T,
    float *__restrict__ out) {
    constexpr bool MINS = F == NIB_Q4_1 || F == NIB_Q4_K;
    extern __shared__ float P[];  // [R * T][33]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t r0 = row_begin + (size_t)blockIdx.x * R, t0 = (size_t)blockIdx.y * T;
    const int nr = (int)((row_end - r0) < (size_t)R ? (row_end - r0) : (size_t)R);
    const int nt = (int)((m - t0) < (size_t)T ? (m - t0) : (size_t)T);
    const int kb = (int)(cols / 32);
    const size_t kbx = kp / 32;  // activation blocks per token
    const int my_r = threadIdx.x / T, my_t = threadIdx.x % T;
    const bool owner = my_r < nr && my_t < nt;
    float acc = 0.0f;
    for (int g0 = 0; g0 < kb; g0 += 32) {
        const int g = g0 + lane;
        if (g < kb) {
            for (int rl = warp; rl < nr; rl += 8) {
                uint32_t v[8];
                float ws, wm;
                nib_load_group<F>(qs, meta, nb, cols, r0 + rl, g, v, ws, wm);
                for (int tl = 0; tl < nt; tl++) {
                    const size_t tok = t0 + tl;
                    const int4 *xp = reinterpret_cast<const int4 *>(xq + tok * kp + 32 * (size_t)g);
                    const int4 a0 = __ldg(xp), a1 = __ldg(xp + 1);
                    int c = __dp4a((int)v[0], a0.x, 0);
                    c = __dp4a((int)v[1], a0.y, c);
                    c = __dp4a((int)v[2], a0.z, c);
                    c = __dp4a((int)v[3], a0.w, c);
                    c = __dp4a((int)v[4], a1.x, c);
                    c = __dp4a((int)v[5], a1.y, c);
                    c = __dp4a((int)v[6], a1.z, c);
                    c = __dp4a((int)v[7], a1.w, c);
                    // exact: |c| <= 32 * 127 * 127 < 2^24
                    float p = __fmul_rn((float)c, __fmul_rn(__ldg(xs + tok * kbx + g), ws));
                    if (MINS) p = __fsub_rn(p, __fmul_rn(__ldg(xsum + tok * kbx + g), wm));
                    P[(rl * T + tl) * 33 + lane] = p;
                }
            }
        }
        __syncthreads();
        if (owner) {
            const float *pp = P + (my_r * T + my_t) * 33;
            const int n = kb - g0 < 32 ? kb - g0 : 32;
            for (int i = 0; i < n; i++) acc = __fadd_rn(acc, pp[i]);
        }
        __syncthreads();
    }
    if (owner) out[(t0 + my_t) * (row_end - row_begin) + (r0 - row_begin) + my_r] = acc;
}

// dequantize_row (repack.rs:5001-5036): out[k] = (f32)w * scale - min, min 0.0 without mins.
// Q4_0 / IQ4_NL blocks whose scale decodes to zero read as code 0 (the reference zeroes them).
template <int F>
__global__ void nibble_dequant_row_kernel(const uint8_t *__restrict__ qs,
                                          const uint8_t *__restrict__ meta, size_t nb,
                                          size_t cols, size_t row, float *__restrict__ out) {
    const size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= cols) return;
    const int g = (int)(k / 32), e = (int)(k % 32);
    const uint8_t *qrow = qs + row * (cols / 2);
    uint32_t code;
    float ws, wm = 0.0f;
    if (F == NIB_Q4_K) {
        const int l = g >> 3, is = g & 7, c = is >> 1;
        const uint8_t byte = qrow[128 * (size_t)l + 32 * c + e];
        code = (is & 1) ? (byte >> 4) : (byte & 0x0F);
        const uint4 h = reinterpret_cast<const uint4 *>(meta)[row * nb + (size_t)l];
        int sc, mn;
        nib_k4_scale_min(h.y, h.z, h.w, is, sc, mn);
        ws = __fmul_rn(nib_f16_finite(h.x & 0xFFFF), (float)sc);
        wm = __fmul_rn(nib_f16_finite(h.x >> 16), (float)mn);
    } else {
        const uint8_t byte = qrow[16 * (size_t)g + (e & 15)];
        code = e < 16 ? (byte & 0x0F) : (byte >> 4);
        if (F == NIB_Q4_1) {
            const uint32_t dm = reinterpret_cast<const uint32_t *>(meta)[row * nb + g];
            ws = nib_f16_finite(dm & 0xFFFF);
            wm = nib_q4_1_min(dm >> 16);
        } else {
            ws = nib_d_scale(reinterpret_cast<const unsigned short *>(meta)[row * nb + g]);
            if (ws == 0.0f) code = 0;
        }
    }
    const int8_t w = (int8_t)(nib_values4<F>(code) & 0xFF);
    out[k] = __fsub_rn(__fmul_rn((float)w, ws), wm);
}

template <int F>
int launch_rows(const jkb_nibble_matrix *w, const jkb_act_q8 *act, float *out, size_t row_begin,
                size_t row_end, cudaStream_t st) {
    const size_t sub_n = row_end - row_begin, m = act->m;
    const int T = m < 32 ? (int)m : 32;
    const int rmax = 256 / T;
    const size_t sms = (size_t)num_sms();
    size_t want = (sub_n + 2 * sms - 1) / (2 * sms);
    int R = (int)(want < (size_t)rmax ? want : (size_t)rmax);
    if (R < 8) R = rmax < 8 ? rmax : 8;
    const size_t gx = (sub_n + R - 1) / R, gy = (m + T - 1) / T;
    if (gx > 0x7FFFFFFFu || gy > 65535)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix::gemm", 0, m, sub_n,
                    "batch of %zu tokens x %zu rows exceeds the launch grid", m, sub_n);
    const size_t smem = (size_t)R * T * 33 * sizeof(float);
    nibble_rows_kernel<F><<<dim3((unsigned)gx, (unsigned)gy), 256, smem, st>>>(
        w->qs, w->meta, w->nb, w->cols, act->q, act->x_scales, act->x_sums, m, act->k_pad,
        row_begin, row_end, R, T, out);
    return check_launch("nibble_rows_kernel");
}

// execute_nibble_gemm_rows validation (repack.rs:5188-5245), then the tensor-core kernel or the
// row kernel.
int nibble_gemm_rows(const char *fn, float *out, size_t out_len, const jkb_nibble_matrix *w,
                     const jkb_act_q8 *act, size_t row_begin, size_t row_end, cudaStream_t st) {
    int rc = check_matrix(w);
    if (rc) return rc;
    if (!act || act->magic != ACT_MAGIC)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed activation handle");
    const size_t packed = w->rows * w->nb * (w->meta_bytes + (w->quant == JKB_Q4_K_M ? 128 : 16));
    if (act->k != w->cols)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix::gemm", 0, out_len * 4, packed,
                    "activation K (%zu) != weight cols (%zu)", act->k, w->cols);
    if (row_begin > row_end || row_end > w->rows)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix::gemm", row_begin,
                    row_end > row_begin ? row_end - row_begin : 0, w->rows,
                    "invalid row_range %zu..%zu for weight rows %zu", row_begin, row_end,
                    w->rows);
    const size_t sub_n = row_end - row_begin;
    if (out_len != act->m * sub_n)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix::gemm", 0, out_len * 4,
                    act->m * sub_n * 4, "output length %zu != m (%zu) * sub_rows (%zu)", out_len,
                    act->m, sub_n);
    if (sub_n == 0 || act->m == 0) return JKB_OK;
    if (!out) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null output");
    rc = check_align(out, 4, fn, "output");
    if (!rc) rc = push_reject(out, out + out_len, fn);
    if (rc) return rc;
    bool used = false;
    rc = gemm_tc_nibble_launch(w, act, out, row_begin, row_end, st, &used);
    if (rc || used) return rc;
    switch (w->quant) {
        case JKB_Q4_0: return launch_rows<NIB_Q4_0>(w, act, out, row_begin, row_end, st);
        case JKB_Q4_1: return launch_rows<NIB_Q4_1>(w, act, out, row_begin, row_end, st);
        case JKB_IQ4_NL: return launch_rows<NIB_IQ4_NL>(w, act, out, row_begin, row_end, st);
        default: return launch_rows<NIB_Q4_K>(w, act, out, row_begin, row_end, st);
    }
}

// Allocates the handle and its planes (qs, then meta, each 256-byte aligned).
int alloc_matrix(int quant, size_t rows, size_t cols, const char *name, jkb_nibble_matrix **out) {
    const Fmt *f = nib_fmt(quant);
    jkb_nibble_matrix *w = new jkb_nibble_matrix();
    memset(w, 0, sizeof(*w));
    w->magic = NIBBLE_MAGIC;
    w->quant = quant;
    w->rows = rows;
    w->cols = cols;
    w->nb = cols / (size_t)f->block_elems;
    w->meta_bytes = meta_bytes_of(quant);
    snprintf(w->name, sizeof(w->name), "%s", name ? name : "");
    Arena a;
    const size_t qb = rows * (cols / 2), mb = rows * w->nb * w->meta_bytes;
    a.cap = Arena::round(qb) + Arena::round(mb);
    cudaError_t e = cudaMalloc(&a.base, a.cap);
    if (e != cudaSuccess) {
        delete w;
        return fail_cuda(e, "PackedNibbleMatrix (device planes)");
    }
    w->base = a.base;
    w->device_bytes = a.cap;
    w->qs = a.take(qb);
    w->meta = a.take(mb);
    *out = w;
    return JKB_OK;
}

void free_matrix(jkb_nibble_matrix *w) {
    w->magic = 0;
    cudaFree(w->base);
    delete w;
}

// PackedNibbleMatrix::from_tensor (repack.rs:4788-4905): validate, then relayout on the device.
int from_tensor(const jkb_tensor_view *v, size_t rows, size_t cols, cudaStream_t st,
                jkb_nibble_matrix **out) {
    if (!v || !out) return fail(JKB_E_INVALID, "PackedNibbleMatrix", 0, 0, 0, "null argument");
    *out = nullptr;
    const char *nm = v->name ? v->name : "";
    int rc = check_nibble_quant("PackedNibbleMatrix::from_tensor", nm, v->quant, v->offset,
                                v->byte_len);
    if (rc) return rc;
    if (!v->data) return fail(JKB_E_INVALID, nm, v->offset, 0, 0, "null tensor data");
    const Fmt *f = nib_fmt(v->quant);
    rc = validate_matrix_view(v, f, rows, cols);
    if (rc) return rc;
    jkb_nibble_matrix *w = nullptr;
    rc = alloc_matrix(v->quant, rows, cols, nm, &w);
    if (rc) return rc;
    const size_t payload = rows * w->nb * (size_t)f->block_bytes;
    uint8_t *raw = nullptr;
    bool owned = false;
    rc = stage_raw(v, payload, st, &raw, &owned);
    if (rc) {
        free_matrix(w);
        return rc;
    }
    const size_t n = rows * w->nb;
    nibble_relayout_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        v->quant, raw, rows, w->nb, f->block_bytes, w->qs, w->meta, (int)w->meta_bytes);
    rc = check_launch("nibble_relayout_kernel");
    if (owned) {
        cudaStreamSynchronize(st);
        cudaFree(raw);
    }
    if (rc) {
        free_matrix(w);
        return rc;
    }
    *out = w;
    return JKB_OK;
}

// Nibble k (0..31) of row j (0..7) in one 128-byte reference tile (layout of
// pack_pair_split_nibbles_into_tile, repack.rs:4281-4305): bytes 0..64 hold columns 0..15,
// bytes 64..128 columns 16..31; pair j / 2 at 16 * (j / 2); even rows low nibble, odd rows high.
inline uint8_t tile_nibble(const uint8_t *tile, int j, int k) {
    const uint8_t b = tile[(k < 16 ? 0 : 64) + 16 * (j >> 1) + (k & 15)];
    return (j & 1) ? (uint8_t)(b >> 4) : (uint8_t)(b & 0x0F);
}

// Planes from the reference's tiles (host), then one upload.
int from_tiles(int quant, size_t rows, size_t cols, const uint8_t *tiles, const uint16_t *scales,
               const uint8_t *headers, cudaStream_t st, jkb_nibble_matrix **out) {
    const size_t kb = cols / 32, nsb = cols / 256, nt_count = (rows + 7) / 8;
    (void)nt_count;
    jkb_nibble_matrix *w = nullptr;
    int rc = alloc_matrix(quant, rows, cols, "PackedNibbleMatrix", &w);
    if (rc) return rc;
    std::vector<uint8_t> qs(rows * (cols / 2)), meta(rows * w->nb * w->meta_bytes);
    for (size_t r = 0; r < rows; r++) {
        const size_t nt = r / 8;
        const int j = (int)(r % 8);
        uint8_t *qrow = qs.data() + r * (cols / 2);
        if (quant == JKB_Q4_K_M) {
            for (size_t l = 0; l < nsb; l++) {
                memcpy(meta.data() + (r * nsb + l) * 16, headers + ((nt * nsb + l) * 8 + j) * 16, 16);
                for (int c = 0; c < 4; c++) {
                    const uint8_t *tlo = tiles + (nt * kb + l * 8 + 2 * c) * 128, *thi = tlo + 128;
                    for (int e = 0; e < 32; e++)
                        qrow[128 * l + 32 * c + e] =
                            (uint8_t)(tile_nibble(tlo, j, e) | (tile_nibble(thi, j, e) << 4));
                }
            }
        } else {
            for (size_t b = 0; b < kb; b++) {
                const uint8_t *t = tiles + (nt * kb + b) * 128;
                for (int e = 0; e < 16; e++)
                    qrow[16 * b + e] = (uint8_t)(tile_nibble(t, j, e) | (tile_nibble(t, j, e + 16) << 4));
                const uint16_t d = scales[(nt * kb + b) * 8 + j];
                memcpy(meta.data() + (r * kb + b) * 2, &d, 2);
            }
        }
    }
    cudaError_t e = cudaMemcpyAsync(w->qs, qs.data(), qs.size(), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(w->meta, meta.data(), meta.size(), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        free_matrix(w);
        return fail_cuda(e, "PackedNibbleMatrix (tile upload)");
    }
    *out = w;
    return JKB_OK;
}

inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// f16_to_f32_finite(bits) == 0.0 (lib.rs:714-717): +-0, and NaN / Inf (which decode to 0).
inline bool f16_finite_is_zero(uint16_t b) {
    return (b & 0x7FFF) == 0 || ((b >> 10) & 0x1F) == 0x1F;
}

}  // namespace

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_packed_nibble_matrix_from_tensor(const jkb_tensor_view *view, size_t rows, size_t cols,
                                         void *stream, jkb_nibble_matrix **out) {
    return from_tensor(view, rows, cols, as_stream(stream), out);
}

int jkb_packed_nibble_matrix_repack(const jkb_tensor_view *view, void *stream,
                                    jkb_nibble_matrix **out) {
    if (!view || !out)
        return fail(JKB_E_INVALID, "PackedNibbleMatrix::repack", 0, 0, 0, "null argument");
    const Fmt *f = nib_fmt(view->quant);
    size_t r = 0, c = 0;
    if (f) {
        // PackedNibbleMatrix::repack (repack.rs:4654-4679): 2-D only, orientation inferred,
        // then from_tensor (which reports an unsupported quant)
        int rc = infer_rows_cols(view, f, &r, &c, "PackedNibbleMatrix::repack");
        if (rc) return rc;
    } else {
        if (view->ndim != 2)
            return fail(JKB_E_BOUNDS, view->name ? view->name : "", view->offset, view->byte_len,
                        view->byte_len, "PackedNibbleMatrix::repack requires a 2D tensor, got %uD",
                        view->ndim);
        r = view->shape[1];
        c = view->shape[0];
    }
    return from_tensor(view, r, c, as_stream(stream), out);
}

int jkb_packed_nibble_matrix_from_scale_f16_buffers(int32_t quant, size_t rows, size_t cols,
                                                    const uint8_t *nibble_tiles, size_t n_tiles,
                                                    const uint16_t *scales_f16, size_t n_scales,
                                                    void *stream, jkb_nibble_matrix **out) {
    if (!out) return fail(JKB_E_INVALID, "PackedNibbleMatrix", 0, 0, 0, "null argument");
    *out = nullptr;
    // repack.rs:4686-4741
    if (quant != JKB_Q4_0 && quant != JKB_IQ4_NL)
        return fail(JKB_E_CAPABILITY, "buffers", 0, 0, 0,
                    "PackedNibbleMatrix::from_scale_f16_buffers: unsupported tensor quant %s",
                    quant_name(quant));
    const size_t nt = (rows + 7) / 8;
    if (rows == 0 || cols == 0 || cols % 32 != 0)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix", 0, rows, cols,
                    "invalid rows/cols for block format");
    const size_t kb = cols / 32;
    if (n_tiles != nt * kb || n_scales != nt * kb * 8)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix", 0, n_tiles, nt * kb,
                    "nibble buffer lengths do not match geometry");
    if (!nibble_tiles || !scales_f16)
        return fail(JKB_E_INVALID, "PackedNibbleMatrix", 0, 0, 0, "null buffer");
    return from_tiles(quant, rows, cols, nibble_tiles, scales_f16, nullptr, as_stream(stream), out);
}

int jkb_packed_nibble_matrix_from_q4_k_buffers(size_t rows, size_t cols,
                                               const uint8_t *nibble_tiles, size_t n_tiles,
                                               const uint8_t *headers, size_t n_headers,
                                               void *stream, jkb_nibble_matrix **out) {
    if (!out) return fail(JKB_E_INVALID, "PackedNibbleMatrix", 0, 0, 0, "null argument");
    *out = nullptr;
    // repack.rs:4743-4786
    const size_t nt = (rows + 7) / 8;
    if (rows == 0 || cols == 0 || cols % 256 != 0)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix", 0, rows, cols,
                    "invalid rows/cols for Q4_K_M");
    const size_t kb = cols / 32, nsb = cols / 256;
    if (n_tiles != nt * kb || n_headers != nt * nsb * 8)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix", 0, n_tiles, nt * kb,
                    "Q4_K_M nibble buffer lengths do not match geometry");
    if (!nibble_tiles || !headers)
        return fail(JKB_E_INVALID, "PackedNibbleMatrix", 0, 0, 0, "null buffer");
    return from_tiles(JKB_Q4_K_M, rows, cols, nibble_tiles, nullptr, headers, as_stream(stream),
                      out);
}

// repack_nibble_into_tile_range (repack.rs:4414-4645), host memory in and out.
int jkb_repack_nibble_into_tile_range(const jkb_tensor_view *view, size_t rows, size_t cols,
                                      size_t tile_begin, size_t tile_end, uint8_t *out_tiles,
                                      size_t n_out_tiles, uint16_t *out_scales_f16,
                                      size_t n_scales, uint16_t *out_mins_f16, size_t n_mins,
                                      uint8_t *out_headers, size_t n_headers) {
    if (!view) return fail(JKB_E_INVALID, "repack_nibble_into_tile_range", 0, 0, 0, "null view");
    const char *nm = view->name ? view->name : "";
    int rc = check_nibble_quant("repack_nibble_into_tile_range", nm, view->quant, view->offset,
                                view->byte_len);
    if (rc) return rc;
    const Fmt *f = nib_fmt(view->quant);
    rc = validate_matrix_view(view, f, rows, cols);
    if (rc) return rc;
    if (!view->data || view->data_on_device)
        return fail(JKB_E_INVALID, nm, view->offset, view->byte_len, view->byte_len,
                    "repack_nibble_into_tile_range reads host bytes");
    const size_t n_tiles = (rows + 7) / 8, kb = cols / 32;
    if (tile_begin > tile_end || tile_end > n_tiles)
        return fail(JKB_E_BOUNDS, nm, tile_begin, tile_end > tile_begin ? tile_end - tile_begin : 0,
                    n_tiles, "tile_range %zu..%zu exceeds n_tiles (%zu)", tile_begin, tile_end,
                    n_tiles);
    const size_t sub = tile_end - tile_begin, expected_tiles = sub * kb;
    if (n_out_tiles != expected_tiles || (expected_tiles && !out_tiles))
        return fail(JKB_E_BOUNDS, nm, tile_begin, n_out_tiles, expected_tiles,
                    "nibble out_tiles length %zu != %zu", n_out_tiles, expected_tiles);
    const int quant = view->quant;
    const size_t meta_per = sub * kb * 8;
    if (quant == JKB_Q4_0 || quant == JKB_IQ4_NL || quant == JKB_Q4_1) {
        if (n_scales != meta_per || (meta_per && !out_scales_f16))
            return fail(JKB_E_BOUNDS, nm, 0, n_scales, meta_per,
                        "out_scales_f16 slice length mismatch");
        if (quant == JKB_Q4_1) {
            if (!out_mins_f16 && meta_per)
                return fail(JKB_E_BOUNDS, nm, 0, 0, meta_per, "Q4_1 requires out_mins_f16 slice");
            if (n_mins != meta_per)
                return fail(JKB_E_BOUNDS, nm, 0, n_mins, meta_per,
                            "out_mins_f16 slice length mismatch");
        }
    } else {
        const size_t expected = sub * (cols / 256) * 8;
        if (!out_headers && expected)
            return fail(JKB_E_BOUNDS, nm, 0, 0, expected, "Q4_K_M requires out_q4k_headers slice");
        if (n_headers != expected)
            return fail(JKB_E_BOUNDS, nm, 0, n_headers, expected,
                        "out_q4k_headers slice length mismatch");
    }
    if (expected_tiles) memset(out_tiles, 0, expected_tiles * 128);
    if (quant == JKB_Q4_K_M) {
        if (n_headers) memset(out_headers, 0, n_headers * 16);
    } else {
        if (meta_per) memset(out_scales_f16, 0, meta_per * 2);
        if (quant == JKB_Q4_1 && meta_per) memset(out_mins_f16, 0, meta_per * 2);
    }
    const uint8_t *raw = (const uint8_t *)view->data;
    const size_t rb = cols / (size_t)f->block_elems * (size_t)f->block_bytes;
    const size_t nsb = cols / 256;
    static const uint8_t zero[32] = {0};
    // pack_pair_split_nibbles_into_tile / pack_q4k_pair_chunk32_into_tiles (:4281-4392)
    auto pack = [](const uint8_t *e, const uint8_t *o, uint8_t *lo, uint8_t *hi, int pair) {
        for (int k = 0; k < 16; k++) {
            lo[pair * 16 + k] = (uint8_t)((e[k] & 0x0F) | ((o[k] & 0x0F) << 4));
            hi[pair * 16 + k] = (uint8_t)((e[k] >> 4) | (o[k] & 0xF0));
        }
    };
    for (size_t lt = 0; lt < sub; lt++) {
        const size_t nt = tile_begin + lt;
        uint8_t *tl = out_tiles + lt * kb * 128;
        for (int pair = 0; pair < 4; pair++) {
            const size_t re = nt * 8 + 2 * (size_t)pair;
            if (re >= rows) break;
            const bool has_odd = re + 1 < rows;
            const uint8_t *er = raw + re * rb, *orw = has_odd ? raw + (re + 1) * rb : nullptr;
            if (quant == JKB_Q4_0 || quant == JKB_IQ4_NL) {
                for (size_t b = 0; b < kb; b++) {
                    const uint8_t *be = er + b * 18;
                    const uint16_t eb = rd16(be);
                    const bool ez = f16_finite_is_zero(eb);
                    out_scales_f16[(lt * kb + b) * 8 + 2 * pair] = ez ? 0 : eb;
                    bool oz = true;
                    const uint8_t *no = zero;
                    if (has_odd) {
                        const uint8_t *bo = orw + b * 18;
                        const uint16_t ob = rd16(bo);
                        oz = f16_finite_is_zero(ob);
                        out_scales_f16[(lt * kb + b) * 8 + 2 * pair + 1] = oz ? 0 : ob;
                        if (!oz) no = bo + 2;
                    }
                    if (!ez || !oz)
                        pack(ez ? zero : be + 2, no, tl + b * 128, tl + b * 128 + 64, pair);
                }
            } else if (quant == JKB_Q4_1) {
                for (size_t b = 0; b < kb; b++) {
                    const uint8_t *be = er + b * 20;
                    const size_t ie = (lt * kb + b) * 8 + 2 * pair;
                    out_scales_f16[ie] = rd16(be);
                    out_mins_f16[ie] = rd16(be + 2);
                    const uint8_t *no = zero;
                    if (has_odd) {
                        const uint8_t *bo = orw + b * 20;
                        out_scales_f16[ie + 1] = rd16(bo);
                        out_mins_f16[ie + 1] = rd16(bo + 2);
                        no = bo + 4;
                    }
                    pack(be + 4, no, tl + b * 128, tl + b * 128 + 64, pair);
                }
            } else {
                for (size_t sb = 0; sb < nsb; sb++) {
                    const uint8_t *be = er + sb * 144;
                    memcpy(out_headers + ((lt * nsb + sb) * 8 + 2 * pair) * 16, be, 16);
                    const uint8_t *bo = nullptr;
                    if (has_odd) {
                        bo = orw + sb * 144;
                        memcpy(out_headers + ((lt * nsb + sb) * 8 + 2 * pair + 1) * 16, bo, 16);
                    }
                    for (int c = 0; c < 4; c++) {
                        const uint8_t *qe = be + 16 + 32 * c, *qo = bo ? bo + 16 + 32 * c : zero;
                        uint8_t *lo = tl + (sb * 8 + 2 * c) * 128, *hi = lo + 128;
                        // columns 0..15 of both blocks from qs[0..16], 16..31 from qs[16..32]
                        pack(qe, qo, lo, hi, pair);
                        pack(qe + 16, qo + 16, lo + 64, hi + 64, pair);
                    }
                }
            }
        }
    }
    return JKB_OK;
}

int jkb_packed_nibble_matrix_destroy(jkb_nibble_matrix *w) {
    int rc = check_matrix(w);
    if (rc) return rc;
    free_matrix(w);
    return JKB_OK;
}

int jkb_packed_nibble_matrix_info(const jkb_nibble_matrix *w, size_t *rows, size_t *cols,
                                  int32_t *quant, size_t *n_tiles, size_t *k_blocks32,
                                  size_t *packed_bytes, size_t *raw_tensor_bytes) {
    int rc = check_matrix(w);
    if (rc) return rc;
    const Fmt *f = nib_fmt(w->quant);
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (quant) *quant = w->quant;
    if (n_tiles) *n_tiles = (w->rows + 7) / 8;
    if (k_blocks32) *k_blocks32 = w->cols / 32;
    if (packed_bytes)
        *packed_bytes = w->rows * (w->cols / 2) + w->rows * w->nb * w->meta_bytes;
    if (raw_tensor_bytes) *raw_tensor_bytes = w->rows * w->nb * (size_t)f->block_bytes;
    return JKB_OK;
}

int jkb_packed_nibble_matrix_buffers(const jkb_nibble_matrix *w, uint8_t **qs, uint8_t **meta) {
    int rc = check_matrix(w);
    if (rc) return rc;
    if (qs) *qs = w->qs;
    if (meta) *meta = w->meta;
    return JKB_OK;
}

int jkb_packed_nibble_matrix_gemm(float *out, size_t out_len, const jkb_nibble_matrix *w,
                                  const jkb_act_q8 *act, void *stream) {
    int rc = check_matrix(w);
    if (rc) return rc;
    return nibble_gemm_rows("PackedNibbleMatrix::gemm", out, out_len, w, act, 0, w->rows,
                            as_stream(stream));
}

int jkb_packed_nibble_matrix_gemm_rows(float *out, size_t out_len, const jkb_nibble_matrix *w,
                                       const jkb_act_q8 *act, size_t row_begin, size_t row_end,
                                       void *stream) {
    return nibble_gemm_rows("PackedNibbleMatrix::gemm_rows", out, out_len, w, act, row_begin,
                            row_end, as_stream(stream));
}

int jkb_packed_nibble_matrix_gemv(float *out, size_t out_len, const jkb_nibble_matrix *w,
                                  const jkb_act_q8 *act, void *stream) {
    int rc = check_matrix(w);
    if (rc) return rc;
    if (!act || act->magic != ACT_MAGIC)
        return fail(JKB_E_INVALID, "PackedNibbleMatrix::gemv", 0, 0, 0,
                    "null or destroyed activation handle");
    // repack.rs:4968-4980
    if (act->m != 1)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix::gemv", 0, act->m, 1,
                    "gemv requires act.m() == 1, got %zu", act->m);
    return nibble_gemm_rows("PackedNibbleMatrix::gemv", out, out_len, w, act, 0, w->rows,
                            as_stream(stream));
}

int jkb_packed_nibble_matrix_dequantize_row(const jkb_nibble_matrix *w, size_t row, float *out,
                                            size_t out_len, void *stream) {
    int rc = check_matrix(w);
    if (rc) return rc;
    // repack.rs:5001-5015
    if (row >= w->rows || out_len != w->cols)
        return fail(JKB_E_BOUNDS, "PackedNibbleMatrix::dequantize_row", row, out_len, w->cols,
                    "row (%zu) >= rows (%zu) or out.len() (%zu) != cols (%zu)", row, w->rows,
                    out_len, w->cols);
    if (!out) return fail(JKB_E_INVALID, "PackedNibbleMatrix::dequantize_row", 0, 0, 0, "null");
    rc = check_align(out, 4, "PackedNibbleMatrix::dequantize_row", "output");
    if (rc) return rc;
    cudaStream_t st = as_stream(stream);
    const unsigned grid = (unsigned)((w->cols + 255) / 256);
    switch (w->quant) {
        case JKB_Q4_0:
            nibble_dequant_row_kernel<NIB_Q4_0><<<grid, 256, 0, st>>>(w->qs, w->meta, w->nb, w->cols, row, out);
            break;
        case JKB_Q4_1:
            nibble_dequant_row_kernel<NIB_Q4_1><<<grid, 256, 0, st>>>(w->qs, w->meta, w->nb, w->cols, row, out);
            break;
        case JKB_IQ4_NL:
            nibble_dequant_row_kernel<NIB_IQ4_NL><<<grid, 256, 0, st>>>(w->qs, w->meta, w->nb, w->cols, row, out);
            break;
        default:
            nibble_dequant_row_kernel<NIB_Q4_K><<<grid, 256, 0, st>>>(w->qs, w->meta, w->nb, w->cols, row, out);
            break;
    }
    return check_launch("nibble_dequant_row_kernel");
}

// gemm_q4_0_ime / gemm_q4_k_ime (repack.rs:5140-5175): format check, then the GEMM.
int jkb_gemm_q4_0_ime(float *out, size_t out_len, const jkb_nibble_matrix *w,
                      const jkb_act_q8 *act, void *stream) {
    int rc = check_matrix(w);
    if (rc) return rc;
    if (w->quant != JKB_Q4_0)
        return fail(JKB_E_CAPABILITY, "PackedNibbleMatrix", 0, 0, 0,
                    "gemm_q4_0_ime: unsupported tensor quant %s", quant_name(w->quant));
    return nibble_gemm_rows("gemm_q4_0_ime", out, out_len, w, act, 0, w->rows, as_stream(stream));
}

int jkb_gemm_q4_k_ime(float *out, size_t out_len, const jkb_nibble_matrix *w,
                      const jkb_act_q8 *act, void *stream) {
    int rc = check_matrix(w);
    if (rc) return rc;
    if (w->quant != JKB_Q4_K_M)
        return fail(JKB_E_CAPABILITY, "PackedNibbleMatrix", 0, 0, 0,
                    "gemm_q4_k_ime: unsupported tensor quant %s", quant_name(w->quant));
    return nibble_gemm_rows("gemm_q4_k_ime", out, out_len, w, act, 0, w->rows, as_stream(stream));
}

}  // extern "C"
