// Load-time weight handles: validation (repack.rs:1208-1284), upload and relayout into the
// GPU layouts used by the GEMV / BitLinear kernels (jkb_weight) and by the GEMM
// (jkb_repacked_weight, the i8-expanded RepackedWeight of repack.rs:1092-1133).
//
// jkb_weight planes (every row contiguous, rows back to back, block order kept; the quant
// plane's 16-byte chunks are lane-interleaved in groups of 32 blocks, see gpu_layout.cuh):
//   Q4_0   qs: 16 B/block, the GGUF nibble bytes        d: f16 per block
//   Q8_0   qs: 32 B/block, the GGUF i8 quants           d: f16 per block
//   Q4_K_M qs: 128 B/block, GGUF qs bytes               sc: 16 B/block = d, dmin, scales[12]
//   Q5_0   qs: 16 B/block, the GGUF nibble bytes        sc: 4 B/block = qh   d: f16 per block
//   Q5_K   qs: 160 B/block, GGUF qs[128] then qh[32]    sc: 16 B/block = d, dmin, scales[12]
//   Q6_K   qs: 192 B/block, GGUF ql[128] then qh[64]    sc: 16 B/block i8 scales, d: f16
//   TQ2_0  qs: 64 B/block, 2-bit codes re-ordered so that chunk p, word W, bit pair j, byte b
//          holds element 64p+16W+4j+b                   d: f16 per block
//   TQ1_0  decoded at load into the TQ2_0 GPU layout (same codes 0..2)
//   I2_S   qs: 32 B/block, GGUF bytes unchanged; the trailer scale is kept on the host
// Byte counts equal the GGUF payload (except TQ1_0, whose base-3 bytes grow from 54 to 66).
#include <cstdio>
#include <cstring>
#include <vector>

#include "gpu_layout.cuh"
#include "jkb_internal.h"
#include "repack_block.cuh"

namespace jkb {

__device__ __forceinline__ uint16_t rd16(const uint8_t *p) {
    return (uint16_t)(p[0] | (p[1] << 8));
}

// One thread per (row, block): scale planes are written [row][block], quant bytes go to the
// lane-interleaved chunk positions of gpu_layout.cuh. `payload` holds the block's quant bytes
// in GPU chunk order (chunk j = payload[16j .. 16j+16]).
__global__ void relayout_kernel(int quant, int gpu_format, const uint8_t *__restrict__ raw,
                                size_t rows, size_t nb, size_t raw_row, int bb,
                                uint8_t *__restrict__ qs, size_t qs_row, uint8_t *__restrict__ sc,
                                size_t sc_row, uint16_t *__restrict__ d) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * nb) return;
    size_t r = idx / nb, b = idx % nb;
    const uint8_t *blk = raw + r * raw_row + b * (size_t)bb;
    uint8_t payload[192];
    switch (quant) {
    case JKB_Q4_0:  // 16 nibble bytes, GGUF order
        d[idx] = rd16(blk);
        for (int i = 0; i < 16; i++) payload[i] = blk[2 + i];
        break;
    case JKB_Q8_0:  // 32 i8 quants
        d[idx] = rd16(blk);
        for (int i = 0; i < 32; i++) payload[i] = blk[2 + i];
        break;
    case JKB_Q4_K_M: {  // d, dmin, scales[12] to the scale plane; qs[128] in GGUF order
        uint8_t *s = sc + r * sc_row + 16 * b;
        for (int i = 0; i < 16; i++) s[i] = blk[i];
        for (int i = 0; i < 128; i++) payload[i] = blk[16 + i];
        break;
    }
    case JKB_Q5_0: {  // 16 nibble bytes, GGUF order; qh to the scale plane, d to its plane
        uint8_t *s = sc + r * sc_row + 4 * b;
        for (int i = 0; i < 4; i++) s[i] = blk[2 + i];
        d[idx] = rd16(blk);
        for (int i = 0; i < 16; i++) payload[i] = blk[6 + i];
        break;
    }
    case JKB_Q5_K: {  // d, dmin, scales[12] to the scale plane; qs[128] then qh[32]
        uint8_t *s = sc + r * sc_row + 16 * b;
        for (int i = 0; i < 16; i++) s[i] = blk[i];
        for (int i = 0; i < 128; i++) payload[i] = blk[48 + i];
        for (int i = 0; i < 32; i++) payload[128 + i] = blk[16 + i];
        break;
    }
    case JKB_Q6_K: {  // ql[128] qh[64] in GGUF order; i8 scales and d to their planes
        uint8_t *s = sc + r * sc_row + 16 * b;
        for (int i = 0; i < 16; i++) s[i] = blk[192 + i];
        d[idx] = rd16(blk + 208);
        for (int i = 0; i < 192; i++) payload[i] = blk[i];
        break;
    }
    case JKB_TQ2_0:
    case JKB_TQ1_0: {
        // 2-bit codes (value + 1) re-ordered so that chunk p, word W, bit pair j, byte q holds
        // element 64p + 16W + 4j + q: (word >> 2j) & 0x03030303 then lines up with four
        // consecutive activations.
        d[idx] = rd16(blk);
        uint8_t codes[256];
        if (quant == JKB_TQ2_0) {
            for (int e = 0; e < 256; e++) codes[e] = (blk[2 + e / 4] >> (2 * (e % 4))) & 3;
        } else {
            for (int i = 0; i < 51; i++) {
                unsigned v = blk[2 + i];
                for (int j = 0; j < 5; j++) {
                    codes[5 * i + j] = (uint8_t)(v % 3);
                    v /= 3;
                }
            }
            codes[255] = (uint8_t)(blk[53] % 3);
        }
        for (int i = 0; i < 64; i++) payload[i] = 0;
        for (int e = 0; e < 256; e++) {
            int p = e >> 6, W = (e & 63) >> 4, j = (e & 15) >> 2, bq = e & 3;
            payload[16 * p + 4 * W + bq] |= (uint8_t)(codes[e] << (2 * j));
        }
        break;
    }
    case JKB_I2_S:  // 32 bytes, GGUF order (byte g carries elements g, 32+g, 64+g, 96+g)
        for (int i = 0; i < 32; i++) payload[i] = blk[i];
        break;
    default: return;
    }
    const int qch = qs_chunks(gpu_format);
    uint8_t *row = qs + r * qs_row;
    for (int j = 0; j < qch; j++) {
        uint8_t *o = row + qs_chunk_offset((int)nb, qch, (int)b, j);
        for (int i = 0; i < 16; i++) o[i] = payload[16 * j + i];
    }
}

// repack_block_scaled_range_into_i8 (repack.rs:1724-2103), one thread per (row, block): i8
// values row-major [rows][k_pad], f32 scales (and mins) [rows][groups]. The per-block decoder
// (repack_block.cuh) is shared with the host tile packer of jkb_repack_into_tile_range.
__global__ void repack_i8_kernel(int quant, const uint8_t *__restrict__ raw, size_t rows,
                                 size_t nb, size_t raw_row, int bb, float i2s, int8_t *q,
                                 size_t k_pad, float *scales, float *mins, size_t groups) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * nb) return;
    size_t r = idx / nb, b = idx % nb;
    const int be = repack_block_elems(quant), gpb = be / repack_group_elems(quant);
    repack_block_i8(quant, raw + r * raw_row + b * (size_t)bb, q + r * k_pad + b * (size_t)be,
                    scales + r * groups + b * (size_t)gpb,
                    mins ? mins + r * groups + b * (size_t)gpb : nullptr, i2s);
}

// validate_matrix_shape + validate_matrix_view (repack.rs:1151-1284).
int validate_matrix_view(const jkb_tensor_view *v, const Fmt *f, size_t rows,
                                size_t cols) {
    const char *nm = v->name ? v->name : "";
    if (rows == 0 || cols == 0)
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "repack dimensions must be non-zero, got [%zu, %zu]", rows, cols);
    if (cols % (size_t)f->block_elems != 0)
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "columns (%zu) must be a multiple of %s block size (%d)", cols, f->name,
                    f->block_elems);
    if (v->ndim == 1) {
        if (rows * cols != v->shape[0])
            return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                        "1D tensor length %zu does not match rows (%zu) * cols (%zu)",
                        v->shape[0], rows, cols);
    } else if (v->ndim == 2) {
        size_t d0 = v->shape[0], d1 = v->shape[1];
        if (!((d0 == rows && d1 == cols) || (d0 == cols && d1 == rows)))
            return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                        "tensor shape [%zu, %zu] does not match requested rows=%zu, cols=%zu",
                        d0, d1, rows, cols);
    } else {
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "expected 1D or 2D weight tensor, got %uD", v->ndim);
    }
    size_t need = storage_bytes(f, rows * cols);
    if (v->byte_len < need)
        return fail(JKB_E_BOUNDS, nm, v->offset, v->byte_len, v->byte_len,
                    "backing bytes %zu < required %zu", v->byte_len, need);
    return JKB_OK;
}

// RepackedWeight::repack orientation rule (repack.rs:2255-2282; PackedNibbleMatrix::repack
// :4654-4679 is the same rule). `who` names the caller in the error.
int infer_rows_cols(const jkb_tensor_view *v, const Fmt *f, size_t *rows, size_t *cols,
                    const char *who) {
    if (v->ndim != 2)
        return fail(JKB_E_BOUNDS, v->name ? v->name : "", v->offset, v->byte_len, v->byte_len,
                    "%s requires a 2D tensor, got %uD", who, v->ndim);
    size_t d0 = v->shape[0], d1 = v->shape[1], be = (size_t)f->block_elems;
    if (d0 % be == 0 && d1 % be != 0) {
        *rows = d1;
        *cols = d0;
    } else if (d1 % be == 0 && d0 % be != 0) {
        *rows = d0;
        *cols = d1;
    } else {
        *rows = d1;
        *cols = d0;
    }
    return JKB_OK;
}

// Stages the raw GGUF bytes on the device (a load-time temporary) and reads the I2_S trailer.
int stage_raw(const jkb_tensor_view *v, size_t need, cudaStream_t st, uint8_t **dev,
              bool *owned) {
    if (v->data_on_device) {
        *dev = (uint8_t *)v->data;
        *owned = false;
        return JKB_OK;
    }
    cudaError_t e = cudaMalloc(dev, need);
    if (e != cudaSuccess) return fail_cuda(e, "weight upload (staging)");
    *owned = true;
    e = cudaMemcpyAsync(*dev, v->data, need, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
        cudaFree(*dev);
        return fail_cuda(e, "weight upload (copy)");
    }
    return JKB_OK;
}

static float read_i2s_trailer(const jkb_tensor_view *v, size_t payload) {
    float s = 0.0f;
    if (v->data_on_device)
        cudaMemcpy(&s, (const uint8_t *)v->data + payload, 4, cudaMemcpyDeviceToHost);
    else
        memcpy(&s, (const uint8_t *)v->data + payload, 4);
    // read_i2_s_trailer_scale (quant.rs:360-366): non-finite -> 0.0
    uint32_t u;
    memcpy(&u, &s, 4);
    return ((u >> 23) & 0xFF) == 0xFF ? 0.0f : s;
}

static int weight_upload(const jkb_tensor_view *v, size_t rows, size_t cols, cudaStream_t st,
                         jkb_weight **out) {
    if (!v || !out) return fail(JKB_E_INVALID, "jkb_weight_upload", 0, 0, 0, "null argument");
    *out = nullptr;
    const Fmt *f = fmt_of(v->quant);
    const char *nm = v->name ? v->name : "";
    // Q4_1, Q5_1, IQ4_NL, Q2_K and Q3_K have no block dot against Q8 activations in the
    // reference (quant_q8.rs): they exist only as RepackedWeights and nibble matrices
    const bool gemv_fmt = f && v->quant != JKB_Q4_1 && v->quant != JKB_Q5_1 &&
                          v->quant != JKB_IQ4_NL && v->quant != JKB_Q2_K && v->quant != JKB_Q3_K;
    if (!gemv_fmt)
        return fail(JKB_E_CAPABILITY, nm, v->offset, v->byte_len, v->byte_len,
                    "unsupported tensor quant %s for the GEMV layout", quant_name(v->quant));
    if (!v->data) return fail(JKB_E_INVALID, nm, v->offset, 0, 0, "null tensor data");
    int rc = validate_matrix_view(v, f, rows, cols);
    if (rc) return rc;

    jkb_weight *w = new jkb_weight();
    memset(w, 0, sizeof(*w));
    w->magic = WEIGHT_MAGIC;
    w->quant = v->quant;
    w->rows = rows;
    w->cols = cols;
    w->nb = cols / (size_t)f->block_elems;
    w->ndim = v->ndim;
    for (uint32_t i = 0; i < v->ndim && i < 4; i++) w->shape[i] = v->shape[i];
    snprintf(w->name, sizeof(w->name), "%s", nm);
    w->offset = v->offset;
    w->byte_len = v->byte_len;
    w->gguf_bytes = storage_bytes(f, rows * cols);

    size_t qp = 0, scp = 0;
    bool has_d = false;
    switch (v->quant) {
    case JKB_Q4_0: qp = 16; has_d = true; w->gpu_format = GF_Q4_0; break;
    case JKB_Q8_0: qp = 32; has_d = true; w->gpu_format = GF_Q8_0; break;
    case JKB_Q4_K_M: qp = 128; scp = 16; w->gpu_format = GF_Q4_K; break;
    case JKB_Q6_K: qp = 192; scp = 16; has_d = true; w->gpu_format = GF_Q6_K; break;
    case JKB_Q5_0: qp = 16; scp = 4; has_d = true; w->gpu_format = GF_Q5_0; break;
    case JKB_Q5_K: qp = 160; scp = 16; w->gpu_format = GF_Q5_K; break;
    case JKB_TQ1_0:
    case JKB_TQ2_0: qp = 64; has_d = true; w->gpu_format = GF_TQ2_0; break;
    case JKB_I2_S: qp = 32; w->gpu_format = GF_I2_S; break;
    }
    Arena a;
    size_t qs_bytes = rows * w->nb * qp, sc_bytes = rows * w->nb * scp,
           d_bytes = has_d ? rows * w->nb * 2 : 0;
    a.cap = Arena::round(qs_bytes) + Arena::round(sc_bytes) + Arena::round(d_bytes);
    cudaError_t e = cudaMalloc(&a.base, a.cap);
    if (e != cudaSuccess) {
        delete w;
        return fail_cuda(e, "jkb_weight_upload (device planes)");
    }
    w->base = a.base;
    w->device_bytes = a.cap;
    uint8_t *qs = a.take(qs_bytes);
    uint8_t *sc = scp ? a.take(sc_bytes) : nullptr;
    uint16_t *d = has_d ? (uint16_t *)a.take(d_bytes) : nullptr;
    w->p.qs = qs;
    w->p.qs_row = w->nb * qp;
    w->p.sc = sc;
    w->p.sc_row = w->nb * scp;
    w->p.d = d;
    size_t payload = rows * w->nb * (size_t)f->block_bytes;
    if (v->quant == JKB_I2_S) w->p.i2s_scale = read_i2s_trailer(v, payload);

    uint8_t *raw = nullptr;
    bool owned = false;
    rc = stage_raw(v, payload, st, &raw, &owned);
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    size_t n = rows * w->nb;
    relayout_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        v->quant, w->gpu_format, raw, rows, w->nb, w->nb * (size_t)f->block_bytes,
        f->block_bytes, qs, w->p.qs_row, sc, w->p.sc_row, d);
    rc = check_launch("relayout_kernel");
    // The GEMV kernels may issue their first weight loads before their programmatic-launch
    // wait (weights never depend on the kernel before them), so a handle is returned only once
    // its planes are written.
    const cudaError_t se = cudaStreamSynchronize(st);
    if (!rc && se != cudaSuccess) rc = fail_cuda(se, "jkb_weight_upload");
    if (owned) cudaFree(raw);
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    *out = w;
    return JKB_OK;
}

// RepackedWeight::dequantize_row (repack.rs:2529-2598), BlockScaledI8 storage: per element
// scale * q - min of its group, two roundings.
__global__ void repacked_dequant_row_kernel(const int8_t *__restrict__ q,
                                            const float *__restrict__ scales,
                                            const float *__restrict__ mins, size_t cols,
                                            int group_elems, float *__restrict__ out) {
    const size_t c = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const size_t g = c / (size_t)group_elems;
    const float wm = mins ? mins[g] : 0.0f;
    out[c] = __fsub_rn(__fmul_rn(scales[g], (float)q[c]), wm);
}

static int repacked_upload(const jkb_tensor_view *v, size_t rows, size_t cols, cudaStream_t st,
                           jkb_repacked_weight **out) {
    if (!v || !out)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null argument");
    *out = nullptr;
    const char *nm = v->name ? v->name : "";
    const Fmt *f = fmt_of(v->quant);
    if (!f)
        // Dense F32/F16/BF16 storage (RepackedStorage::DenseF32/DenseHalf) and the formats
        // outside the hot path are not built on the GPU.
        return fail(JKB_E_CAPABILITY, nm, v->offset, v->byte_len, v->byte_len,
                    "unsupported tensor quant %s for repack", quant_name(v->quant));
    if (!v->data) return fail(JKB_E_INVALID, nm, v->offset, 0, 0, "null tensor data");
    int rc = validate_matrix_view(v, f, rows, cols);
    if (rc) return rc;
    jkb_repacked_weight *w = new jkb_repacked_weight();
    memset(w, 0, sizeof(*w));
    w->magic = REPACKED_MAGIC;
    w->quant = v->quant;
    w->rows = rows;
    w->cols = cols;
    w->k_pad = (cols + 31) / 32 * 32;
    // BlockScaledTileLayout::from_validated_dims (repack.rs:1338-1366)
    w->group_elems =
        (v->quant == JKB_Q6_K || v->quant == JKB_Q3_K || v->quant == JKB_Q2_K) ? 16 : 32;
    w->scale_groups = w->k_pad / w->group_elems;
    snprintf(w->name, sizeof(w->name), "%s", nm);
    bool mins = v->quant == JKB_Q4_K_M || v->quant == JKB_Q5_K || v->quant == JKB_Q4_1 ||
                v->quant == JKB_Q5_1 || v->quant == JKB_Q2_K;
    Arena a;
    size_t qb = rows * w->k_pad, sb = rows * w->scale_groups * 4;
    a.cap = Arena::round(qb) + Arena::round(sb) * (mins ? 2 : 1);
    cudaError_t e = cudaMalloc(&a.base, a.cap);
    if (e != cudaSuccess) {
        delete w;
        return fail_cuda(e, "jkb_repacked_weight (device buffers)");
    }
    w->base = a.base;
    w->device_bytes = a.cap;
    w->q = (int8_t *)a.take(qb);
    w->scales = (float *)a.take(sb);
    w->mins = mins ? (float *)a.take(sb) : nullptr;
    size_t nb = cols / (size_t)f->block_elems;
    size_t payload = rows * nb * (size_t)f->block_bytes;
    float i2s = v->quant == JKB_I2_S ? read_i2s_trailer(v, payload) : 0.0f;
    uint8_t *raw = nullptr;
    bool owned = false;
    rc = stage_raw(v, payload, st, &raw, &owned);
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    cudaMemsetAsync(w->q, 0, qb, st);
    size_t n = rows * nb;
    repack_i8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        v->quant, raw, rows, nb, nb * (size_t)f->block_bytes, f->block_bytes, i2s, w->q,
        w->k_pad, w->scales, w->mins, w->scale_groups);
    rc = check_launch("repack_i8_kernel");
    if (owned) {
        cudaStreamSynchronize(st);
        cudaFree(raw);
    }
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    *out = w;
    return JKB_OK;
}


// ---- parallel load path: BlockScaledTileLayout, repack_into_tile_range, from_tile_buffers ----
// The reference tile layout (repack.rs:1286-1449): tiles [n_tile][k_chunk] of 128 bytes, each
// 8 weight rows x 16 K values (row j of the tile at bytes 16j .. 16j + 16); scales and mins
// [n_tile][scale_group][8] f32. These host buffers are what a loader fills on worker threads;
// from_tile_buffers uploads them and converts them to the device layout above.
constexpr size_t TILE_N = 8, TILE_K = 16, TILE_BYTES = 128;

// BlockScaledTileLayout::for_tensor (repack.rs:1308-1336) and from_validated_dims
// (:1338-1366) for an explicit [rows, cols] interpretation.
static int block_layout(const jkb_tensor_view *v, size_t rows, size_t cols, const char *fn,
                        jkb_block_scaled_tile_layout *L) {
    const char *nm = v->name ? v->name : "";
    const Fmt *f = fmt_of(v->quant);
    if (!f)
        return fail(JKB_E_CAPABILITY, nm, v->offset, v->byte_len, v->byte_len,
                    "%s: unsupported tensor quant %s", fn, quant_name(v->quant));
    int rc = validate_matrix_view(v, f, rows, cols);
    if (rc) return rc;
    memset(L, 0, sizeof(*L));
    L->quant = v->quant;
    L->rows = rows;
    L->cols = cols;
    L->row_bytes = cols / (size_t)f->block_elems * (size_t)f->block_bytes;
    L->k_padded = (cols + 31) / 32 * 32;
    L->n_tiles = (rows + TILE_N - 1) / TILE_N;
    L->k_chunks = L->k_padded / TILE_K;
    L->chunks_per_scale = repack_group_elems(v->quant) == 16 ? 1 : 2;
    L->scale_groups = L->k_chunks / L->chunks_per_scale;
    L->has_mins = repack_has_mins(v->quant) ? 1 : 0;
    L->total_tiles = L->n_tiles * L->k_chunks;
    L->total_scales = L->n_tiles * L->scale_groups * TILE_N;
    L->total_mins = L->has_mins ? L->total_scales : 0;
    return JKB_OK;
}

// repack_block_scaled_range_into_i8 (repack.rs:1724-2103) on the host for tiles [t0, t1):
// zero-fills the outputs, then expands every block of every row of those tiles with the shared
// decoder and scatters its values into the tile layout. No heap allocation.
static void repack_tiles_host(const jkb_block_scaled_tile_layout &L, const uint8_t *raw, float i2s,
                              size_t t0, size_t t1, int8_t *tiles, float *scales, float *mins) {
    const size_t tile_stride = L.k_chunks * TILE_BYTES, sc_stride = L.scale_groups * TILE_N;
    memset(tiles, 0, (t1 - t0) * tile_stride);
    memset(scales, 0, (t1 - t0) * sc_stride * 4);
    if (mins) memset(mins, 0, (t1 - t0) * sc_stride * 4);
    const Fmt *f = fmt_of(L.quant);
    const int be = repack_block_elems(L.quant), ge = repack_group_elems(L.quant), gpb = be / ge;
    const size_t nb = L.cols / (size_t)be;
    int8_t qb[256];
    float sb[16], mb[16];
    for (size_t nt = t0; nt < t1; nt++) {
        int8_t *tb = tiles + (nt - t0) * tile_stride;
        float *st = scales + (nt - t0) * sc_stride;
        float *mt = mins ? mins + (nt - t0) * sc_stride : nullptr;
        for (size_t j = 0; j < TILE_N; j++) {
            const size_t row = nt * TILE_N + j;
            if (row >= L.rows) break;
            const uint8_t *rr = raw + row * L.row_bytes;
            for (size_t b = 0; b < nb; b++) {
                repack_block_i8(L.quant, rr + b * (size_t)f->block_bytes, qb, sb, mb, i2s);
                for (int e = 0; e < be; e++) {
                    const size_t k = b * (size_t)be + (size_t)e;
                    tb[(k / TILE_K) * TILE_BYTES + j * TILE_K + k % TILE_K] = qb[e];
                }
                for (int g = 0; g < gpb; g++) {
                    st[(b * (size_t)gpb + (size_t)g) * TILE_N + j] = sb[g];
                    if (mt) mt[(b * (size_t)gpb + (size_t)g) * TILE_N + j] = mb[g];
                }
            }
        }
    }
}

// The reference tile layout -> the device layout: one thread per (row, 16-byte K chunk) and per
// (row, scale group).
__global__ void detile_kernel(const uint8_t *__restrict__ tiles, const float *__restrict__ sc,
                              const float *__restrict__ mn, size_t rows, size_t k_chunks,
                              size_t groups, int8_t *__restrict__ q, size_t k_pad,
                              float *__restrict__ scales, float *__restrict__ mins) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t nq = rows * k_chunks;
    if (idx < nq) {
        const size_t r = idx / k_chunks, ch = idx % k_chunks;
        const uint4 *src = reinterpret_cast<const uint4 *>(
            tiles + (r / TILE_N) * k_chunks * TILE_BYTES + ch * TILE_BYTES + (r % TILE_N) * TILE_K);
        *reinterpret_cast<uint4 *>(q + r * k_pad + ch * TILE_K) = *src;
        return;
    }
    const size_t i = idx - nq;
    if (i >= rows * groups) return;
    const size_t r = i / groups, g = i % groups;
    const size_t at = (r / TILE_N) * groups * TILE_N + g * TILE_N + r % TILE_N;
    scales[r * groups + g] = sc[at];
    if (mins) mins[r * groups + g] = mn[at];
}

static int check_tile_range(const jkb_tensor_view *v, const jkb_block_scaled_tile_layout &L,
                            size_t t0, size_t t1) {
    if (t0 > t1 || t1 > L.n_tiles)
        return fail(JKB_E_BOUNDS, v->name ? v->name : "", t0, t1 > t0 ? t1 - t0 : 0, L.n_tiles,
                    "tile_range %zu..%zu exceeds n_tiles (%zu)", t0, t1, L.n_tiles);
    return JKB_OK;
}

static int host_raw(const jkb_tensor_view *v, const char *fn, const uint8_t **raw) {
    if (!v->data || v->data_on_device)
        return fail(JKB_E_INVALID, v->name ? v->name : "", v->offset, v->byte_len, v->byte_len,
                    "%s reads host bytes", fn);
    *raw = (const uint8_t *)v->data;
    return JKB_OK;
}

}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_weight_upload(const jkb_tensor_view *view, size_t rows, size_t cols, void *stream,
                      jkb_weight **out) {
    return weight_upload(view, rows, cols, as_stream(stream), out);
}

int jkb_weight_upload_infer(const jkb_tensor_view *view, void *stream, jkb_weight **out) {
    if (!view || !out) return fail(JKB_E_INVALID, "jkb_weight_upload_infer", 0, 0, 0, "null");
    const Fmt *f = fmt_of(view->quant);
    if (!f)
        return fail(JKB_E_CAPABILITY, view->name ? view->name : "", view->offset,
                    view->byte_len, view->byte_len, "unsupported tensor quant %s",
                    quant_name(view->quant));
    size_t r = 0, c = 0;
    int rc = infer_rows_cols(view, f, &r, &c, "RepackedWeight::repack");
    if (rc) return rc;
    return weight_upload(view, r, c, as_stream(stream), out);
}

int jkb_weight_destroy(jkb_weight *w) {
    int rc = check_weight(w);
    if (rc) return rc;
    w->magic = 0;
    cudaFree(w->base);
    delete w;
    return JKB_OK;
}

int jkb_weight_info(const jkb_weight *w, size_t *rows, size_t *cols, int32_t *quant,
                    size_t *device_bytes, size_t *gguf_bytes) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (quant) *quant = w->quant;
    if (device_bytes) *device_bytes = w->device_bytes;
    if (gguf_bytes) *gguf_bytes = w->gguf_bytes;
    return JKB_OK;
}

int jkb_repacked_weight_from_tensor(const jkb_tensor_view *view, size_t rows, size_t cols,
                                    void *stream, jkb_repacked_weight **out) {
    return repacked_upload(view, rows, cols, as_stream(stream), out);
}

int jkb_repacked_weight_repack(const jkb_tensor_view *view, void *stream,
                               jkb_repacked_weight **out) {
    if (!view || !out) return fail(JKB_E_INVALID, "jkb_repacked_weight_repack", 0, 0, 0, "null");
    const Fmt *f = fmt_of(view->quant);
    if (!f)
        return fail(JKB_E_CAPABILITY, view->name ? view->name : "", view->offset,
                    view->byte_len, view->byte_len, "unsupported tensor quant %s for repack",
                    quant_name(view->quant));
    size_t r = 0, c = 0;
    int rc = infer_rows_cols(view, f, &r, &c, "RepackedWeight::repack");
    if (rc) return rc;
    return repacked_upload(view, r, c, as_stream(stream), out);
}

int jkb_repacked_weight_destroy(jkb_repacked_weight *w) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null or destroyed handle");
    w->magic = 0;
    cudaFree(w->base);
    delete w;
    return JKB_OK;
}

int jkb_repacked_weight_dequantize_row(const jkb_repacked_weight *w, size_t row, float *out,
                                       size_t out_len, void *stream) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null or destroyed handle");
    if (row >= w->rows || out_len != w->cols)
        return fail(JKB_E_BOUNDS, "RepackedWeight::dequantize_row", row, out_len * 4,
                    w->cols * 4, "invalid row (%zu/%zu) or output length (%zu/%zu)", row,
                    w->rows, out_len, w->cols);
    if (!out) return fail(JKB_E_INVALID, "RepackedWeight::dequantize_row", 0, 0, 0, "null output");
    int rc = check_align(out, 4, "RepackedWeight::dequantize_row", "output");
    if (rc) return rc;
    repacked_dequant_row_kernel<<<(unsigned)((w->cols + 255) / 256), 256, 0, as_stream(stream)>>>(
        w->q + row * w->k_pad, w->scales + row * w->scale_groups,
        w->mins ? w->mins + row * w->scale_groups : nullptr, w->cols, (int)w->group_elems, out);
    return check_launch("repacked_dequant_row_kernel");
}

int jkb_repacked_weight_buffers(const jkb_repacked_weight *w, size_t *rows, size_t *cols,
                                int32_t *quant, size_t *scale_groups, int8_t **q,
                                float **scales, float **mins) {
    if (!w || w->magic != REPACKED_MAGIC)
        return fail(JKB_E_INVALID, "jkb_repacked_weight", 0, 0, 0, "null or destroyed handle");
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (quant) *quant = w->quant;
    if (scale_groups) *scale_groups = w->scale_groups;
    if (q) *q = w->q;
    if (scales) *scales = w->scales;
    if (mins) *mins = w->mins;
    return JKB_OK;
}


int jkb_block_scaled_layout(const jkb_tensor_view *view, size_t rows, size_t cols,
                            jkb_block_scaled_tile_layout *out) {
    if (!view || !out) return fail(JKB_E_INVALID, "block_scaled_layout", 0, 0, 0, "null argument");
    return block_layout(view, rows, cols, "block_scaled_layout", out);
}

int jkb_repack_into_tile_range(const jkb_tensor_view *view, size_t rows, size_t cols,
                               size_t tile_begin, size_t tile_end, uint8_t *out_tiles,
                               size_t n_out_tiles, float *out_scales, size_t n_scales,
                               float *out_mins, size_t n_mins) {
    static const char *fn = "repack_into_tile_range";
    if (!view) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null view");
    jkb_block_scaled_tile_layout L;
    int rc = block_layout(view, rows, cols, fn, &L);
    if (rc || (rc = check_tile_range(view, L, tile_begin, tile_end))) return rc;
    const char *nm = view->name ? view->name : "";
    const size_t sub = tile_end - tile_begin, exp_tiles = sub * L.k_chunks,
                 exp_scales = sub * L.scale_groups * TILE_N;
    if (n_out_tiles != exp_tiles || n_scales != exp_scales ||
        (exp_tiles && (!out_tiles || !out_scales)))
        return fail(JKB_E_BOUNDS, nm, tile_begin, n_out_tiles, exp_tiles,
                    "tile/scale slice lengths (%zu, %zu) != expected (%zu, %zu)", n_out_tiles,
                    n_scales, exp_tiles, exp_scales);
    if (L.has_mins) {
        if (!out_mins)
            return fail(JKB_E_BOUNDS, nm, tile_begin, 0, exp_scales, "%s requires out_mins slice",
                        quant_name(L.quant));
        if (n_mins != exp_scales)
            return fail(JKB_E_BOUNDS, nm, tile_begin, n_mins, exp_scales,
                        "out_mins length %zu != expected %zu", n_mins, exp_scales);
    }
    const uint8_t *raw = nullptr;
    if ((rc = host_raw(view, fn, &raw))) return rc;
    if (sub == 0) return JKB_OK;
    const float i2s = L.quant == JKB_I2_S ? read_i2s_trailer(view, L.rows * L.row_bytes) : 0.0f;
    repack_tiles_host(L, raw, i2s, tile_begin, tile_end, (int8_t *)out_tiles, out_scales,
                      L.has_mins ? out_mins : nullptr);
    return JKB_OK;
}

int jkb_repack_q4_k_m_parallel_slices(const jkb_tensor_view *view, size_t rows, size_t cols,
                                      size_t tile_begin, size_t tile_end, int8_t *out_tiles_i8,
                                      size_t tiles_len, float *out_scales, size_t n_scales,
                                      float *out_mins, size_t n_mins) {
    static const char *fn = "repack_q4_k_m_parallel_slices";
    if (!view) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null view");
    const char *nm = view->name ? view->name : "";
    if (view->quant != JKB_Q4_K_M)
        return fail(JKB_E_CAPABILITY, nm, view->offset, view->byte_len, view->byte_len,
                    "%s: unsupported tensor quant %s", fn, quant_name(view->quant));
    jkb_block_scaled_tile_layout L;
    int rc = block_layout(view, rows, cols, fn, &L);
    if (rc || (rc = check_tile_range(view, L, tile_begin, tile_end))) return rc;
    const size_t sub = tile_end - tile_begin, exp_bytes = sub * L.k_chunks * TILE_BYTES,
                 exp_scales = sub * L.scale_groups * TILE_N;
    if (tiles_len != exp_bytes || n_scales != exp_scales || n_mins != exp_scales ||
        (exp_bytes && (!out_tiles_i8 || !out_scales || !out_mins)))
        return fail(JKB_E_BOUNDS, nm, tile_begin, tiles_len, exp_bytes,
                    "parallel slice lengths (%zu, %zu, %zu) != expected (%zu, %zu, %zu)",
                    tiles_len, n_scales, n_mins, exp_bytes, exp_scales, exp_scales);
    const uint8_t *raw = nullptr;
    if ((rc = host_raw(view, fn, &raw))) return rc;
    if (sub == 0) return JKB_OK;
    repack_tiles_host(L, raw, 0.0f, tile_begin, tile_end, out_tiles_i8, out_scales, out_mins);
    return JKB_OK;
}

int jkb_repacked_weight_from_tile_buffers(const jkb_block_scaled_tile_layout *layout,
                                          const uint8_t *tiles, size_t n_tiles,
                                          const float *scales, size_t n_scales,
                                          const float *mins, size_t n_mins, void *stream,
                                          jkb_repacked_weight **out) {
    static const char *fn = "RepackedWeight::from_tile_buffers";
    if (!layout || !out) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null argument");
    *out = nullptr;
    const jkb_block_scaled_tile_layout &L = *layout;
    // the layout must be one block_scaled_layout produced (its fields follow from quant, rows
    // and cols)
    const Fmt *f = fmt_of(L.quant);
    if (!f) return fail(JKB_E_CAPABILITY, fn, 0, 0, 0, "unsupported tensor quant %s",
                        quant_name(L.quant));
    const size_t kp = (L.cols + 31) / 32 * 32, ge = (size_t)repack_group_elems(L.quant);
    if (L.rows == 0 || L.cols == 0 || L.cols % (size_t)f->block_elems || L.k_padded != kp ||
        L.n_tiles != (L.rows + TILE_N - 1) / TILE_N || L.k_chunks != kp / TILE_K ||
        L.chunks_per_scale != ge / TILE_K || L.scale_groups != kp / ge ||
        L.has_mins != (repack_has_mins(L.quant) ? 1 : 0) ||
        L.row_bytes != L.cols / (size_t)f->block_elems * (size_t)f->block_bytes ||
        L.total_tiles != L.n_tiles * L.k_chunks ||
        L.total_scales != L.n_tiles * L.scale_groups * TILE_N ||
        L.total_mins != (L.has_mins ? L.total_scales : 0))
        return fail(JKB_E_BOUNDS, fn, 0, 0, 0,
                    "layout fields do not describe a %s [%zu, %zu] block-scaled layout",
                    quant_name(L.quant), L.rows, L.cols);
    if (n_tiles != L.total_tiles || n_scales != L.total_scales)
        return fail(JKB_E_BOUNDS, fn, 0, n_tiles, L.total_tiles,
                    "buffer lengths (%zu, %zu) != expected (%zu, %zu)", n_tiles, n_scales,
                    L.total_tiles, L.total_scales);
    if (L.has_mins) {
        if (!mins || n_mins != L.total_mins)
            return fail(JKB_E_BOUNDS, fn, 0, mins ? n_mins : 0, L.total_mins,
                        "%s requires mins buffer of length %zu", quant_name(L.quant),
                        L.total_mins);
    } else if (mins) {
        return fail(JKB_E_BOUNDS, fn, 0, n_mins, 0, "%s does not use mins buffer",
                    quant_name(L.quant));
    }
    if (!tiles || !scales) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null buffer");
    cudaStream_t st = as_stream(stream);
    jkb_repacked_weight *w = new jkb_repacked_weight();
    memset(w, 0, sizeof(*w));
    w->magic = REPACKED_MAGIC;
    w->quant = L.quant;
    w->rows = L.rows;
    w->cols = L.cols;
    w->k_pad = kp;
    w->group_elems = ge;
    w->scale_groups = L.scale_groups;
    snprintf(w->name, sizeof(w->name), "%s", "from_tile_buffers");
    Arena a;
    const size_t qb = L.rows * kp, sb = L.rows * L.scale_groups * 4;
    a.cap = Arena::round(qb) + Arena::round(sb) * (L.has_mins ? 2 : 1);
    // staging of the host tiles (freed before returning): tiles, scales, mins
    const size_t tb = L.total_tiles * TILE_BYTES, ssb = L.total_scales * 4;
    Arena s;
    s.cap = Arena::round(tb) + Arena::round(ssb) * (L.has_mins ? 2 : 1);
    cudaError_t e = cudaMalloc(&a.base, a.cap);
    if (e != cudaSuccess) {
        delete w;
        return fail_cuda(e, "from_tile_buffers (device buffers)");
    }
    e = cudaMalloc(&s.base, s.cap);
    if (e != cudaSuccess) {
        cudaFree(a.base);
        delete w;
        return fail_cuda(e, "from_tile_buffers (staging)");
    }
    w->base = a.base;
    w->device_bytes = a.cap;
    w->q = (int8_t *)a.take(qb);
    w->scales = (float *)a.take(sb);
    w->mins = L.has_mins ? (float *)a.take(sb) : nullptr;
    uint8_t *d_tiles = s.take(tb);
    float *d_sc = (float *)s.take(ssb), *d_mn = L.has_mins ? (float *)s.take(ssb) : nullptr;
    cudaMemcpyAsync(d_tiles, tiles, tb, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(d_sc, scales, ssb, cudaMemcpyHostToDevice, st);
    if (d_mn) cudaMemcpyAsync(d_mn, mins, ssb, cudaMemcpyHostToDevice, st);
    const size_t n = L.rows * (L.k_chunks + L.scale_groups);
    detile_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(d_tiles, d_sc, d_mn, L.rows,
                                                               L.k_chunks, L.scale_groups, w->q,
                                                               kp, w->scales, w->mins);
    int rc = check_launch("detile_kernel");
    e = cudaStreamSynchronize(st);
    cudaFree(s.base);
    if (!rc && e != cudaSuccess) rc = fail_cuda(e, "from_tile_buffers");
    if (rc) {
        cudaFree(a.base);
        delete w;
        return rc;
    }
    *out = w;
    return JKB_OK;
}

}  // extern "C"
