// Internal host-side declarations shared by the .cu files of libjkb200.so.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "jkb200.h"

namespace jkb {

// ---- errors (errors.cu) ----
// Records a K3Error::TensorBoundsError-shaped failure for this thread and returns `status`.
int fail(int status, const char *tensor, size_t offset, size_t byte_len, size_t buffer_len,
         const char *fmt, ...) __attribute__((format(printf, 6, 7)));
int fail_cuda(cudaError_t e, const char *where);
// Rejects a device pointer that is not `align`-byte aligned (JKB_E_BOUNDS). Block activations
// carry an f32 field (align 4, like the reference #[repr(C)] structs); outputs are f32.
int check_align(const void *p, size_t align, const char *fn, const char *what);
// The device error word of kernels with bounded waits (per-device address; nullptr on failure).
int *device_error_word();
// Checks cudaGetLastError after a launch.
int check_launch(const char *where);
void clear_error();

// ---- quant format table ----
struct Fmt {
    int quant;
    const char *name;
    int block_elems;
    int block_bytes;
    int trailer_bytes;
};
const Fmt *fmt_of(int quant);  // nullptr for formats the hot path does not cover
const char *quant_name(int quant);

// Bytes of `n` logical elements in GGUF storage (QuantType::storage_bytes incl. trailer).
inline size_t storage_bytes(const Fmt *f, size_t n) {
    return n / (size_t)f->block_elems * (size_t)f->block_bytes + (size_t)f->trailer_bytes;
}

// ---- device buffers ----
// One cudaMalloc per handle; planes are carved at 256-byte boundaries.
struct Arena {
    uint8_t *base = nullptr;
    size_t used = 0, cap = 0;
    static size_t round(size_t n) { return (n + 255) & ~(size_t)255; }
    uint8_t *take(size_t n) {
        uint8_t *p = base + used;
        used += round(n);
        return p;
    }
};

// Load-time helpers shared by the weight handles (weights.cu): validate_matrix_view
// (repack.rs:1151-1284), the RepackedWeight::repack orientation rule (repack.rs:2255-2282) and
// the device staging of a view's raw bytes (*owned: a temporary the caller frees).
int validate_matrix_view(const jkb_tensor_view *v, const Fmt *f, size_t rows, size_t cols);
int infer_rows_cols(const jkb_tensor_view *v, const Fmt *f, size_t *rows, size_t *cols,
                    const char *who);
int stage_raw(const jkb_tensor_view *v, size_t need, cudaStream_t st, uint8_t **dev,
              bool *owned);

// GPU layout of one weight matrix (see weights.cu for the per-format plane contents).
struct WeightPlanes {
    const uint8_t *qs = nullptr;  // quant plane, row pitch qs_row bytes
    size_t qs_row = 0;
    const uint8_t *sc = nullptr;  // per-block scale plane: 16 B (Q4_K_M, Q5_K, Q6_K), 4 B (Q5_0 qh)
    size_t sc_row = 0;
    const uint16_t *d = nullptr;  // f16 block scales [rows][nb] (Q4_0, Q8_0, Q6_K, TQ*)
    float i2s_scale = 0.0f;       // I2_S per-tensor trailer scale (non-finite -> 0)
};

}  // namespace jkb

struct jkb_weight {
    uint32_t magic;
    int quant;       // source QuantType
    int gpu_format;  // kernel format (TQ1_0 is stored in the TQ2_0 GPU layout)
    size_t rows, cols, nb;
    uint32_t ndim;
    size_t shape[4];
    char name[64];
    size_t offset, byte_len, gguf_bytes;
    uint8_t *base;
    size_t device_bytes;
    jkb::WeightPlanes p;
};

struct jkb_repacked_weight {
    uint32_t magic;
    int quant;
    size_t rows, cols, k_pad, scale_groups, group_elems;
    char name[64];
    uint8_t *base;
    size_t device_bytes;
    int8_t *q;       // [rows][k_pad]
    float *scales;   // [rows][scale_groups]
    float *mins;     // [rows][scale_groups] or nullptr
};

// Compact 4-bit weight (PackedNibbleMatrix); plane layout in nibble.cuh.
struct jkb_nibble_matrix {
    uint32_t magic;
    int quant;            // JKB_Q4_0, JKB_Q4_1, JKB_IQ4_NL or JKB_Q4_K_M
    size_t rows, cols;
    size_t nb;            // format blocks per row (cols / 32, or cols / 256 for Q4_K_M)
    size_t meta_bytes;    // scale bytes per block: 2, 4 or 16
    char name[64];
    uint8_t *base;
    size_t device_bytes;  // allocation (planes rounded to 256 bytes)
    uint8_t *qs;          // [rows][cols / 2]
    uint8_t *meta;        // [rows][nb] x meta_bytes
};

struct jkb_act_q8 {
    uint32_t magic;
    size_t m_cap, k, k_pad, m;
    uint8_t *base;
    int8_t *q;            // [m_cap][k_pad]
    float *x_scales;      // [m_cap][k_pad/32]
    float *x_sums;        // [m_cap][k_pad/32]
    float *x_sums_16;     // [m_cap][k_pad/16]
    float *super_scales;  // [m_cap][ceil(k/256)]
    // x_scales transposed, [k_pad/32][xt_pitch] (xt_pitch = capacity rounded up to 32), tokens
    // permuted within 32-token blocks as the tensor-core GEMM epilogue reads them (see
    // act_q8_kernel). nullptr when the buffer has no room for it (the GEMM then takes the dp4a
    // path).
    float *x_scales_t;
    // -x_sums in the same transposed, permuted layout (the tensor-core GEMM's min term for
    // Q4_K_M weights); nullptr when x_scales_t is
    float *x_nsums_t;
    // -x_sums_16 in the same transposed, permuted layout, [k_pad/16][xt_pitch] (the min term of
    // 16-element groups, Q2_K); nullptr when x_scales_t is
    float *x_nsums16_t;
    size_t xt_pitch;
};

namespace jkb {
constexpr uint32_t WEIGHT_MAGIC = 0x4A4B5731u;    // "JKW1"
constexpr uint32_t REPACKED_MAGIC = 0x4A4B5231u;  // "JKR1"
constexpr uint32_t ACT_MAGIC = 0x4A4B4131u;       // "JKA1"
constexpr uint32_t NIBBLE_MAGIC = 0x4A4B4E31u;    // "JKN1"

int num_sms();
inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Launches with programmatic stream serialization: the kernel may start while the previous
// kernel in the stream finishes; it must execute griddepcontrol.wait before touching memory
// the previous kernel writes or reads. cluster_x > 1 launches thread-block clusters of
// cluster_x CTAs along x (grid.x must be a multiple of it).
template <class... KArgsT, class... ArgsT>
cudaError_t launch_pdl_cluster(void (*kern)(KArgsT...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t st, unsigned cluster_x, ArgsT... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cluster_x > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}
template <class... KArgsT, class... ArgsT>
cudaError_t launch_pdl(void (*kern)(KArgsT...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, ArgsT... args) {
    return launch_pdl_cluster(kern, grid, block, smem, st, 1u, args...);
}

// Reference validators over a stored 2-D/1-D shape (quant.rs:1810-1894 and its per-format
// twins quant.rs:762-892, :1315-1394, lib.rs:1195-1260): accepts [rows, cols] or GGUF
// [cols, rows]; writes the (rows, cols) interpretation.
int validate_matvec_shape(const char *tensor, size_t offset, size_t byte_len, size_t buffer_len,
                          int quant, const size_t *shape, uint32_t ndim, size_t output_len,
                          size_t input_len, size_t *rows, size_t *cols);
// Handle-level wrapper: runs the validator on the handle's shape and checks that the
// interpretation matches the orientation the handle was uploaded with.
int validate_weight_call(const char *fn, const jkb_weight *w, int expected_quant,
                         size_t output_len, size_t input_len);
int check_weight(const jkb_weight *w);

// gemv.cu entry used by bitlinear.cu and the sharded paths.
enum GpuFormat { GF_Q4_0, GF_Q8_0, GF_Q4_K, GF_Q6_K, GF_TQ2_0, GF_I2_S, GF_Q5_0, GF_Q5_K };
// ACT_F32_*: f32 input rows that every CTA quantizes into its shared-memory staging buffer with
// the bit-exact BlockQ8_0 / BlockQ8K quantizer (the reference's vec_dot_*_rvv paths).
enum ActKind { ACT_Q8_0 = 0, ACT_Q8_K = 1, ACT_I8 = 2, ACT_F32_Q8_0 = 3, ACT_F32_Q8_K = 4 };
constexpr int GEMV_MAX_MATS = 8;
struct GemvLaunch {
    const jkb_weight *w;     // the weight (the first one when nmat > 1)
    // nmat > 1: one launch over weights ws[0..nmat) that share format, cols and activation;
    // weight i writes outs[i][0..rows_i). row_begin/row_end/out/m are ignored (m = 1).
    int nmat;
    const jkb_weight *ws[GEMV_MAX_MATS];
    float *outs[GEMV_MAX_MATS];
    const void *x;           // activation rows (AoS blocks, i8 or f32)
    size_t x_row_stride;     // bytes between tokens (batch)
    int act_kind;
    const float *act_scales; // per-token scale (i8 activations, device) or nullptr
    float act_scale;         // per-tensor scale when act_scales == nullptr
    float *out;
    size_t out_ld;           // floats between tokens
    size_t row_begin, row_end;
    size_t m;                // tokens
    int32_t *dbg_sumi, *dbg_mins;
    float *dbg_val;
};
int launch_gemv(const GemvLaunch &L, cudaStream_t st);

// Output pushing (peer.cu): the peers of a peer group with push enabled, as byte offsets from an
// address in this rank's buffer to the same position in each peer's mapping of its buffer.
struct PushTarget {
    int n = 0;  // peers to store to (0: the range is in no pushing group)
    long long delta[JKB_PEER_MAX_RANKS - 1] = {};
    const void *group = nullptr;
};
// Looks up the byte range [lo, hi) among the buffers of this device's pushing peer groups:
// JKB_OK with t->n = 0 when it is in none, filled in when it lies inside one, JKB_E_BOUNDS when
// it crosses the edge of one. `who` names the caller in the error.
int push_lookup(const void *lo, const void *hi, PushTarget *t, const char *who);
// JKB_E_CAPABILITY when [lo, hi) overlaps a pushing group's buffer: for the entry points whose
// kernels write outputs without pushing them (the repacked GEMMs).
int push_reject(const void *lo, const void *hi, const char *who);

// Fills a jkb_act_q8 from i8 BitLinear activations with per-token scales (quantize.cu).
int act_q8_from_i8(jkb_act_q8 *a, const int8_t *act_i8, const float *scales, size_t m,
                   cudaStream_t st);
// Tensor-core BitLinear GEMM (gemm_tc.cu); *used = false when its conditions do not hold.
int gemm_tc_bitlinear_launch(const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                             cudaStream_t st, bool *used);

// validate_bitlinear_dimensions (ime.rs:660-763) on a handle (dots.cu).
int validate_bitlinear(const jkb_weight *w, size_t output_len, size_t input_len);

// subln_quantize_absmax_i8 over m rows of len (quantize.cu); gate: the rows are
// relu_squared_gate_f32(input, up), stored to relu_out when non-null. Arguments are validated
// by the caller; len <= SUBLN_MAX_LEN.
constexpr size_t SUBLN_MAX_LEN = 200 * 1024 / 4;
int launch_subln(bool gate, int8_t *out_i8, float *relu_out, const float *input,
                 const float *up, const float *norm_weight, size_t m, size_t len, float eps,
                 float *scales_out, cudaStream_t st);


}  // namespace jkb
