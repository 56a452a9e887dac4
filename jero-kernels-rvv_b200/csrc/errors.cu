// Error records, the quant format table and the reference shape validators.
#include <cstdio>
#include <cstring>

#include "jkb_internal.h"

namespace jkb {

static thread_local jkb_error_info g_err = {JKB_OK, {0}, 0, 0, 0, {0}};
static thread_local char g_msg[512];

int fail(int status, const char *tensor, size_t offset, size_t byte_len, size_t buffer_len,
         const char *fmt, ...) {
    g_err.status = status;
    snprintf(g_err.tensor_name, sizeof(g_err.tensor_name), "%s", tensor ? tensor : "");
    g_err.offset = offset;
    g_err.byte_len = byte_len;
    g_err.buffer_len = buffer_len;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err.reason, sizeof(g_err.reason), fmt, ap);
    va_end(ap);
    return status;
}

int fail_cuda(cudaError_t e, const char *where) {
    return fail(JKB_E_CUDA, where, 0, 0, 0, "%s: CUDA error %d (%s)", where, (int)e,
                cudaGetErrorString(e));
}

int check_align(const void *p, size_t align, const char *fn, const char *what) {
    if (((uintptr_t)p) % align == 0) return JKB_OK;
    return fail(JKB_E_BOUNDS, fn, (size_t)((uintptr_t)p % align), 0, align,
                "%s: %s pointer %p is not %zu-byte aligned", fn, what, p, align);
}

int check_launch(const char *where) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? JKB_OK : fail_cuda(e, where);
}

void clear_error() {
    g_err.status = JKB_OK;
    g_err.tensor_name[0] = 0;
    g_err.reason[0] = 0;
    g_err.offset = g_err.byte_len = g_err.buffer_len = 0;
}

// Block geometry (quant.rs:20-91, ime.rs:28-37, lib.rs:129-132). I2_S carries a 32-byte
// per-tensor scale trailer after the payload (quant.rs:85-91).
static const Fmt FMTS[] = {
    {JKB_Q4_0, "Q4_0", 32, 18, 0},     {JKB_Q8_0, "Q8_0", 32, 34, 0},
    {JKB_Q4_K_M, "Q4_K_M", 256, 144, 0}, {JKB_Q6_K, "Q6_K", 256, 210, 0},
    {JKB_TQ1_0, "TQ1_0", 256, 54, 0},  {JKB_TQ2_0, "TQ2_0", 256, 66, 0},
    {JKB_I2_S, "I2_S", 128, 32, 32},  {JKB_Q5_0, "Q5_0", 32, 22, 0},
    {JKB_Q5_K, "Q5_K", 256, 176, 0},   {JKB_Q4_1, "Q4_1", 32, 20, 0},
    {JKB_Q5_1, "Q5_1", 32, 24, 0},     {JKB_IQ4_NL, "IQ4_NL", 32, 18, 0},
    {JKB_Q2_K, "Q2_K", 256, 84, 0},    {JKB_Q3_K, "Q3_K", 256, 110, 0},
};

const Fmt *fmt_of(int quant) {
    for (const Fmt &f : FMTS)
        if (f.quant == quant) return &f;
    return nullptr;
}

const char *quant_name(int quant) {
    switch (quant) {
    case JKB_F32: return "F32";
    case JKB_F16: return "F16";
    case JKB_BF16: return "BF16";
    default: {
        const Fmt *f = fmt_of(quant);
        return f ? f->name : "Unknown";
    }
    }
}

int num_sms() {
    static thread_local int cached_dev = -1, cached_sms = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != cached_dev) {
        cudaDeviceGetAttribute(&cached_sms, cudaDevAttrMultiProcessorCount, dev);
        cached_dev = dev;
    }
    return cached_sms > 0 ? cached_sms : 148;
}

// validate_quant_matvec_dimensions quant.rs:1810-1894 (same rule as validate_q8_0_dimensions
// :762, validate_q6_k_dimensions :828, validate_q4_0_dimensions :1315 and
// validate_q4_k_m_dimensions lib.rs:1195): 2-D [rows, cols] or [cols, rows] with the input
// dimension a multiple of the block size; 1-D needs output_len * input_len == elements.
int validate_matvec_shape(const char *tensor, size_t offset, size_t byte_len, size_t buffer_len,
                          int quant, const size_t *shape, uint32_t ndim, size_t output_len,
                          size_t input_len, size_t *rows, size_t *cols) {
    const Fmt *f = fmt_of(quant);
    if (!f)
        return fail(JKB_E_CAPABILITY, tensor, offset, byte_len, buffer_len,
                    "unsupported tensor quant %s", quant_name(quant));
    if (ndim == 0)
        return fail(JKB_E_BOUNDS, tensor, offset, byte_len, buffer_len, "empty tensor shape");
    size_t be = (size_t)f->block_elems;
    if (ndim == 2) {
        size_t d0 = shape[0], d1 = shape[1];
        if (output_len == d0 && input_len == d1 && d1 % be == 0) {
            *rows = d0;
            *cols = d1;
        } else if (output_len == d1 && input_len == d0 && d0 % be == 0) {
            *rows = d1;
            *cols = d0;
        } else {
            return fail(JKB_E_BOUNDS, tensor, offset, byte_len, buffer_len,
                        "matrix shape [%zu, %zu] does not match output len %zu and %s-aligned "
                        "input len %zu",
                        d0, d1, output_len, f->name, input_len);
        }
    } else {
        size_t total = 1;
        for (uint32_t i = 0; i < ndim; i++) total *= shape[i];
        if (input_len == 0 || output_len == 0 || input_len % be != 0 ||
            output_len * input_len != total)
            return fail(JKB_E_BOUNDS, tensor, offset, byte_len, buffer_len,
                        "tensor elements %zu do not match output len %zu * input len %zu", total,
                        output_len, input_len);
        *rows = output_len;
        *cols = input_len;
    }
    size_t need = storage_bytes(f, (*rows) * (*cols));
    if (buffer_len < need)
        return fail(JKB_E_BOUNDS, tensor, offset, byte_len, buffer_len,
                    "%s buffer length %zu < required %zu", f->name, buffer_len, need);
    return JKB_OK;
}

int check_weight(const jkb_weight *w) {
    if (!w || w->magic != WEIGHT_MAGIC)
        return fail(JKB_E_INVALID, "jkb_weight", 0, 0, 0, "null or destroyed weight handle");
    return JKB_OK;
}

int validate_weight_call(const char *fn, const jkb_weight *w, int expected_quant,
                         size_t output_len, size_t input_len) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (expected_quant >= 0 && w->quant != expected_quant)
        return fail(JKB_E_BOUNDS, w->name, w->offset, w->byte_len, w->gguf_bytes,
                    "expected %s quant type, got %s", quant_name(expected_quant),
                    quant_name(w->quant));
    size_t r = 0, c = 0;
    rc = validate_matvec_shape(w->name, w->offset, w->byte_len, w->gguf_bytes, w->quant, w->shape,
                               w->ndim, output_len, input_len, &r, &c);
    if (rc) return rc;
    if (r != w->rows || c != w->cols)
        return fail(JKB_E_BOUNDS, w->name, w->offset, w->byte_len, w->gguf_bytes,
                    "%s: call interprets the tensor as [%zu, %zu] but it was uploaded as "
                    "[%zu, %zu]",
                    fn, r, c, w->rows, w->cols);
    return JKB_OK;
}

// Device error word shared by the kernels with bounded waits: bit 0, a wait in the tensor-core
// GEMM expired; bit 1, a peer-group wait (peer.cu) expired. Kernels get its address as an
// argument; host code reads and clears it in jkb_device_status.
__device__ int g_device_error;

int *device_error_word() {
    static int *ptr_by_device[128] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return nullptr;
    if (!ptr_by_device[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        ptr_by_device[dev] = (int *)p;
    }
    return ptr_by_device[dev];
}

}  // namespace jkb

extern "C" {

int jkb_abi_version(void) { return JKB_ABI_VERSION; }

int jkb_device_status(int32_t *flags, void *stream) {
    using namespace jkb;
    if (!flags) return fail(JKB_E_INVALID, "device_status", 0, 0, 0, "null pointer");
    int *err = device_error_word();
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
                    "a bounded wait expired on the device (flags %d: bit 0 tensor-core GEMM, "
                    "bit 1 peer-group wait)",
                    v)
             : JKB_OK;
}

const char *jkb_last_error(void) {
    using namespace jkb;
    if (g_err.status == JKB_OK) return "";
    snprintf(g_msg, sizeof(g_msg),
             "TensorBoundsError{tensor_name: %s, offset: %zu, byte_len: %zu, buffer_len: %zu, "
             "reason: %s} (status %d)",
             g_err.tensor_name, g_err.offset, g_err.byte_len, g_err.buffer_len, g_err.reason,
             g_err.status);
    return g_msg;
}

int jkb_last_error_info(jkb_error_info *out) {
    if (!out) return JKB_E_INVALID;
    *out = jkb::g_err;
    return JKB_OK;
}

void jkb_clear_error(void) { jkb::clear_error(); }

}  // extern "C"
