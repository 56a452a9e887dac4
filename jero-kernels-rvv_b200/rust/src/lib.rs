//! jero-kernels-rvv's quantized-matmul hot path on B200 (sm_100a), behind the crate's own public
//! signatures: the engine crates keep calling `quantize_row_q8_0(&[f32], &mut [BlockQ8_0])`,
//! `gemv_q4_k_q8_k(&mut [f32], &TensorView, &[BlockQ8K])`, `RepackedWeight::gemm`, ... and these
//! functions run the hand-written CUDA kernels of libjkb200.so through its C ABI
//! (include/jkb200.h, bound by bindgen in build.rs).
//!
//! Host slices stay host slices: each call copies its inputs to the calling thread's device
//! staging buffers on that thread's stream, runs the kernel, copies the outputs back and
//! synchronizes, so the caller sees the reference's synchronous semantics. Weights given as
//! `&TensorView` are uploaded (validated, relaid) on first use and cached by the address, length
//! and interpretation of their bytes, as a model's mmap'd tensors live for the process;
//! `release_weight` drops a cached upload. Engines that keep activations on the device use the
//! raw entry points of `ffi` with device pointers instead, which skip the staging copies.
//!
//! Errors: a failed call returns the K3Error the reference returns (same variant, tensor name,
//! offsets and reason text), built from the library's thread-local error record. Nothing runs on
//! the GPU when validation fails.
//!
//! Not compiled in this repository: the build image has no Rust toolchain and jero-core is not
//! vendored. The C ABI it binds is tested through ctypes (tests/test_abi_cpu.py and the
//! tests/test_gpu_*.py parity suites).

mod ffi;

use core::ffi::{c_int, c_void, CStr};
use std::cell::RefCell;
use std::collections::HashMap;
use std::ops::Range;
use std::sync::Mutex;

use jero_core::{K3Error, QuantType, TensorView};

/// quant_q8.rs:37-44 (36 bytes, the C ABI's jkb_block_q8_0).
#[repr(C)]
#[derive(Clone, Copy, Debug, PartialEq)]
pub struct BlockQ8_0 {
    pub d: f32,
    pub qs: [i8; 32],
}

/// quant_q8.rs:62-71 (292 bytes, the C ABI's jkb_block_q8_k).
#[repr(C)]
#[derive(Clone, Copy, Debug, PartialEq)]
pub struct BlockQ8K {
    pub d: f32,
    pub qs: [i8; 256],
    pub bsums: [i16; 16],
}

// ------------------------------------------------------------------------------------ errors

fn cstr(buf: &[core::ffi::c_char]) -> String {
    unsafe { CStr::from_ptr(buf.as_ptr()) }.to_string_lossy().into_owned()
}

/// The K3Error of the library's last failure on this thread (`op` and `quant` name the call for
/// a CapabilityMismatch, as K3Error::unsupported_tensor_quant does in the reference; calls that
/// cannot return one pass F32).
fn check(rc: c_int, op: &str, quant: QuantType) -> Result<(), K3Error> {
    if rc == ffi::jkb_status_JKB_OK as c_int {
        return Ok(());
    }
    let mut e = ffi::jkb_error_info::default();
    unsafe { ffi::jkb_last_error_info(&mut e) };
    let name = cstr(&e.tensor_name);
    if rc == ffi::jkb_status_JKB_E_CAPABILITY as c_int {
        return Err(K3Error::unsupported_tensor_quant(op, &name, quant));
    }
    Err(K3Error::TensorBoundsError {
        tensor_name: name,
        offset: e.offset,
        byte_len: e.byte_len,
        buffer_len: e.buffer_len,
        reason: cstr(&e.reason),
    })
}

fn cuda(rc: c_int, what: &str) -> Result<(), K3Error> {
    if rc == 0 {
        return Ok(());
    }
    Err(K3Error::TensorBoundsError {
        tensor_name: "jkb200".to_owned(),
        offset: 0,
        byte_len: 0,
        buffer_len: 0,
        reason: format!("CUDA error {rc} in {what}"),
    })
}

fn quant_code(q: QuantType) -> i32 {
    match q {
        QuantType::F32 => 0,
        QuantType::F16 => 1,
        QuantType::Q4_0 => 2,
        QuantType::Q4_1 => 3,
        QuantType::Q5_0 => 6,
        QuantType::Q5_1 => 7,
        QuantType::Q8_0 => 8,
        QuantType::Q2_K => 10,
        QuantType::Q3_K => 11,
        QuantType::Q4_K_M => 12,
        QuantType::Q5_K => 13,
        QuantType::Q6_K => 14,
        QuantType::IQ4_NL => 20,
        QuantType::BF16 => 30,
        QuantType::TQ1_0 => 34,
        QuantType::TQ2_0 => 35,
        QuantType::I2_S => 36,
        _ => -1, // formats the GPU path does not build: the library answers CapabilityMismatch
    }
}

// ------------------------------------------------------------------ per-thread device staging

/// A stream and grow-only device staging buffers per calling thread (the reference's functions
/// are synchronous and single-threaded per call; callers parallelize over threads).
struct Gpu {
    stream: *mut c_void,
    bufs: [(*mut c_void, usize); 3],
}

impl Gpu {
    fn new() -> Self {
        let mut s = core::ptr::null_mut();
        unsafe { ffi::cudaStreamCreate(&mut s) };
        Gpu { stream: s, bufs: [(core::ptr::null_mut(), 0); 3] }
    }

    /// Device buffer `i` of at least `n` bytes (allocated or grown on first use of a size).
    fn buf(&mut self, i: usize, n: usize) -> Result<*mut c_void, K3Error> {
        if self.bufs[i].1 < n {
            unsafe { ffi::cudaFree(self.bufs[i].0) };
            let mut p = core::ptr::null_mut();
            cuda(unsafe { ffi::cudaMalloc(&mut p, n.max(256)) }, "staging cudaMalloc")?;
            self.bufs[i] = (p, n.max(256));
        }
        Ok(self.bufs[i].0)
    }

    fn upload<T>(&mut self, i: usize, src: &[T]) -> Result<*mut c_void, K3Error> {
        let n = core::mem::size_of_val(src);
        let d = self.buf(i, n)?;
        cuda(unsafe { ffi::cudaMemcpyAsync(d, src.as_ptr().cast(), n,
                                           ffi::CUDA_MEMCPY_HOST_TO_DEVICE, self.stream) },
             "staging upload")?;
        Ok(d)
    }

    fn download<T>(&mut self, dst: &mut [T], src: *const c_void) -> Result<(), K3Error> {
        let n = core::mem::size_of_val(dst);
        cuda(unsafe { ffi::cudaMemcpyAsync(dst.as_mut_ptr().cast(), src, n,
                                           ffi::CUDA_MEMCPY_DEVICE_TO_HOST, self.stream) },
             "staging download")?;
        cuda(unsafe { ffi::cudaStreamSynchronize(self.stream) }, "stream synchronize")
    }
}

thread_local! {
    static GPU: RefCell<Gpu> = RefCell::new(Gpu::new());
}

fn with_gpu<R>(f: impl FnOnce(&mut Gpu) -> Result<R, K3Error>) -> Result<R, K3Error> {
    GPU.with(|g| f(&mut g.borrow_mut()))
}

// ------------------------------------------------------------------------- weight uploads

#[derive(Clone, Copy, PartialEq, Eq, Hash)]
struct WeightKey {
    addr: usize,
    len: usize,
    quant: i32,
    rows: usize,
    cols: usize,
}

struct Handle(*mut ffi::jkb_weight);
unsafe impl Send for Handle {}

static WEIGHTS: Mutex<Option<HashMap<WeightKey, Handle>>> = Mutex::new(None);

fn view_c(w: &TensorView<'_>, name: &std::ffi::CString) -> ffi::jkb_tensor_view {
    let mut v = ffi::jkb_tensor_view::default();
    v.name = name.as_ptr();
    v.quant = quant_code(w.quant());
    let shape = w.shape();
    v.ndim = shape.len().min(4) as u32;
    for (i, s) in shape.iter().take(4).enumerate() {
        v.shape[i] = *s;
    }
    v.offset = w.offset();
    v.data = w.as_bytes().as_ptr().cast();
    v.byte_len = w.as_bytes().len();
    v.data_on_device = 0;
    v
}

/// The device upload of `w` as a [rows, cols] matrix (validated like the reference's
/// validate_matrix_view, quant.rs:1315-1358), uploaded on first use.
fn weight(w: &TensorView<'_>, rows: usize, cols: usize) -> Result<*const ffi::jkb_weight, K3Error> {
    let key = WeightKey { addr: w.as_bytes().as_ptr() as usize, len: w.as_bytes().len(),
                          quant: quant_code(w.quant()), rows, cols };
    let mut map = WEIGHTS.lock().unwrap();
    let map = map.get_or_insert_with(HashMap::new);
    if let Some(h) = map.get(&key) {
        return Ok(h.0);
    }
    let name = std::ffi::CString::new(w.name()).unwrap_or_default();
    let v = view_c(w, &name);
    let mut h = core::ptr::null_mut();
    check(unsafe { ffi::jkb_weight_upload(&v, rows, cols, core::ptr::null_mut(), &mut h) },
          "weight upload", w.quant())?;
    map.insert(key, Handle(h));
    Ok(h)
}

/// Drops every cached upload of `w`'s bytes (call before freeing or reusing them).
pub fn release_weight(w: &TensorView<'_>) {
    let addr = w.as_bytes().as_ptr() as usize;
    if let Some(map) = WEIGHTS.lock().unwrap().as_mut() {
        map.retain(|k, h| {
            let keep = k.addr != addr;
            if !keep {
                unsafe { ffi::jkb_weight_destroy(h.0) };
            }
            keep
        });
    }
}

// ------------------------------------------------------------------ activation quantizers

/// quant_q8.rs:395 quantize_row_q8_0.
pub fn quantize_row_q8_0(x: &[f32], out: &mut [BlockQ8_0]) -> Result<(), K3Error> {
    with_gpu(|g| {
        let dx = g.upload(0, x)?;
        let dout = g.buf(1, core::mem::size_of_val(out))?;
        check(unsafe { ffi::jkb_quantize_row_q8_0(dx.cast(), x.len(), dout.cast(), out.len(),
                                                  g.stream) },
              "quantize_row_q8_0", QuantType::F32)?;
        g.download(out, dout)
    })
}

/// quant_q8.rs:370 quantize_row_q8_0_f32 (the same quantizer).
pub fn quantize_row_q8_0_f32(x: &[f32], out: &mut [BlockQ8_0]) -> Result<(), K3Error> {
    quantize_row_q8_0(x, out)
}

/// quant_q8.rs:576 quantize_row_q8_k.
pub fn quantize_row_q8_k(x: &[f32], out: &mut [BlockQ8K]) -> Result<(), K3Error> {
    with_gpu(|g| {
        let dx = g.upload(0, x)?;
        let dout = g.buf(1, core::mem::size_of_val(out))?;
        check(unsafe { ffi::jkb_quantize_row_q8_k(dx.cast(), x.len(), dout.cast(), out.len(),
                                                  g.stream) },
              "quantize_row_q8_k", QuantType::F32)?;
        g.download(out, dout)
    })
}

// ------------------------------------------------------------------------ decode GEMVs

macro_rules! gemv_q8 {
    ($(#[$doc:meta])* $name:ident, $c:ident, $blk:ty, $elems:expr, $quant:expr) => {
        $(#[$doc])*
        pub fn $name(out: &mut [f32], weights: &TensorView<'_>, x_blocks: &[$blk])
                     -> Result<(), K3Error> {
            let w = weight(weights, out.len(), x_blocks.len() * $elems)?;
            with_gpu(|g| {
                let dx = g.upload(0, x_blocks)?;
                let dout = g.buf(1, core::mem::size_of_val(out))?;
                check(unsafe { ffi::$c(dout.cast(), out.len(), w, dx.cast(), x_blocks.len(),
                                       g.stream) }, stringify!($name), $quant)?;
                g.download(out, dout)
            })
        }
    };
}

gemv_q8!(/// quant_q8.rs:1586
         gemv_q4_0_q8_0, jkb_gemv_q4_0_q8_0, BlockQ8_0, 32, QuantType::Q4_0);
gemv_q8!(/// quant_q8.rs:1612 (the 4-row driver of the same result)
         gemv_q4_0_q8_0_4x, jkb_gemv_q4_0_q8_0_4x, BlockQ8_0, 32, QuantType::Q4_0);
gemv_q8!(/// quant_q8.rs:1670
         gemv_q8_0_q8_0, jkb_gemv_q8_0_q8_0, BlockQ8_0, 32, QuantType::Q8_0);
gemv_q8!(/// quant_q8.rs:1628
         gemv_q5_0_q8_0, jkb_gemv_q5_0_q8_0, BlockQ8_0, 32, QuantType::Q5_0);
gemv_q8!(/// quant_q8.rs:3101
         gemv_q4_k_q8_k, jkb_gemv_q4_k_q8_k, BlockQ8K, 256, QuantType::Q4_K_M);
gemv_q8!(/// quant_q8.rs:3160
         gemv_q5_k_q8_k, jkb_gemv_q5_k_q8_k, BlockQ8K, 256, QuantType::Q5_K);
gemv_q8!(/// quant_q8.rs:3189
         gemv_q6_k_q8_k, jkb_gemv_q6_k_q8_k, BlockQ8K, 256, QuantType::Q6_K);
gemv_q8!(/// quant_q8.rs:3221
         gemv_tq1_0_q8_k, jkb_gemv_tq1_0_q8_k, BlockQ8K, 256, QuantType::TQ1_0);
gemv_q8!(/// quant_q8.rs:3250
         gemv_tq2_0_q8_k, jkb_gemv_tq2_0_q8_k, BlockQ8K, 256, QuantType::TQ2_0);

macro_rules! vec_dot_q8 {
    ($(#[$doc:meta])* $name:ident, $c:ident, $blk:ty, $quant:expr) => {
        $(#[$doc])*
        pub fn $name(w_blocks: &[u8], x_blocks: &[$blk]) -> Result<f32, K3Error> {
            with_gpu(|g| {
                let dw = g.upload(0, w_blocks)?;
                let dx = g.upload(1, x_blocks)?;
                let dr = g.buf(2, 4)?;
                check(unsafe { ffi::$c(dw.cast(), w_blocks.len(), dx.cast(), x_blocks.len(),
                                       dr.cast(), g.stream) }, stringify!($name), $quant)?;
                let mut r = [0.0f32];
                g.download(&mut r, dr)?;
                Ok(r[0])
            })
        }
    };
}

vec_dot_q8!(/// quant_q8.rs:1463
            vec_dot_q4_0_q8_0, jkb_vec_dot_q4_0_q8_0, BlockQ8_0, QuantType::Q4_0);
vec_dot_q8!(/// quant_q8.rs:1493
            vec_dot_q8_0_q8_0, jkb_vec_dot_q8_0_q8_0, BlockQ8_0, QuantType::Q8_0);
vec_dot_q8!(/// quant_q8.rs:3019
            vec_dot_q4_k_q8_k, jkb_vec_dot_q4_k_q8_k, BlockQ8K, QuantType::Q4_K_M);
vec_dot_q8!(/// quant_q8.rs:3056
            vec_dot_q6_k_q8_k, jkb_vec_dot_q6_k_q8_k, BlockQ8K, QuantType::Q6_K);
vec_dot_q8!(/// quant_q8.rs:3086
            vec_dot_tq2_0_q8_k, jkb_vec_dot_tq2_0_q8_k, BlockQ8K, QuantType::TQ2_0);

// ----------------------------------------------------------------------------- BitLinear

/// ime.rs:882 bitlinear_i8_rvv (ime.rs:1005 bitlinear_i8_ime is bit-identical).
pub fn bitlinear_i8_rvv(out: &mut [f32], weights: &TensorView<'_>, act_i8: &[i8],
                        act_scale: f32) -> Result<(), K3Error> {
    let w = weight(weights, out.len(), act_i8.len())?;
    with_gpu(|g| {
        let da = g.upload(0, act_i8)?;
        let dout = g.buf(1, core::mem::size_of_val(out))?;
        check(unsafe { ffi::jkb_bitlinear_i8_rvv(dout.cast(), out.len(), w, da.cast(),
                                                 act_i8.len(), act_scale, g.stream) },
              "bitlinear_i8_rvv", weights.quant())?;
        g.download(out, dout)
    })
}

pub fn bitlinear_i8_ime(out: &mut [f32], weights: &TensorView<'_>, act_i8: &[i8],
                        act_scale: f32) -> Result<(), K3Error> {
    bitlinear_i8_rvv(out, weights, act_i8, act_scale)
}

// --------------------------------------------- QuantizedActQ8 / RepackedWeight (repack.rs)

/// repack.rs:461-724: the quantized batch lives on the device (capacity grows on demand).
pub struct QuantizedActQ8 {
    h: *mut ffi::jkb_act_q8,
    m_cap: usize,
    k: usize,
    m: usize,
}

impl QuantizedActQ8 {
    /// repack.rs:512
    pub const fn new() -> Self {
        QuantizedActQ8 { h: core::ptr::null_mut(), m_cap: 0, k: 0, m: 0 }
    }

    /// repack.rs:522
    pub fn quantize(act: &[f32], m: usize, k: usize) -> Result<Self, K3Error> {
        let mut q = Self::new();
        q.quantize_into(act, m, k)?;
        Ok(q)
    }

    /// repack.rs:531
    pub fn quantize_row(act: &[f32]) -> Result<Self, K3Error> {
        Self::quantize(act, 1, act.len())
    }

    /// repack.rs:542
    pub fn quantize_into(&mut self, act: &[f32], m: usize, k: usize) -> Result<(), K3Error> {
        if m != 0 && k != 0 && (self.h.is_null() || m > self.m_cap || k != self.k) {
            if !self.h.is_null() {
                unsafe { ffi::jkb_act_q8_destroy(self.h) };
                self.h = core::ptr::null_mut();
            }
            check(unsafe { ffi::jkb_act_q8_create(m, k, &mut self.h) }, "QuantizedActQ8",
                  QuantType::F32)?;
            self.m_cap = m;
            self.k = k;
        }
        with_gpu(|g| {
            let da = g.upload(0, act)?;
            check(unsafe { ffi::jkb_act_q8_quantize(self.h, da.cast(), act.len(), m, k,
                                                    g.stream) },
                  "QuantizedActQ8", QuantType::F32)?;
            cuda(unsafe { ffi::cudaStreamSynchronize(g.stream) }, "stream synchronize")
        })?;
        self.m = m;
        Ok(())
    }

    pub const fn m(&self) -> usize {
        self.m
    }

    pub const fn k(&self) -> usize {
        self.k
    }
}

impl Drop for QuantizedActQ8 {
    fn drop(&mut self) {
        if !self.h.is_null() {
            unsafe { ffi::jkb_act_q8_destroy(self.h) };
        }
    }
}

/// repack.rs:1124-1133: the i8-expanded weight, resident on the device.
pub struct RepackedWeight {
    h: *mut ffi::jkb_repacked_weight,
    rows: usize,
    cols: usize,
    quant: QuantType,
}

unsafe impl Send for RepackedWeight {}
unsafe impl Sync for RepackedWeight {}

impl RepackedWeight {
    /// repack.rs:2288
    pub fn from_tensor(weights: &TensorView<'_>, rows: usize, cols: usize)
                       -> Result<Self, K3Error> {
        let name = std::ffi::CString::new(weights.name()).unwrap_or_default();
        let v = view_c(weights, &name);
        let mut h = core::ptr::null_mut();
        check(unsafe { ffi::jkb_repacked_weight_from_tensor(&v, rows, cols,
                                                            core::ptr::null_mut(), &mut h) },
              "repack", weights.quant())?;
        Ok(RepackedWeight { h, rows, cols, quant: weights.quant() })
    }

    pub const fn rows(&self) -> usize {
        self.rows
    }

    pub const fn cols(&self) -> usize {
        self.cols
    }

    /// repack.rs:2661 gemm_rows (gemm, gemv, gemv_rows are the same call over full ranges or
    /// m == 1): out [m][row_range.len()] on the host.
    pub fn gemm_rows(&self, out: &mut [f32], act: &QuantizedActQ8, row_range: Range<usize>)
                     -> Result<(), K3Error> {
        with_gpu(|g| {
            let dout = g.buf(1, core::mem::size_of_val(out))?;
            check(unsafe { ffi::jkb_gemm_repacked_rows(dout.cast(), out.len(), self.h, act.h,
                                                       row_range.start, row_range.end,
                                                       g.stream) },
                  "gemm_repacked", self.quant)?;
            g.download(out, dout)
        })
    }

    /// repack.rs:2652
    pub fn gemm(&self, out: &mut [f32], act: &QuantizedActQ8) -> Result<(), K3Error> {
        self.gemm_rows(out, act, 0..self.rows)
    }

    /// repack.rs:2605 (act.m() must be 1)
    pub fn gemv(&self, out: &mut [f32], act: &QuantizedActQ8) -> Result<(), K3Error> {
        self.gemv_rows(out, act, 0..self.rows)
    }

    /// repack.rs:2614
    pub fn gemv_rows(&self, out: &mut [f32], act: &QuantizedActQ8, row_range: Range<usize>)
                     -> Result<(), K3Error> {
        with_gpu(|g| {
            let dout = g.buf(1, core::mem::size_of_val(out))?;
            check(unsafe { ffi::jkb_gemv_repacked_rows(dout.cast(), out.len(), self.h, act.h,
                                                       row_range.start, row_range.end,
                                                       g.stream) },
                  "gemv_repacked", self.quant)?;
            g.download(out, dout)
        })
    }
}

impl Drop for RepackedWeight {
    fn drop(&mut self) {
        unsafe { ffi::jkb_repacked_weight_destroy(self.h) };
    }
}

/// repack.rs:4073
pub fn gemm_repacked(out: &mut [f32], weights: &RepackedWeight, act: &QuantizedActQ8)
                     -> Result<(), K3Error> {
    weights.gemm(out, act)
}

/// repack.rs:4087
pub fn gemm_repacked_rows(out: &mut [f32], weights: &RepackedWeight, act: &QuantizedActQ8,
                          row_range: Range<usize>) -> Result<(), K3Error> {
    weights.gemm_rows(out, act, row_range)
}

/// repack.rs:3999
pub fn gemv_repacked(out: &mut [f32], weights: &RepackedWeight, act: &QuantizedActQ8)
                     -> Result<(), K3Error> {
    weights.gemv(out, act)
}

/// repack.rs:4014
pub fn gemv_repacked_rows(out: &mut [f32], weights: &RepackedWeight, act: &QuantizedActQ8,
                          row_range: Range<usize>) -> Result<(), K3Error> {
    weights.gemv_rows(out, act, row_range)
}

/// repack.rs:4143 (the quantized batch is a temporary QuantizedActQ8, as in the reference)
pub fn gemm_repacked_f32_rows(out: &mut [f32], weights: &RepackedWeight, input: &[f32],
                              m: usize, row_range: Range<usize>) -> Result<(), K3Error> {
    if m == 0 || weights.cols == 0 || input.len() != m.saturating_mul(weights.cols) {
        return Err(K3Error::TensorBoundsError {
            tensor_name: "gemm_repacked_f32".to_owned(),
            offset: 0,
            byte_len: core::mem::size_of_val(input),
            buffer_len: m.saturating_mul(weights.cols) * 4,
            reason: format!("input length {} != m ({m}) * cols ({})", input.len(), weights.cols),
        });
    }
    let act = QuantizedActQ8::quantize(input, m, weights.cols)?;
    gemm_repacked_rows(out, weights, &act, row_range)
}

/// repack.rs:4129
pub fn gemm_repacked_f32(out: &mut [f32], weights: &RepackedWeight, input: &[f32], m: usize)
                         -> Result<(), K3Error> {
    gemm_repacked_f32_rows(out, weights, input, m, 0..weights.rows)
}

/// repack.rs:4101
pub fn gemv_repacked_f32(out: &mut [f32], weights: &RepackedWeight, input: &[f32])
                         -> Result<(), K3Error> {
    gemv_repacked_f32_rows(out, weights, input, 0..weights.rows)
}

/// repack.rs:4114
pub fn gemv_repacked_f32_rows(out: &mut [f32], weights: &RepackedWeight, input: &[f32],
                              row_range: Range<usize>) -> Result<(), K3Error> {
    let act = QuantizedActQ8::quantize_row(input)?;
    gemv_repacked_rows(out, weights, &act, row_range)
}
