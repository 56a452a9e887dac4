"""Python mirror of the jero-kernels-rvv public API over the jkb200 C ABI.

Names, argument meaning and error behaviour follow the Rust crate (file:line in each
docstring). Device arguments are torch CUDA tensors; block activations are uint8 tensors
holding packed BlockQ8_0 (36 B) / BlockQ8K (292 B) structs. Errors raise K3Error subclasses
carrying the TensorBoundsError fields; nothing is launched when validation fails.
"""
from __future__ import annotations

import ctypes as C
import enum

import numpy as np
import torch

from . import _lib

__all__ = [
    "QuantType", "BLOCK", "BLOCK_Q8_0_BYTES", "BLOCK_Q8_K_BYTES", "K3Error", "TensorBoundsError",
    "CapabilityMismatch", "CudaError", "InvalidHandle", "TensorView", "Weight", "RepackedWeight",
    "QuantizedActQ8", "abi_version", "quantize_row_q8_0", "quantize_row_q8_0_f32",
    "quantize_row_q8_k", "quantize_rows_q8_0", "quantize_rows_q8_k", "subln_quantize_absmax_i8",
    "subln_quantize_absmax_i8_rows", "vec_dot_q4_0_q8_0", "vec_dot_q8_0_q8_0",
    "vec_dot_q4_k_q8_k", "vec_dot_q6_k_q8_k", "vec_dot_tq1_0_q8_k", "vec_dot_tq2_0_q8_k",
    "gemv_q4_0_q8_0", "gemv_q4_0_q8_0_4x", "gemv_q8_0_q8_0", "gemv_q8_0_q8_0_4x",
    "gemv_q4_k_q8_k", "gemv_q6_k_q8_k", "gemv_tq1_0_q8_k", "gemv_tq2_0_q8_k", "gemv_rows",
    "gemv_block_dots", "vec_dot_q4_k_m", "vec_dot_q8_0", "vec_dot_q6_k", "vec_dot_q4_0",
    "vec_dot_i2_s", "vec_dot_q4_k_m_rvv", "vec_dot_q6_k_rvv", "vec_dot_q8_0_rvv",
    "vec_dot_q4_0_rvv", "vec_dot_grouped_rvv", "bitlinear_i8", "bitlinear_i8_rvv", "bitlinear_i8_ime",
    "bitlinear_i8_batch", "gemm_repacked", "gemm_repacked_rows", "gemv_repacked",
    "gemv_repacked_rows", "gemm_repacked_f32", "gemm_repacked_f32_noalloc",
    "empty_q8_0_blocks", "empty_q8_k_blocks", "device_status", "gemm_set_exact", "gemm_get_exact",
    "gemm_exact", "PeerGroup", "gemv_batch",
    "device_view", "PackedNibbleMatrix", "gemm_q4_0_ime", "gemm_q4_k_ime",
    "repack_nibble_into_tile_range", "vec_dot_q5_0_q8_0_blocks", "vec_dot_q5_k_q8_k",
    "gemv_q5_0_q8_0", "gemv_q5_0_q8_0_4x", "gemv_q5_k_q8_k", "vec_dot_q5_0", "vec_dot_q5_k",
    "vec_dot_q5_0_rvv", "vec_dot_q5_k_rvv", "relu_squared_gate_f32",
    "relu_squared_subln_quantize_i8_rows", "BitNetFFN", "bitlinear_i8_gemm",
    "quantize_row_f32_to_q8_32", "ScratchWorkspace", "ScratchScope",
    "quantize_row_q8_0_in_scratch", "quantize_row_q8_0_in_scope", "quantize_row_q8_k_in_scratch",
    "quantize_row_q8_k_in_scope", "QuantizedActQ8View", "gemv_repacked_view",
    "gemv_repacked_view_rows", "gemv_repacked_f32", "gemv_repacked_f32_rows",
    "gemm_repacked_f32_rows", "BlockScaledTileLayout", "block_scaled_layout",
    "repack_into_tile_range", "repack_q4_k_m_parallel_slices",
]


class QuantType(enum.IntEnum):
    """jero_core::QuantType codes used at the boundary (GGML type ids)."""
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q2_K = 10
    Q3_K = 11
    Q4_K_M = 12
    Q5_K = 13
    Q6_K = 14
    IQ4_NL = 20
    BF16 = 30
    TQ1_0 = 34
    TQ2_0 = 35
    I2_S = 36


# (block elements, block bytes) -- quant.rs:20-91, ime.rs:28-37, lib.rs:129-132
BLOCK = {
    QuantType.Q4_0: (32, 18), QuantType.Q8_0: (32, 34), QuantType.Q4_K_M: (256, 144),
    QuantType.Q6_K: (256, 210), QuantType.TQ1_0: (256, 54), QuantType.TQ2_0: (256, 66),
    QuantType.I2_S: (128, 32), QuantType.Q4_1: (32, 20), QuantType.IQ4_NL: (32, 18),
    QuantType.Q5_0: (32, 22), QuantType.Q5_K: (256, 176), QuantType.Q5_1: (32, 24),
    QuantType.Q2_K: (256, 84), QuantType.Q3_K: (256, 110),
}
BLOCK_Q8_0_BYTES = 36
BLOCK_Q8_K_BYTES = 292


class K3Error(Exception):
    """Mirror of jero_core::K3Error carrying the TensorBoundsError fields."""

    def __init__(self, status, tensor_name, offset, byte_len, buffer_len, reason):
        self.status = status
        self.tensor_name = tensor_name
        self.offset = offset
        self.byte_len = byte_len
        self.buffer_len = buffer_len
        self.reason = reason
        super().__init__(f"{type(self).__name__}{{tensor_name: {tensor_name!r}, offset: {offset}, "
                         f"byte_len: {byte_len}, buffer_len: {buffer_len}, reason: {reason!r}}}")


class TensorBoundsError(K3Error):
    pass


class CapabilityMismatch(K3Error):
    pass


class CudaError(K3Error):
    pass


class InvalidHandle(K3Error):
    pass


_STATUS = {1: TensorBoundsError, 2: CapabilityMismatch, 3: CudaError, 4: K3Error, 5: K3Error,
           6: InvalidHandle}


def _check(rc: int):
    if rc == 0:
        return
    info = _lib.jkb_error_info()
    L = _lib.load()
    L.jkb_last_error_info(C.byref(info))
    cls = _STATUS.get(rc, K3Error)
    raise cls(rc, info.tensor_name.decode(errors="replace"), info.offset, info.byte_len,
              info.buffer_len, info.reason.decode(errors="replace"))


def _L():
    return _lib.load()


def abi_version() -> int:
    return int(_L().jkb_abi_version())


def device_status(stream=None) -> int:
    """Synchronizes the stream and returns (and clears) the device error word of the
    tensor-core GEMM; raises K3Error (JKB_E_TIMEOUT) when a bounded wait in it expired."""
    v = C.c_int32(0)
    _check(_L().jkb_device_status(C.byref(v), _stream(stream)))
    return int(v.value)


def gemm_set_exact(exact: bool) -> None:
    """Selects the tensor-core GEMM epilogue: False (default) fused multiply-add per scale group,
    within the reference's 1e-5 relative tolerance; True the reference's separately rounded
    product and sum, bit-identical outputs (accumulate_scaled_tile_scalar, repack.rs:3045)."""
    _check(_L().jkb_gemm_set_exact(1 if exact else 0))


def gemm_get_exact() -> bool:
    return bool(_L().jkb_gemm_get_exact())


class gemm_exact:
    """Context manager: the bit-exact GEMM epilogue inside the block, the previous one after."""

    def __init__(self, exact: bool = True):
        self.exact = exact

    def __enter__(self):
        self.prev = gemm_get_exact()
        gemm_set_exact(self.exact)
        return self

    def __exit__(self, *exc):
        gemm_set_exact(self.prev)
        return False


def _dptr(t):
    """Device pointer of a CUDA tensor (must be contiguous)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("expected a CUDA torch.Tensor")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _nblocks(t, block_bytes):
    n = t.numel() * t.element_size()
    if n % block_bytes:
        raise ValueError(f"block buffer of {n} bytes is not a multiple of {block_bytes}")
    return n // block_bytes


class _CudaArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2,
                                         "strides": None}


def device_view(ptr: int, shape, dtype: str) -> torch.Tensor:
    """Zero-copy torch view of library-owned device memory (handles' buffers)."""
    return torch.as_tensor(_CudaArray(ptr, shape, np.dtype(dtype).str), device="cuda")


def empty_q8_0_blocks(n: int, device="cuda") -> torch.Tensor:
    return torch.empty(n * BLOCK_Q8_0_BYTES, dtype=torch.uint8, device=device)


def empty_q8_k_blocks(n: int, device="cuda") -> torch.Tensor:
    return torch.empty(n * BLOCK_Q8_K_BYTES, dtype=torch.uint8, device=device)


# ------------------------------------------------------------------------------- TensorView

class TensorView:
    """jero_core::TensorView: name, quant, shape and the raw GGUF bytes (host or device)."""

    def __init__(self, name: str, quant, shape, data, offset: int = 0):
        self.name = name
        self.quant = int(quant)
        self.shape = tuple(int(s) for s in shape)
        self.offset = int(offset)
        if isinstance(data, torch.Tensor):
            self._keep = data.contiguous()
            self.on_device = self._keep.is_cuda
            self.ptr = self._keep.data_ptr()
            self.byte_len = self._keep.numel() * self._keep.element_size()
        else:
            self._keep = np.ascontiguousarray(data).view(np.uint8)
            self.on_device = False
            self.ptr = self._keep.ctypes.data
            self.byte_len = self._keep.nbytes
        self._name_b = name.encode()

    def _c(self):
        v = _lib.jkb_tensor_view()
        v.name = self._name_b
        v.quant = self.quant
        v.ndim = len(self.shape)
        for i, s in enumerate(self.shape[:4]):
            v.shape[i] = s
        v.offset = self.offset
        v.data = self.ptr
        v.byte_len = self.byte_len
        v.data_on_device = 1 if self.on_device else 0
        return v


class Weight:
    """Device-resident GEMV/BitLinear weight (validate + upload + relayout at load time).

    ``Weight(view, rows, cols)`` follows RepackedWeight::from_tensor (repack.rs:2288);
    ``Weight(view)`` infers the orientation like RepackedWeight::repack (repack.rs:2255).
    """

    def __init__(self, view: TensorView, rows=None, cols=None, stream=None):
        h = C.c_void_p()
        v = view._c()
        if rows is None:
            _check(_L().jkb_weight_upload_infer(C.byref(v), _stream(stream), C.byref(h)))
        else:
            _check(_L().jkb_weight_upload(C.byref(v), rows, cols, _stream(stream), C.byref(h)))
        self._h = h.value
        r, c, q = C.c_size_t(), C.c_size_t(), C.c_int32()
        db, gb = C.c_size_t(), C.c_size_t()
        _check(_L().jkb_weight_info(self._h, C.byref(r), C.byref(c), C.byref(q), C.byref(db),
                                    C.byref(gb)))
        self.rows, self.cols, self.quant = r.value, c.value, QuantType(q.value)
        self.device_bytes, self.gguf_bytes = db.value, gb.value
        self.name = view.name

    @property
    def handle(self):
        if self._h is None:
            raise InvalidHandle(6, self.name, 0, 0, 0, "weight destroyed")
        return self._h

    def destroy(self):
        if getattr(self, "_h", None):
            _L().jkb_weight_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class QuantizedActQ8:
    """Device QuantizedActQ8 (repack.rs:461-724) with a fixed capacity allocated up front."""

    def __init__(self, m_capacity: int, k: int):
        h = C.c_void_p()
        _check(_L().jkb_act_q8_create(m_capacity, k, C.byref(h)))
        self._h = h.value
        self.m_capacity, self.k = m_capacity, k
        self.k_padded = (k + 31) // 32 * 32

    @classmethod
    def quantize(cls, act: torch.Tensor, m: int, k: int, stream=None) -> "QuantizedActQ8":
        """repack.rs:522 QuantizedActQ8::quantize."""
        q = cls(max(m, 1), max(k, 1))
        q.quantize_into(act, m, k, stream)
        return q

    def quantize_into(self, act: torch.Tensor, m: int, k: int, stream=None):
        """repack.rs:542 QuantizedActQ8::quantize_into."""
        _check(_L().jkb_act_q8_quantize(self._h, _dptr(act), act.numel(), m, k, _stream(stream)))

    def buffers(self):
        """Zero-copy device views: q, x_scales, x_sums, x_sums_16, super_scales (row-major)."""
        m, k, kp = C.c_size_t(), C.c_size_t(), C.c_size_t()
        ptrs = [C.c_void_p() for _ in range(5)]
        _check(_L().jkb_act_q8_buffers(self._h, C.byref(m), C.byref(k), C.byref(kp),
                                       *[C.byref(p) for p in ptrs]))
        m, k, kp = m.value, k.value, kp.value
        return (device_view(ptrs[0].value, (m, kp), "i1"),
                device_view(ptrs[1].value, (m, kp // 32), "<f4"),
                device_view(ptrs[2].value, (m, kp // 32), "<f4"),
                device_view(ptrs[3].value, (m, kp // 16), "<f4"),
                device_view(ptrs[4].value, (m, (k + 255) // 256), "<f4"))

    def as_view(self) -> "QuantizedActQ8View":
        """repack.rs:708 QuantizedActQ8::as_view: the current batch as a borrowed view."""
        v = _lib.jkb_act_q8_view()
        _check(_L().jkb_act_q8_as_view(self._h, C.byref(v)))
        return QuantizedActQ8View(v, owner=self)

    def destroy(self):
        if getattr(self, "_h", None):
            _L().jkb_act_q8_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class RepackedWeight:
    """RepackedWeight (repack.rs:1124-1133): i8-expanded block-scaled weight for the GEMM."""

    def __init__(self, handle, name):
        self._h = handle
        self.name = name
        r, c, q, g = C.c_size_t(), C.c_size_t(), C.c_int32(), C.c_size_t()
        _check(_L().jkb_repacked_weight_buffers(self._h, C.byref(r), C.byref(c), C.byref(q),
                                                C.byref(g), None, None, None))
        self.rows, self.cols, self.quant, self.scale_groups = r.value, c.value, QuantType(
            q.value), g.value

    def dequantize_row(self, row: int, out: torch.Tensor = None, stream=None) -> torch.Tensor:
        """repack.rs:2529 RepackedWeight::dequantize_row (scale * q - min per group)."""
        if out is None:
            out = torch.empty(self.cols, dtype=torch.float32, device="cuda")
        _check(_L().jkb_repacked_weight_dequantize_row(self._h, row, _dptr(out), out.numel(),
                                                       _stream(stream)))
        return out

    @classmethod
    def from_tensor(cls, view: TensorView, rows: int, cols: int, stream=None):
        """repack.rs:2288 RepackedWeight::from_tensor."""
        h = C.c_void_p()
        v = view._c()
        _check(_L().jkb_repacked_weight_from_tensor(C.byref(v), rows, cols, _stream(stream),
                                                    C.byref(h)))
        return cls(h.value, view.name)

    @classmethod
    def repack(cls, view: TensorView, stream=None):
        """repack.rs:2255 RepackedWeight::repack."""
        h = C.c_void_p()
        v = view._c()
        _check(_L().jkb_repacked_weight_repack(C.byref(v), _stream(stream), C.byref(h)))
        return cls(h.value, view.name)

    def buffers(self):
        r, c, q, g = C.c_size_t(), C.c_size_t(), C.c_int32(), C.c_size_t()
        pq, ps, pm = C.c_void_p(), C.c_void_p(), C.c_void_p()
        _check(_L().jkb_repacked_weight_buffers(self._h, C.byref(r), C.byref(c), C.byref(q),
                                                C.byref(g), C.byref(pq), C.byref(ps),
                                                C.byref(pm)))
        kp = (c.value + 31) // 32 * 32
        mins = device_view(pm.value, (r.value, g.value), "<f4") if pm.value else None
        return (device_view(pq.value, (r.value, kp), "i1"),
                device_view(ps.value, (r.value, g.value), "<f4"), mins)

    def gemv(self, out, act, stream=None):
        gemv_repacked(out, self, act, stream)

    def gemv_rows(self, out, act, row_range, stream=None):
        gemv_repacked_rows(out, self, act, row_range, stream)

    def gemm(self, out, act, stream=None):
        gemm_repacked(out, self, act, stream)

    def gemm_rows(self, out, act, row_range, stream=None):
        gemm_repacked_rows(out, self, act, row_range, stream)

    def gemv_view(self, out, act: "QuantizedActQ8View", stream=None):
        """repack.rs:2628 RepackedWeight::gemv_view."""
        gemv_repacked_view(out, self, act, stream)

    def gemv_view_rows(self, out, act: "QuantizedActQ8View", row_range, stream=None):
        """repack.rs:2638 RepackedWeight::gemv_view_rows."""
        gemv_repacked_view_rows(out, self, act, row_range, stream)

    @classmethod
    def block_scaled_layout(cls, view: TensorView, rows: int, cols: int):
        """repack.rs:2372 RepackedWeight::block_scaled_layout."""
        return block_scaled_layout(view, rows, cols)

    @classmethod
    def from_tile_buffers(cls, layout: "BlockScaledTileLayout", tiles, scales, mins=None,
                          stream=None):
        """repack.rs:2386 RepackedWeight::from_tile_buffers: host numpy buffers in the
        reference tile layout (tiles: total_tiles x 128 bytes, scales / mins: f32)."""
        t = np.ascontiguousarray(tiles).view(np.uint8).reshape(-1)
        s = np.ascontiguousarray(scales, np.float32).reshape(-1)
        mn = None if mins is None else np.ascontiguousarray(mins, np.float32).reshape(-1)
        h = C.c_void_p()
        _check(_L().jkb_repacked_weight_from_tile_buffers(
            C.byref(layout._c), t.ctypes.data, t.size // 128, s.ctypes.data, s.size,
            None if mn is None else mn.ctypes.data, 0 if mn is None else mn.size,
            _stream(stream), C.byref(h)))
        return cls(h.value, "from_tile_buffers")

    def destroy(self):
        if getattr(self, "_h", None):
            _L().jkb_repacked_weight_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class PackedNibbleMatrix:
    """PackedNibbleMatrix (repack.rs:4188-5545): Q4_0 / Q4_1 / IQ4_NL / Q4_K_M weights kept
    4-bit on the device (exactly the GGUF bytes) with a GEMM that expands the codes on the fly."""

    def __init__(self, handle, name=""):
        self._h = handle
        self.name = name
        r, c, q, nt, kb = (C.c_size_t(), C.c_size_t(), C.c_int32(), C.c_size_t(),
                           C.c_size_t())
        pb, rb = C.c_size_t(), C.c_size_t()
        _check(_L().jkb_packed_nibble_matrix_info(self._h, C.byref(r), C.byref(c), C.byref(q),
                                                  C.byref(nt), C.byref(kb), C.byref(pb),
                                                  C.byref(rb)))
        self.rows, self.cols, self.quant = r.value, c.value, QuantType(q.value)
        self.n_tiles, self.k_blocks32 = nt.value, kb.value
        self._packed, self._raw = pb.value, rb.value

    @classmethod
    def from_tensor(cls, view: TensorView, rows: int, cols: int, stream=None):
        """repack.rs:4788 PackedNibbleMatrix::from_tensor."""
        h = C.c_void_p()
        v = view._c()
        _check(_L().jkb_packed_nibble_matrix_from_tensor(C.byref(v), rows, cols,
                                                         _stream(stream), C.byref(h)))
        return cls(h.value, view.name)

    @classmethod
    def repack(cls, view: TensorView, stream=None):
        """repack.rs:4654 PackedNibbleMatrix::repack."""
        h = C.c_void_p()
        v = view._c()
        _check(_L().jkb_packed_nibble_matrix_repack(C.byref(v), _stream(stream), C.byref(h)))
        return cls(h.value, view.name)

    @classmethod
    def from_scale_f16_buffers(cls, quant, rows: int, cols: int, nibble_tiles, scales_f16,
                               stream=None):
        """repack.rs:4686: host numpy buffers in the reference's tile layout."""
        t = np.ascontiguousarray(nibble_tiles, np.uint8)
        sc = np.ascontiguousarray(scales_f16, np.uint16)
        h = C.c_void_p()
        _check(_L().jkb_packed_nibble_matrix_from_scale_f16_buffers(
            int(quant), rows, cols, t.ctypes.data, t.size // 128, sc.ctypes.data, sc.size,
            _stream(stream), C.byref(h)))
        return cls(h.value)

    @classmethod
    def from_q4_k_buffers(cls, rows: int, cols: int, nibble_tiles, headers, stream=None):
        """repack.rs:4743: host numpy buffers in the reference's tile layout."""
        t = np.ascontiguousarray(nibble_tiles, np.uint8)
        hd = np.ascontiguousarray(headers, np.uint8)
        h = C.c_void_p()
        _check(_L().jkb_packed_nibble_matrix_from_q4_k_buffers(
            rows, cols, t.ctypes.data, t.size // 128, hd.ctypes.data, hd.size // 16,
            _stream(stream), C.byref(h)))
        return cls(h.value)

    def packed_bytes(self) -> int:
        """repack.rs:4914: device bytes of the codes and scales."""
        return self._packed

    def resident_bytes(self) -> int:
        return self._packed

    def raw_tensor_bytes(self) -> int:
        return self._raw

    def buffers(self):
        """Zero-copy device views: codes [rows][cols / 2] and scale words [rows][blocks * bytes]."""
        pq, pm = C.c_void_p(), C.c_void_p()
        _check(_L().jkb_packed_nibble_matrix_buffers(self.handle, C.byref(pq), C.byref(pm)))
        mb = (self._packed - self.rows * (self.cols // 2)) // max(self.rows, 1)
        return (device_view(pq.value, (self.rows, self.cols // 2), "u1"),
                device_view(pm.value, (self.rows, mb), "u1"))

    @property
    def handle(self):
        if self._h is None:
            raise InvalidHandle(6, self.name, 0, 0, 0, "PackedNibbleMatrix destroyed")
        return self._h

    def gemm(self, out, act: QuantizedActQ8, stream=None):
        """repack.rs:4945 gemm: out [act.m][rows]."""
        _check(_L().jkb_packed_nibble_matrix_gemm(_dptr(out), out.numel(), self.handle, act._h,
                                                  _stream(stream)))

    def gemm_rows(self, out, act: QuantizedActQ8, row_range, stream=None):
        """repack.rs:4954 gemm_rows: out [act.m][len(row_range)]."""
        _check(_L().jkb_packed_nibble_matrix_gemm_rows(_dptr(out), out.numel(), self.handle,
                                                       act._h, row_range.start, row_range.stop,
                                                       _stream(stream)))

    def gemv(self, out, act: QuantizedActQ8, stream=None):
        """repack.rs:4968 gemv (act.m == 1)."""
        _check(_L().jkb_packed_nibble_matrix_gemv(_dptr(out), out.numel(), self.handle, act._h,
                                                  _stream(stream)))

    def dequantize_row(self, row: int, out, stream=None):
        """repack.rs:5001 dequantize_row: out f32 [cols] (device)."""
        _check(_L().jkb_packed_nibble_matrix_dequantize_row(self.handle, row, _dptr(out),
                                                            out.numel(), _stream(stream)))

    def destroy(self):
        if getattr(self, "_h", None):
            _L().jkb_packed_nibble_matrix_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def gemm_q4_0_ime(out, weights: PackedNibbleMatrix, act: QuantizedActQ8, stream=None):
    """repack.rs:5140 gemm_q4_0_ime (CapabilityMismatch unless Q4_0)."""
    _check(_L().jkb_gemm_q4_0_ime(_dptr(out), out.numel(), weights.handle, act._h,
                                  _stream(stream)))


def gemm_q4_k_ime(out, weights: PackedNibbleMatrix, act: QuantizedActQ8, stream=None):
    """repack.rs:5162 gemm_q4_k_ime (CapabilityMismatch unless Q4_K_M)."""
    _check(_L().jkb_gemm_q4_k_ime(_dptr(out), out.numel(), weights.handle, act._h,
                                  _stream(stream)))


def repack_nibble_into_tile_range(view: TensorView, rows: int, cols: int, tile_range):
    """repack.rs:4414 repack_nibble_into_tile_range on host bytes: returns (tiles u8 [n*kb*128],
    scales_f16 or None, mins_f16 or None, headers u8 [n*(cols/256)*8*16] or None) for the tiles
    of tile_range, in the reference's layout."""
    n = tile_range.stop - tile_range.start
    kb = cols // 32
    tiles = np.zeros(max(n, 0) * kb * 128, np.uint8)
    sc = mn = hd = None
    q = view.quant
    if q == QuantType.Q4_K_M:
        hd = np.zeros(max(n, 0) * (cols // 256) * 8 * 16, np.uint8)
    elif q in (QuantType.Q4_0, QuantType.IQ4_NL, QuantType.Q4_1):
        sc = np.zeros(max(n, 0) * kb * 8, np.uint16)
        if q == QuantType.Q4_1:
            mn = np.zeros(max(n, 0) * kb * 8, np.uint16)
    v = view._c()

    def ptr(a):
        return None if a is None else a.ctypes.data

    _check(_L().jkb_repack_nibble_into_tile_range(
        C.byref(v), rows, cols, tile_range.start, tile_range.stop, ptr(tiles), tiles.size // 128,
        ptr(sc), 0 if sc is None else sc.size, ptr(mn), 0 if mn is None else mn.size, ptr(hd),
        0 if hd is None else hd.size // 16))
    return tiles, sc, mn, hd


# ------------------------------------------------------------------------------- quantizers

def quantize_row_q8_0(x, out, stream=None):
    """quant_q8.rs:395 quantize_row_q8_0(x: &[f32], out: &mut [BlockQ8_0])."""
    _check(_L().jkb_quantize_row_q8_0(_dptr(x), x.numel(), _dptr(out),
                                      _nblocks(out, BLOCK_Q8_0_BYTES), _stream(stream)))


def quantize_row_q8_0_f32(x, out, stream=None):
    """quant_q8.rs:370 quantize_row_q8_0_f32."""
    _check(_L().jkb_quantize_row_q8_0_f32(_dptr(x), x.numel(), _dptr(out),
                                          _nblocks(out, BLOCK_Q8_0_BYTES), _stream(stream)))


def quantize_row_q8_k(x, out, stream=None):
    """quant_q8.rs:576 quantize_row_q8_k(x: &[f32], out: &mut [BlockQ8K])."""
    _check(_L().jkb_quantize_row_q8_k(_dptr(x), x.numel(), _dptr(out),
                                      _nblocks(out, BLOCK_Q8_K_BYTES), _stream(stream)))


def quantize_rows_q8_0(x, m, k, out, stream=None):
    _check(_L().jkb_quantize_rows_q8_0(_dptr(x), m, k, _dptr(out),
                                       _nblocks(out, BLOCK_Q8_0_BYTES), _stream(stream)))


def quantize_rows_q8_k(x, m, k, out, stream=None):
    _check(_L().jkb_quantize_rows_q8_k(_dptr(x), m, k, _dptr(out),
                                       _nblocks(out, BLOCK_Q8_K_BYTES), _stream(stream)))


def subln_quantize_absmax_i8(out_i8, x, norm_weight, eps, scale_out, stream=None):
    """lib.rs:1042 subln_quantize_absmax_i8 (the f32 scale lands in scale_out[0])."""
    _check(_L().jkb_subln_quantize_absmax_i8(_dptr(out_i8), out_i8.numel(), _dptr(x), x.numel(),
                                             _dptr(norm_weight), norm_weight.numel(), eps,
                                             _dptr(scale_out), _stream(stream)))


def subln_quantize_absmax_i8_rows(out_i8, x, norm_weight, m, length, eps, scales_out,
                                  stream=None):
    _check(_L().jkb_subln_quantize_absmax_i8_rows(_dptr(out_i8), _dptr(x), _dptr(norm_weight), m,
                                                  length, eps, _dptr(scales_out),
                                                  _stream(stream)))


def relu_squared_gate_f32(out, gate, up, stream=None):
    """lib.rs:1111 relu_squared_gate_f32: out = max(0, gate)^2 * up."""
    _check(_L().jkb_relu_squared_gate_f32(_dptr(out), out.numel(), _dptr(gate), gate.numel(),
                                          _dptr(up), up.numel(), _stream(stream)))


def relu_squared_subln_quantize_i8_rows(out_i8, relu_out, gate, up, norm_weight, m, length, eps,
                                        scales_out, stream=None):
    """relu_squared_gate_f32 then subln_quantize_absmax_i8 on each of m rows, one kernel."""
    _check(_L().jkb_relu_squared_subln_quantize_i8_rows(
        _dptr(out_i8), _dptr(relu_out), _dptr(gate), _dptr(up), _dptr(norm_weight), m, length,
        eps, _dptr(scales_out), _stream(stream)))


class BitNetFFN:
    """The BitNet b1.58 FFN chain (tests/empirical_challenge_m3_bitnet.rs:582-686) over device
    buffers: SubLN -> gate/up bitlinear_i8 -> relu_squared_gate_f32 -> SubLN -> down
    bitlinear_i8. Borrows the weights and the norm weights; owns the intermediates."""

    def __init__(self, w_gate: "Weight", w_up: "Weight", w_down: "Weight", norm1: torch.Tensor,
                 norm2: torch.Tensor, eps: float, m_capacity: int = 1, repacked=None):
        """repacked: None or RepackedWeights (gate, up, down) of the same tensors, for the
        tensor-core projections of batches of at least 32 tokens."""
        h = C.c_void_p()
        rg, ru, rd = (r._h for r in repacked) if repacked else (None, None, None)
        _check(_L().jkb_bitnet_ffn_create(w_gate.handle, w_up.handle, w_down.handle, rg, ru, rd,
                                          _dptr(norm1), norm1.numel(), _dptr(norm2),
                                          norm2.numel(), eps, m_capacity, C.byref(h)))
        self._h = h.value
        # keep the borrowed objects alive as long as the handle
        self._refs = (w_gate, w_up, w_down, norm1, norm2, repacked)
        self.hidden, self.inter = w_gate.cols, w_gate.rows
        self.m_capacity = m_capacity

    def forward(self, out: torch.Tensor, x: torch.Tensor, m: int = 1, stream=None):
        _check(_L().jkb_bitnet_ffn_forward(self._h, _dptr(out), out.numel(), _dptr(x), x.numel(),
                                           m, _stream(stream)))

    def buffers(self):
        """Device views of the intermediates: act1, scale1, gate, up, relu, act2, scale2."""
        ptrs = [C.c_void_p() for _ in range(7)]
        _check(_L().jkb_bitnet_ffn_buffers(self._h, *[C.byref(p) for p in ptrs]))
        M, H, I = self.m_capacity, self.hidden, self.inter
        shapes = [((M, H), "i1"), ((M,), "<f4"), ((M, I), "<f4"), ((M, I), "<f4"),
                  ((M, I), "<f4"), ((M, I), "i1"), ((M,), "<f4")]
        return tuple(device_view(p.value, sh, dt) for p, (sh, dt) in zip(ptrs, shapes))

    def destroy(self):
        if getattr(self, "_h", None):
            _L().jkb_bitnet_ffn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


# ------------------------------------------------------------------------------- block dots

def _vec_dot(fn, w_blocks, x_blocks, bb, result, stream):
    _check(getattr(_L(), fn)(_dptr(w_blocks), w_blocks.numel() * w_blocks.element_size(),
                             _dptr(x_blocks), _nblocks(x_blocks, bb), _dptr(result),
                             _stream(stream)))


def vec_dot_q4_0_q8_0(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:1463 (result: 1-element f32 device tensor)."""
    _vec_dot("jkb_vec_dot_q4_0_q8_0", w_blocks, x_blocks, BLOCK_Q8_0_BYTES, result, stream)


def vec_dot_q8_0_q8_0(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:1493."""
    _vec_dot("jkb_vec_dot_q8_0_q8_0", w_blocks, x_blocks, BLOCK_Q8_0_BYTES, result, stream)


def vec_dot_q4_k_q8_k(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:3019."""
    _vec_dot("jkb_vec_dot_q4_k_q8_k", w_blocks, x_blocks, BLOCK_Q8_K_BYTES, result, stream)


def vec_dot_q6_k_q8_k(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:3056."""
    _vec_dot("jkb_vec_dot_q6_k_q8_k", w_blocks, x_blocks, BLOCK_Q8_K_BYTES, result, stream)


def vec_dot_q5_0_q8_0_blocks(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:1478."""
    _vec_dot("jkb_vec_dot_q5_0_q8_0_blocks", w_blocks, x_blocks, BLOCK_Q8_0_BYTES, result, stream)


def vec_dot_q5_k_q8_k(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:3041."""
    _vec_dot("jkb_vec_dot_q5_k_q8_k", w_blocks, x_blocks, BLOCK_Q8_K_BYTES, result, stream)


def vec_dot_tq1_0_q8_k(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:3071."""
    _vec_dot("jkb_vec_dot_tq1_0_q8_k", w_blocks, x_blocks, BLOCK_Q8_K_BYTES, result, stream)


def vec_dot_tq2_0_q8_k(w_blocks, x_blocks, result, stream=None):
    """quant_q8.rs:3086."""
    _vec_dot("jkb_vec_dot_tq2_0_q8_k", w_blocks, x_blocks, BLOCK_Q8_K_BYTES, result, stream)


# ------------------------------------------------------------------------------- GEMV

def _gemv(fn, out, weights: Weight, x_blocks, bb, stream):
    _check(getattr(_L(), fn)(_dptr(out), out.numel(), weights.handle, _dptr(x_blocks),
                             _nblocks(x_blocks, bb), _stream(stream)))


def gemv_q4_0_q8_0(out, weights, x_blocks, stream=None):
    """quant_q8.rs:1586 gemv_q4_0_q8_0(output, &TensorView, &[BlockQ8_0])."""
    _gemv("jkb_gemv_q4_0_q8_0", out, weights, x_blocks, BLOCK_Q8_0_BYTES, stream)


def gemv_q4_0_q8_0_4x(out, weights, x_blocks, stream=None):
    """quant_q8.rs:1612 alias."""
    _gemv("jkb_gemv_q4_0_q8_0_4x", out, weights, x_blocks, BLOCK_Q8_0_BYTES, stream)


def gemv_q8_0_q8_0(out, weights, x_blocks, stream=None):
    """quant_q8.rs:1670."""
    _gemv("jkb_gemv_q8_0_q8_0", out, weights, x_blocks, BLOCK_Q8_0_BYTES, stream)


def gemv_q8_0_q8_0_4x(out, weights, x_blocks, stream=None):
    """quant_q8.rs:1696 alias."""
    _gemv("jkb_gemv_q8_0_q8_0_4x", out, weights, x_blocks, BLOCK_Q8_0_BYTES, stream)


def gemv_q4_k_q8_k(out, weights, x_blocks, stream=None):
    """quant_q8.rs:3101."""
    _gemv("jkb_gemv_q4_k_q8_k", out, weights, x_blocks, BLOCK_Q8_K_BYTES, stream)


def gemv_q6_k_q8_k(out, weights, x_blocks, stream=None):
    """quant_q8.rs:3189."""
    _gemv("jkb_gemv_q6_k_q8_k", out, weights, x_blocks, BLOCK_Q8_K_BYTES, stream)


def gemv_q5_0_q8_0(out, weights, x_blocks, stream=None):
    """quant_q8.rs:1628."""
    _gemv("jkb_gemv_q5_0_q8_0", out, weights, x_blocks, BLOCK_Q8_0_BYTES, stream)


def gemv_q5_0_q8_0_4x(out, weights, x_blocks, stream=None):
    """quant_q8.rs:1657."""
    _gemv("jkb_gemv_q5_0_q8_0_4x", out, weights, x_blocks, BLOCK_Q8_0_BYTES, stream)


def gemv_q5_k_q8_k(out, weights, x_blocks, stream=None):
    """quant_q8.rs:3160."""
    _gemv("jkb_gemv_q5_k_q8_k", out, weights, x_blocks, BLOCK_Q8_K_BYTES, stream)


def gemv_tq1_0_q8_k(out, weights, x_blocks, stream=None):
    """quant_q8.rs:3221."""
    _gemv("jkb_gemv_tq1_0_q8_k", out, weights, x_blocks, BLOCK_Q8_K_BYTES, stream)


def gemv_tq2_0_q8_k(out, weights, x_blocks, stream=None):
    """quant_q8.rs:3250."""
    _gemv("jkb_gemv_tq2_0_q8_k", out, weights, x_blocks, BLOCK_Q8_K_BYTES, stream)


def _act_block_bytes(quant):
    return (BLOCK_Q8_0_BYTES if quant in (QuantType.Q4_0, QuantType.Q8_0, QuantType.Q5_0)
            else BLOCK_Q8_K_BYTES)


def gemv_rows(out, weights: Weight, x_blocks, row_range, stream=None):
    """Row-sliced GEMV (the gemv_repacked_rows split, repack.rs:4014)."""
    r0, r1 = row_range.start, row_range.stop
    _check(_L().jkb_gemv_rows(_dptr(out), out.numel(), weights.handle, _dptr(x_blocks),
                              _nblocks(x_blocks, _act_block_bytes(weights.quant)), r0, r1,
                              _stream(stream)))


def gemv_batch(out, weights: Weight, x_blocks, m: int, stream=None):
    """M tokens of gemv_* in one launch (no reference counterpart): x_blocks holds m rows of
    Q8 blocks, out is [m][rows]; each token's output equals its single call's."""
    _check(_L().jkb_gemv_batch(_dptr(out), out.numel(), weights.handle, _dptr(x_blocks),
                               _nblocks(x_blocks, _act_block_bytes(weights.quant)), m,
                               _stream(stream)))


def gemv_block_dots(weights: Weight, x_blocks, stream=None):
    """Per-(row, block) integer sums and f32 block values of the GEMV kernels."""
    nb = weights.cols // BLOCK[weights.quant][0]
    sumi = torch.empty((weights.rows, nb), dtype=torch.int32, device="cuda")
    mins = torch.empty((weights.rows, nb), dtype=torch.int32, device="cuda")
    vals = torch.empty((weights.rows, nb), dtype=torch.float32, device="cuda")
    _check(_L().jkb_gemv_block_dots(weights.handle, _dptr(x_blocks),
                                    _nblocks(x_blocks, _act_block_bytes(weights.quant)),
                                    _dptr(sumi), _dptr(mins), _dptr(vals), _stream(stream)))
    return sumi, mins, vals


def _vk(fn, out, weights, x, stream):
    _check(getattr(_L(), fn)(_dptr(out), out.numel(), weights.handle, _dptr(x), x.numel(),
                             _stream(stream)))


def vec_dot_q4_k_m(out, weights, x, stream=None):
    """lib.rs:157 VectorKernel::vec_dot_q4_k_m (f32 activations)."""
    _vk("jkb_vec_dot_q4_k_m", out, weights, x, stream)


def vec_dot_q8_0(out, weights, x, stream=None):
    """quant.rs:1069."""
    _vk("jkb_vec_dot_q8_0", out, weights, x, stream)


def vec_dot_q6_k(out, weights, x, stream=None):
    """quant.rs:1089."""
    _vk("jkb_vec_dot_q6_k", out, weights, x, stream)


def vec_dot_q4_0(out, weights, x, stream=None):
    """quant.rs:1458."""
    _vk("jkb_vec_dot_q4_0", out, weights, x, stream)


def vec_dot_q5_0(out, weights, x, stream=None):
    """quant.rs:2036 vec_dot_q5_0 (host branch)."""
    _vk("jkb_vec_dot_q5_0", out, weights, x, stream)


def vec_dot_q5_k(out, weights, x, stream=None):
    """quant.rs:1238 vec_dot_q5_k / lib.rs:188 VectorKernel::vec_dot_q5_k (host branch)."""
    _vk("jkb_vec_dot_q5_k", out, weights, x, stream)


def vec_dot_q5_0_rvv(out, weights, x, stream=None):
    """vec_dot_q5_0's riscv64 branch (vec_dot_q5_0_4row_rvv): quantize + integer GEMV."""
    _vk("jkb_vec_dot_q5_0_rvv", out, weights, x, stream)


def vec_dot_q5_k_rvv(out, weights, x, stream=None):
    """quant.rs:1225 vec_dot_q5_k_rvv: quantize + integer GEMV."""
    _vk("jkb_vec_dot_q5_k_rvv", out, weights, x, stream)


def vec_dot_i2_s(out, weights, x, stream=None):
    """quant.rs:2199."""
    _vk("jkb_vec_dot_i2_s", out, weights, x, stream)


def vec_dot_q4_k_m_rvv(out, weights, x, stream=None):
    """lib.rs:1313: f32 input quantized to Q8_K, then the integer Q4_K_M x Q8_K GEMV."""
    _vk("jkb_vec_dot_q4_k_m_rvv", out, weights, x, stream)


def vec_dot_q6_k_rvv(out, weights, x, stream=None):
    """quant.rs:1056: f32 input quantized to Q8_K, then the integer Q6_K x Q8_K GEMV."""
    _vk("jkb_vec_dot_q6_k_rvv", out, weights, x, stream)


def vec_dot_q8_0_rvv(out, weights, x, stream=None):
    """quant.rs:999: f32 input quantized to Q8_0, then the integer Q8_0 x Q8_0 GEMV."""
    _vk("jkb_vec_dot_q8_0_rvv", out, weights, x, stream)


def vec_dot_q4_0_rvv(out, weights, x, stream=None):
    """quant.rs:1445: f32 input quantized to Q8_0, then the integer Q4_0 x Q8_0 GEMV."""
    _vk("jkb_vec_dot_q4_0_rvv", out, weights, x, stream)


def vec_dot_grouped_rvv(items, x, stream=None):
    """Several vec_dot_*_rvv products sharing the f32 input `x` in one launch (no reference
    counterpart). `items` is a sequence of (out, weights) pairs; every weight has the quant
    type of the first and x.numel() columns; each output equals its single call's."""
    arr = (_lib.jkb_vec_dot_item * max(1, len(items)))()
    for i, (out, w) in enumerate(items):
        arr[i].out = _dptr(out)
        arr[i].out_len = out.numel()
        arr[i].w = w.handle
    _check(_L().jkb_vec_dot_grouped_rvv(arr, len(items), _dptr(x), x.numel(), _stream(stream)))


class PeerGroup:
    """A rank's peer group (one process per GPU): a device buffer of `nbytes` with the same
    layout on every rank, whose chunks allgather() copies from each rank to all the others over
    NVLink in one kernel. Created collectively: every rank of the default process group (or
    `group`) calls PeerGroup(nbytes); the CUDA IPC handles travel over torch.distributed."""

    HANDLE_BYTES = 64

    def __init__(self, nbytes: int, world: int = None, rank: int = None, group=None):
        import torch.distributed as dist

        if world is None:
            world = dist.get_world_size(group) if dist.is_initialized() else 1
            rank = dist.get_rank(group) if dist.is_initialized() else 0
        h = C.c_void_p()
        _check(_L().jkb_peer_group_create(world, rank, nbytes, C.byref(h)))
        self.handle, self.world, self.rank = h, world, rank
        if world > 1:
            mine = (C.c_uint8 * self.HANDLE_BYTES)()
            _check(_L().jkb_peer_group_handle(h, mine))
            allh = [None] * world
            dist.all_gather_object(allh, bytes(mine), group=group)
            buf = (C.c_uint8 * (self.HANDLE_BYTES * world)).from_buffer_copy(b"".join(allh))
            _check(_L().jkb_peer_group_open(h, buf))
        ptr, n = C.c_void_p(), C.c_size_t()
        _check(_L().jkb_peer_group_buffer(h, C.byref(ptr), C.byref(n)))
        self.buffer = device_view(ptr.value, (n.value // 4,), "<f4")

    def allgather(self, chunks, stream=None):
        """Copy this rank's `chunks` ((byte offset, byte length) pairs of the buffer) to the same
        offsets on every peer and make the stream wait until every peer's chunks of the same call
        have arrived (bounded: on expiry bit 1 of device_status())."""
        self.allgather_arrays(self.chunk_arrays(chunks), stream)

    @staticmethod
    def chunk_arrays(chunks):
        """The ctypes arrays allgather_arrays() takes (built once for a fixed chunk list)."""
        n = len(chunks)
        offs = (C.c_size_t * max(1, n))(*[c[0] for c in chunks])
        lens = (C.c_size_t * max(1, n))(*[c[1] for c in chunks])
        return offs, lens, n

    def allgather_arrays(self, arrays, stream=None):
        offs, lens, n = arrays
        _check(_L().jkb_peer_group_allgather(self.handle, offs, lens, n, _stream(stream)))

    def wait(self, arrivals: int, stream=None):
        """Low level: make the stream wait for `arrivals` more peer signals (bounded)."""
        _check(_L().jkb_peer_group_wait(self.handle, arrivals, _stream(stream)))

    def set_push(self, enable: bool = True):
        """While enabled, the GEMV entry points store every output element that lands in this
        group's buffer into each peer's buffer too, from the kernel that computes it; signal()
        then completes the exchange (jkb_peer_group_set_push)."""
        _check(_L().jkb_peer_group_set_push(self.handle, 1 if enable else 0))

    def signal(self, stream=None):
        """Signal every peer that this rank's pushed outputs are complete and make the stream
        wait for every peer's signal of the same call (bounded: bit 1 of device_status())."""
        _check(_L().jkb_peer_group_signal(self.handle, _stream(stream)))

    def destroy(self):
        if getattr(self, "handle", None):
            _L().jkb_peer_group_destroy(self.handle)
            self.handle = None


# ------------------------------------------------------------------------------- BitLinear

def bitlinear_i8(out, weights, act_i8, act_scale: float, stream=None):
    """ime.rs:882 bitlinear_i8_rvv / :1005 bitlinear_i8_ime."""
    _check(_L().jkb_bitlinear_i8(_dptr(out), out.numel(), weights.handle, _dptr(act_i8),
                                 act_i8.numel(), float(act_scale), _stream(stream)))


bitlinear_i8_rvv = bitlinear_i8
bitlinear_i8_ime = bitlinear_i8


def bitlinear_i8_gemm(out, repacked, act_i8, act_scales, m, scratch, stream=None):
    """bitlinear_i8 for m tokens on the tensor cores (RepackedWeight of TQ1_0 / TQ2_0 / I2_S /
    Q8_0; scratch a QuantizedActQ8 of capacity >= m and k == cols)."""
    _check(_L().jkb_bitlinear_i8_gemm(_dptr(out), out.numel(), repacked._h, _dptr(act_i8),
                                      act_i8.numel(), _dptr(act_scales), m, scratch._h,
                                      _stream(stream)))


def bitlinear_i8_batch(out, weights, act_i8, act_scales, stream=None):
    _check(_L().jkb_bitlinear_i8_batch(_dptr(out), out.numel(), weights.handle, _dptr(act_i8),
                                       act_i8.numel(), _dptr(act_scales), act_scales.numel(),
                                       _stream(stream)))


# ------------------------------------------------------------------------------- GEMM

def gemm_repacked(out, weights: RepackedWeight, act: QuantizedActQ8, stream=None):
    """repack.rs:4073."""
    _check(_L().jkb_gemm_repacked(_dptr(out), out.numel(), weights._h, act._h, _stream(stream)))


def gemm_repacked_rows(out, weights, act, row_range, stream=None):
    """repack.rs:4087."""
    _check(_L().jkb_gemm_repacked_rows(_dptr(out), out.numel(), weights._h, act._h,
                                       row_range.start, row_range.stop, _stream(stream)))


def gemv_repacked(out, weights, act, stream=None):
    """repack.rs:3999."""
    _check(_L().jkb_gemv_repacked(_dptr(out), out.numel(), weights._h, act._h, _stream(stream)))


def gemv_repacked_rows(out, weights, act, row_range, stream=None):
    """repack.rs:4014."""
    _check(_L().jkb_gemv_repacked_rows(_dptr(out), out.numel(), weights._h, act._h,
                                       row_range.start, row_range.stop, _stream(stream)))


def gemm_repacked_f32(out, weights, x, m, scratch: QuantizedActQ8, stream=None):
    """repack.rs:4129 (the caller supplies the QuantizedActQ8 scratch handle)."""
    _check(_L().jkb_gemm_repacked_f32(_dptr(out), out.numel(), weights._h, _dptr(x), x.numel(),
                                      m, scratch._h, _stream(stream)))


def gemm_repacked_f32_noalloc(out, weights, x, m, stream=None):
    """gemm_repacked_f32 for callers that cannot allocate device memory (and so cannot create
    a QuantizedActQ8 handle). It uses a scratch array built into the library, limited to
    m * round_up(cols, 32) <= 2**21 elements. Calls that overlap on the GPU share that array
    and race, so serialize them. No counterpart in the reference."""
    _check(_L().jkb_gemm_repacked_f32_noalloc(_dptr(out), out.numel(), weights._h, _dptr(x),
                                              x.numel(), m, _stream(stream)))


# ------------------------------------------------------------------------------- row quantizer

def quantize_row_f32_to_q8_32(x, out_quants, out_scales, out_sums, stream=None):
    """repack.rs:441 quantize_row_f32_to_q8_32: device f32 x -> i8 quants (round_up(len, 32)),
    per-32 scales and sequential f32 sums (device tensors)."""
    _check(_L().jkb_quantize_row_f32_to_q8_32(_dptr(x), x.numel(), _dptr(out_quants),
                                              out_quants.numel(), _dptr(out_scales),
                                              out_scales.numel(), _dptr(out_sums),
                                              out_sums.numel(), _stream(stream)))


# ------------------------------------------------------------------------------- scratch arenas

class ScratchWorkspace:
    """jero_core::ScratchWorkspace on the device: a bump arena of `nbytes` (allocated here), or
    over a caller-owned CUDA tensor (`wrap`, nothing allocated). Carves start at 128 bytes."""

    def __init__(self, nbytes: int = None, *, wrap: torch.Tensor = None):
        h = C.c_void_p()
        if wrap is not None:
            self._keep = wrap
            _check(_L().jkb_scratch_wrap(_dptr(wrap), wrap.numel() * wrap.element_size(),
                                         C.byref(h)))
        else:
            _check(_L().jkb_scratch_create(nbytes, C.byref(h)))
        self._h = h.value

    @property
    def handle(self):
        if self._h is None:
            raise InvalidHandle(6, "ScratchWorkspace", 0, 0, 0, "scratch destroyed")
        return self._h

    def reset(self):
        _check(_L().jkb_scratch_reset(self.handle))

    def used_bytes(self) -> int:
        v = C.c_size_t()
        _check(_L().jkb_scratch_used_bytes(self.handle, C.byref(v)))
        return v.value

    def remaining_bytes(self) -> int:
        v = C.c_size_t()
        _check(_L().jkb_scratch_remaining_bytes(self.handle, C.byref(v)))
        return v.value

    def alloc(self, nbytes: int) -> int:
        """Carves nbytes; returns the device address."""
        p = C.c_void_p()
        _check(_L().jkb_scratch_alloc(self.handle, nbytes, C.byref(p)))
        return p.value

    def scope(self) -> "ScratchScope":
        """ScratchWorkspace::scope: carves inside the `with` block are released at its end."""
        return ScratchScope(self)

    def destroy(self):
        if getattr(self, "_h", None):
            _L().jkb_scratch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class ScratchScope:
    """jero_core::ScratchScope: a saved cursor of a workspace, rewound on exit."""

    def __init__(self, ws: ScratchWorkspace):
        self.ws = ws
        self.handle = ws.handle

    def __enter__(self):
        m = C.c_size_t()
        _check(_L().jkb_scratch_scope_begin(self.ws.handle, C.byref(m)))
        self.mark = m.value
        return self

    def __exit__(self, *exc):
        _check(_L().jkb_scratch_scope_end(self.ws.handle, self.mark))
        return False


def _in_scratch(fn, x, ws, bb, stream):
    p = C.c_void_p()
    _check(getattr(_L(), fn)(_dptr(x), x.numel(), ws.handle, C.byref(p), _stream(stream)))
    n = x.numel() // (32 if bb == BLOCK_Q8_0_BYTES else 256)
    return device_view(p.value, (n * bb,), "u1")


def quantize_row_q8_0_in_scratch(x, ws: ScratchWorkspace, stream=None) -> torch.Tensor:
    """quant_q8.rs:405: BlockQ8_0 blocks carved from the arena (a uint8 device view)."""
    return _in_scratch("jkb_quantize_row_q8_0_in_scratch", x, ws, BLOCK_Q8_0_BYTES, stream)


def quantize_row_q8_0_in_scope(x, scope: ScratchScope, stream=None) -> torch.Tensor:
    """quant_q8.rs:429."""
    return _in_scratch("jkb_quantize_row_q8_0_in_scope", x, scope, BLOCK_Q8_0_BYTES, stream)


def quantize_row_q8_k_in_scratch(x, ws: ScratchWorkspace, stream=None) -> torch.Tensor:
    """quant_q8.rs:602: BlockQ8K blocks carved from the arena (a uint8 device view)."""
    return _in_scratch("jkb_quantize_row_q8_k_in_scratch", x, ws, BLOCK_Q8_K_BYTES, stream)


def quantize_row_q8_k_in_scope(x, scope: ScratchScope, stream=None) -> torch.Tensor:
    """quant_q8.rs:626."""
    return _in_scratch("jkb_quantize_row_q8_k_in_scope", x, scope, BLOCK_Q8_K_BYTES, stream)


class QuantizedActQ8View:
    """QuantizedActQ8View (repack.rs:806-1090): quantized activations in device memory the
    library does not own (an arena's planes or a QuantizedActQ8's)."""

    def __init__(self, c_view, owner=None):
        self._c = c_view
        self._owner = owner  # keeps the arena or handle alive
        self.m, self.k, self.k_padded = c_view.m, c_view.k, c_view.k_padded

    @staticmethod
    def scratch_bytes_for_row(k: int) -> int:
        """repack.rs:827."""
        return int(_L().jkb_act_q8_view_scratch_bytes_for_row(k))

    @classmethod
    def quantize_row_in_scratch(cls, act, ws: ScratchWorkspace, stream=None):
        """repack.rs:870."""
        v = _lib.jkb_act_q8_view()
        _check(_L().jkb_act_q8_view_quantize_row_in_scratch(_dptr(act), act.numel(), ws.handle,
                                                            C.byref(v), _stream(stream)))
        return cls(v, ws)

    @classmethod
    def quantize_row_in_scope(cls, act, scope: ScratchScope, stream=None):
        """repack.rs:969."""
        v = _lib.jkb_act_q8_view()
        _check(_L().jkb_act_q8_view_quantize_row_in_scope(_dptr(act), act.numel(),
                                                          scope.handle, C.byref(v),
                                                          _stream(stream)))
        return cls(v, scope)

    def buffers(self):
        """Zero-copy device views: q, x_scales, x_sums, x_sums_16, super_scales."""
        c, m, kp = self._c, self.m, self.k_padded
        return (device_view(c.q, (m, kp), "i1"), device_view(c.x_scales, (m, kp // 32), "<f4"),
                device_view(c.x_sums, (m, kp // 32), "<f4"),
                device_view(c.x_sums_16, (m, kp // 16), "<f4"),
                device_view(c.super_scales, (m, (self.k + 255) // 256), "<f4"))


def gemv_repacked_view(out, weights: RepackedWeight, act: QuantizedActQ8View, stream=None):
    """repack.rs:4030 gemv_repacked_view."""
    _check(_L().jkb_gemv_repacked_view(_dptr(out), out.numel(), weights._h, C.byref(act._c),
                                       _stream(stream)))


def gemv_repacked_view_rows(out, weights: RepackedWeight, act: QuantizedActQ8View, row_range,
                            stream=None):
    """repack.rs:4045 gemv_repacked_view_rows."""
    _check(_L().jkb_gemv_repacked_view_rows(_dptr(out), out.numel(), weights._h,
                                            C.byref(act._c), row_range.start, row_range.stop,
                                            _stream(stream)))


def gemv_repacked_f32(out, weights: RepackedWeight, x, scratch: QuantizedActQ8, stream=None):
    """repack.rs:4101 gemv_repacked_f32 (the quantized row goes to the caller's handle)."""
    _check(_L().jkb_gemv_repacked_f32(_dptr(out), out.numel(), weights._h, _dptr(x), x.numel(),
                                      scratch._h, _stream(stream)))


def gemv_repacked_f32_rows(out, weights: RepackedWeight, x, row_range, scratch: QuantizedActQ8,
                           stream=None):
    """repack.rs:4114 gemv_repacked_f32_rows."""
    _check(_L().jkb_gemv_repacked_f32_rows(_dptr(out), out.numel(), weights._h, _dptr(x),
                                           x.numel(), row_range.start, row_range.stop,
                                           scratch._h, _stream(stream)))


def gemm_repacked_f32_rows(out, weights: RepackedWeight, x, m, row_range,
                           scratch: QuantizedActQ8, stream=None):
    """repack.rs:4143 gemm_repacked_f32_rows."""
    _check(_L().jkb_gemm_repacked_f32_rows(_dptr(out), out.numel(), weights._h, _dptr(x),
                                           x.numel(), m, row_range.start, row_range.stop,
                                           scratch._h, _stream(stream)))


# ------------------------------------------------------------------------------- load path

class BlockScaledTileLayout:
    """BlockScaledTileLayout (repack.rs:1286-1449) as block_scaled_layout fills it."""

    def __init__(self, c_layout):
        self._c = c_layout
        for name, _ in _lib.jkb_block_scaled_tile_layout._fields_:
            setattr(self, name, getattr(c_layout, name))
        self.quant = QuantType(self.quant)
        self.has_mins = bool(self.has_mins)


def block_scaled_layout(view: TensorView, rows: int, cols: int) -> BlockScaledTileLayout:
    """repack.rs:2372 RepackedWeight::block_scaled_layout (host only)."""
    L = _lib.jkb_block_scaled_tile_layout()
    v = view._c()
    _check(_L().jkb_block_scaled_layout(C.byref(v), rows, cols, C.byref(L)))
    return BlockScaledTileLayout(L)


def repack_into_tile_range(view: TensorView, rows: int, cols: int, tile_range, out_tiles=None,
                           out_scales=None, out_mins=None):
    """repack.rs:1579 repack_into_tile_range on host buffers (allocated here when not given):
    returns (tiles [tiles * k_chunks][128] u8, scales f32, mins f32 or None)."""
    L = block_scaled_layout(view, rows, cols)
    n = len(tile_range)
    if out_tiles is None:
        out_tiles = np.zeros((n * L.k_chunks, 128), np.uint8)
    if out_scales is None:
        out_scales = np.zeros(n * L.scale_groups * 8, np.float32)
    if out_mins is None and L.has_mins:
        out_mins = np.zeros(n * L.scale_groups * 8, np.float32)
    v = view._c()

    def ptr(a):
        return None if a is None else a.ctypes.data
    _check(_L().jkb_repack_into_tile_range(
        C.byref(v), rows, cols, tile_range.start, tile_range.stop, ptr(out_tiles),
        out_tiles.size // 128, ptr(out_scales), out_scales.size, ptr(out_mins),
        0 if out_mins is None else out_mins.size))
    return out_tiles, out_scales, out_mins


def repack_q4_k_m_parallel_slices(view: TensorView, rows: int, cols: int, tile_range,
                                  out_tiles_i8, out_scales, out_mins):
    """repack.rs:1659 repack_q4_k_m_parallel_slices (host numpy buffers)."""
    v = view._c()
    _check(_L().jkb_repack_q4_k_m_parallel_slices(
        C.byref(v), rows, cols, tile_range.start, tile_range.stop, out_tiles_i8.ctypes.data,
        out_tiles_i8.size, out_scales.ctypes.data, out_scales.size, out_mins.ctypes.data,
        out_mins.size))
