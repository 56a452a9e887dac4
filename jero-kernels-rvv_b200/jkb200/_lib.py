"""Loads libjkb200.so (the C ABI of include/jkb200.h) and declares its signatures.

The shared object is built in-tree by ``jero-kernels-rvv_b200/Makefile`` (nvcc, sm_100a only).
There is no fallback: if the library is missing, importing the package raises.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(ROOT_DIR, "libjkb200.so")


class jkb_tensor_view(C.Structure):
    _fields_ = [
        ("name", C.c_char_p),
        ("quant", C.c_int32),
        ("ndim", C.c_uint32),
        ("shape", C.c_size_t * 4),
        ("offset", C.c_size_t),
        ("data", C.c_void_p),
        ("byte_len", C.c_size_t),
        ("data_on_device", C.c_int32),
    ]


class jkb_vec_dot_item(C.Structure):
    _fields_ = [
        ("out", C.c_void_p),
        ("out_len", C.c_size_t),
        ("w", C.c_void_p),
    ]


class jkb_error_info(C.Structure):
    _fields_ = [
        ("status", C.c_int32),
        ("tensor_name", C.c_char * 64),
        ("offset", C.c_size_t),
        ("byte_len", C.c_size_t),
        ("buffer_len", C.c_size_t),
        ("reason", C.c_char * 256),
    ]


class jkb_block_scaled_tile_layout(C.Structure):
    _fields_ = [
        ("quant", C.c_int32),
        ("has_mins", C.c_int32),
        ("rows", C.c_size_t),
        ("cols", C.c_size_t),
        ("row_bytes", C.c_size_t),
        ("k_padded", C.c_size_t),
        ("n_tiles", C.c_size_t),
        ("k_chunks", C.c_size_t),
        ("chunks_per_scale", C.c_size_t),
        ("scale_groups", C.c_size_t),
        ("total_tiles", C.c_size_t),
        ("total_scales", C.c_size_t),
        ("total_mins", C.c_size_t),
    ]


class jkb_act_q8_view(C.Structure):
    _fields_ = [
        ("m", C.c_size_t),
        ("k", C.c_size_t),
        ("k_padded", C.c_size_t),
        ("q", C.c_void_p),
        ("x_scales", C.c_void_p),
        ("x_sums", C.c_void_p),
        ("x_sums_16", C.c_void_p),
        ("super_scales", C.c_void_p),
    ]


P, S, I, F = C.c_void_p, C.c_size_t, C.c_int, C.c_float
PP = C.POINTER(C.c_void_p)
PS = C.POINTER(C.c_size_t)
PI32 = C.POINTER(C.c_int32)

# name -> argument types (every entry point returns int status unless listed in _RESTYPE)
SIGNATURES = {
    "jkb_abi_version": [],
    "jkb_last_error": [],
    "jkb_last_error_info": [C.POINTER(jkb_error_info)],
    "jkb_clear_error": [],
    "jkb_device_status": [PI32, P],
    "jkb_gemm_set_exact": [I],
    "jkb_gemm_get_exact": [],
    "jkb_quantize_row_q8_0": [P, S, P, S, P],
    "jkb_quantize_row_q8_0_f32": [P, S, P, S, P],
    "jkb_quantize_row_q8_k": [P, S, P, S, P],
    "jkb_quantize_rows_q8_0": [P, S, S, P, S, P],
    "jkb_quantize_rows_q8_k": [P, S, S, P, S, P],
    "jkb_subln_quantize_absmax_i8": [P, S, P, S, P, S, F, P, P],
    "jkb_subln_quantize_absmax_i8_rows": [P, P, P, S, S, F, P, P],
    "jkb_relu_squared_gate_f32": [P, S, P, S, P, S, P],
    "jkb_relu_squared_subln_quantize_i8_rows": [P, P, P, P, P, S, S, F, P, P],
    "jkb_bitnet_ffn_create": [P, P, P, P, P, P, P, S, P, S, F, S, PP],
    "jkb_bitnet_ffn_forward": [P, P, S, P, S, S, P],
    "jkb_bitnet_ffn_buffers": [P, PP, PP, PP, PP, PP, PP, PP],
    "jkb_bitnet_ffn_destroy": [P],
    "jkb_bitlinear_i8_gemm": [P, S, P, P, S, P, S, P, P],
    "jkb_repacked_weight_dequantize_row": [P, S, P, S, P],
    "jkb_act_q8_create": [S, S, PP],
    "jkb_act_q8_destroy": [P],
    "jkb_act_q8_quantize": [P, P, S, S, S, P],
    "jkb_act_q8_buffers": [P, PS, PS, PS, PP, PP, PP, PP, PP],
    "jkb_weight_upload": [C.POINTER(jkb_tensor_view), S, S, P, PP],
    "jkb_weight_upload_infer": [C.POINTER(jkb_tensor_view), P, PP],
    "jkb_weight_destroy": [P],
    "jkb_weight_info": [P, PS, PS, PI32, PS, PS],
    "jkb_vec_dot_q4_0_q8_0": [P, S, P, S, P, P],
    "jkb_vec_dot_q8_0_q8_0": [P, S, P, S, P, P],
    "jkb_vec_dot_q4_k_q8_k": [P, S, P, S, P, P],
    "jkb_vec_dot_q6_k_q8_k": [P, S, P, S, P, P],
    "jkb_vec_dot_q5_0_q8_0_blocks": [P, S, P, S, P, P],
    "jkb_vec_dot_q5_k_q8_k": [P, S, P, S, P, P],
    "jkb_vec_dot_tq1_0_q8_k": [P, S, P, S, P, P],
    "jkb_vec_dot_tq2_0_q8_k": [P, S, P, S, P, P],
    "jkb_gemv_q4_0_q8_0": [P, S, P, P, S, P],
    "jkb_gemv_q4_0_q8_0_4x": [P, S, P, P, S, P],
    "jkb_gemv_q8_0_q8_0": [P, S, P, P, S, P],
    "jkb_gemv_q8_0_q8_0_4x": [P, S, P, P, S, P],
    "jkb_gemv_q4_k_q8_k": [P, S, P, P, S, P],
    "jkb_gemv_q6_k_q8_k": [P, S, P, P, S, P],
    "jkb_gemv_q5_0_q8_0": [P, S, P, P, S, P],
    "jkb_gemv_q5_0_q8_0_4x": [P, S, P, P, S, P],
    "jkb_gemv_q5_k_q8_k": [P, S, P, P, S, P],
    "jkb_gemv_tq1_0_q8_k": [P, S, P, P, S, P],
    "jkb_gemv_tq2_0_q8_k": [P, S, P, P, S, P],
    "jkb_gemv_rows": [P, S, P, P, S, S, S, P],
    "jkb_gemv_batch": [P, S, P, P, S, S, P],
    "jkb_gemv_block_dots": [P, P, S, P, P, P, P],
    "jkb_vec_dot_q4_k_m": [P, S, P, P, S, P],
    "jkb_vec_dot_q8_0": [P, S, P, P, S, P],
    "jkb_vec_dot_q6_k": [P, S, P, P, S, P],
    "jkb_vec_dot_q4_0": [P, S, P, P, S, P],
    "jkb_vec_dot_q5_0": [P, S, P, P, S, P],
    "jkb_vec_dot_q5_k": [P, S, P, P, S, P],
    "jkb_vec_dot_i2_s": [P, S, P, P, S, P],
    "jkb_vec_dot_q5_0_rvv": [P, S, P, P, S, P],
    "jkb_vec_dot_q5_k_rvv": [P, S, P, P, S, P],
    "jkb_vec_dot_q4_k_m_rvv": [P, S, P, P, S, P],
    "jkb_vec_dot_q6_k_rvv": [P, S, P, P, S, P],
    "jkb_vec_dot_q8_0_rvv": [P, S, P, P, S, P],
    "jkb_vec_dot_q4_0_rvv": [P, S, P, P, S, P],
    "jkb_vec_dot_grouped_rvv": [C.POINTER(jkb_vec_dot_item), S, P, S, P],
    "jkb_peer_group_create": [I, I, S, PP],
    "jkb_peer_group_handle": [P, P],
    "jkb_peer_group_open": [P, P],
    "jkb_peer_group_buffer": [P, PP, PS],
    "jkb_peer_group_allgather": [P, PS, PS, S, P],
    "jkb_peer_group_wait": [P, C.c_uint64, P],
    "jkb_peer_group_set_push": [P, I],
    "jkb_peer_group_signal": [P, P],
    "jkb_peer_group_destroy": [P],
    "jkb_bitlinear_i8": [P, S, P, P, S, F, P],
    "jkb_bitlinear_i8_rvv": [P, S, P, P, S, F, P],
    "jkb_bitlinear_i8_ime": [P, S, P, P, S, F, P],
    "jkb_bitlinear_i8_batch": [P, S, P, P, S, P, S, P],
    "jkb_repacked_weight_from_tensor": [C.POINTER(jkb_tensor_view), S, S, P, PP],
    "jkb_repacked_weight_repack": [C.POINTER(jkb_tensor_view), P, PP],
    "jkb_repacked_weight_destroy": [P],
    "jkb_repacked_weight_buffers": [P, PS, PS, PI32, PS, PP, PP, PP],
    "jkb_gemm_repacked": [P, S, P, P, P],
    "jkb_gemm_repacked_rows": [P, S, P, P, S, S, P],
    "jkb_gemv_repacked": [P, S, P, P, P],
    "jkb_gemv_repacked_rows": [P, S, P, P, S, S, P],
    "jkb_gemm_repacked_f32": [P, S, P, P, S, S, P, P],
    "jkb_gemm_repacked_f32_noalloc": [P, S, P, P, S, S, P],
    "jkb_packed_nibble_matrix_from_tensor": [C.POINTER(jkb_tensor_view), S, S, P, PP],
    "jkb_packed_nibble_matrix_repack": [C.POINTER(jkb_tensor_view), P, PP],
    "jkb_packed_nibble_matrix_from_scale_f16_buffers": [I, S, S, P, S, P, S, P, PP],
    "jkb_packed_nibble_matrix_from_q4_k_buffers": [S, S, P, S, P, S, P, PP],
    "jkb_repack_nibble_into_tile_range": [C.POINTER(jkb_tensor_view), S, S, S, S, P, S, P, S, P,
                                          S, P, S],
    "jkb_packed_nibble_matrix_destroy": [P],
    "jkb_packed_nibble_matrix_info": [P, PS, PS, PI32, PS, PS, PS, PS],
    "jkb_packed_nibble_matrix_buffers": [P, PP, PP],
    "jkb_packed_nibble_matrix_gemm": [P, S, P, P, P],
    "jkb_packed_nibble_matrix_gemm_rows": [P, S, P, P, S, S, P],
    "jkb_packed_nibble_matrix_gemv": [P, S, P, P, P],
    "jkb_packed_nibble_matrix_dequantize_row": [P, S, P, S, P],
    "jkb_gemm_q4_0_ime": [P, S, P, P, P],
    "jkb_gemm_q4_k_ime": [P, S, P, P, P],
    "jkb_quantize_row_f32_to_q8_32": [P, S, P, S, P, S, P, S, P],
    "jkb_scratch_create": [S, PP],
    "jkb_scratch_wrap": [P, S, PP],
    "jkb_scratch_destroy": [P],
    "jkb_scratch_reset": [P],
    "jkb_scratch_used_bytes": [P, PS],
    "jkb_scratch_remaining_bytes": [P, PS],
    "jkb_scratch_alloc": [P, S, PP],
    "jkb_scratch_scope_begin": [P, PS],
    "jkb_scratch_scope_end": [P, S],
    "jkb_quantize_row_q8_0_in_scratch": [P, S, P, PP, P],
    "jkb_quantize_row_q8_0_in_scope": [P, S, P, PP, P],
    "jkb_quantize_row_q8_k_in_scratch": [P, S, P, PP, P],
    "jkb_quantize_row_q8_k_in_scope": [P, S, P, PP, P],
    "jkb_act_q8_view_scratch_bytes_for_row": [S],
    "jkb_act_q8_view_quantize_row_in_scratch": [P, S, P, C.POINTER(jkb_act_q8_view), P],
    "jkb_act_q8_view_quantize_row_in_scope": [P, S, P, C.POINTER(jkb_act_q8_view), P],
    "jkb_act_q8_as_view": [P, C.POINTER(jkb_act_q8_view)],
    "jkb_gemv_repacked_view": [P, S, P, C.POINTER(jkb_act_q8_view), P],
    "jkb_gemv_repacked_view_rows": [P, S, P, C.POINTER(jkb_act_q8_view), S, S, P],
    "jkb_gemv_repacked_f32": [P, S, P, P, S, P, P],
    "jkb_gemv_repacked_f32_rows": [P, S, P, P, S, S, S, P, P],
    "jkb_gemm_repacked_f32_rows": [P, S, P, P, S, S, S, S, P, P],
    "jkb_block_scaled_layout": [C.POINTER(jkb_tensor_view), S, S,
                                C.POINTER(jkb_block_scaled_tile_layout)],
    "jkb_repack_into_tile_range": [C.POINTER(jkb_tensor_view), S, S, S, S, P, S, P, S, P, S],
    "jkb_repack_q4_k_m_parallel_slices": [C.POINTER(jkb_tensor_view), S, S, S, S, P, S, P, S, P,
                                          S],
    "jkb_repacked_weight_from_tile_buffers": [C.POINTER(jkb_block_scaled_tile_layout), P, S, P, S,
                                              P, S, P, PP],
}
_RESTYPE = {"jkb_last_error": C.c_char_p, "jkb_clear_error": None,
            "jkb_act_q8_view_scratch_bytes_for_row": C.c_size_t}

_lib = None


def load() -> C.CDLL:
    """Return the loaded ABI library; raise ImportError (no fallback) when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C {ROOT_DIR}` (nvcc, sm_100a). "
            "jkb200 has no CPU fallback.")
    lib = C.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, C.c_int)
    _lib = lib
    return lib


def declared_symbols():
    return list(SIGNATURES)
