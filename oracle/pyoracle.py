"""ctypes view of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline use
this module as the checker. The product path (``jkb200``) never imports it.

The oracle restates the jero-kernels-rvv scalar fallback; each C function cites the reference
file:line it follows. numpy arrays are passed by pointer; block activations use structured
dtypes laid out exactly like the reference ``#[repr(C)]`` structs.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

# QuantType codes shared with include/jkb200.h (GGML type ids where one exists).
Q4_0, Q8_0, Q4_K, Q6_K, TQ1_0, TQ2_0, I2_S = 2, 8, 12, 14, 34, 35, 36
Q4_1, IQ4_NL, Q5_0, Q5_K = 3, 20, 6, 13
Q5_1, Q2_K, Q3_K = 7, 10, 11
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210),
         TQ1_0: (256, 54), TQ2_0: (256, 66), I2_S: (128, 32), Q4_1: (32, 20), IQ4_NL: (32, 18),
         Q5_0: (32, 22), Q5_K: (256, 176), Q5_1: (32, 24), Q2_K: (256, 84), Q3_K: (256, 110)}
# formats a RepackedWeight holds (BlockScaledTileLayout::for_tensor, repack.rs:1308-1336)
REPACKABLE = (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ4_NL, TQ1_0,
              TQ2_0, I2_S)
NIBBLE = (Q4_0, Q4_1, IQ4_NL, Q4_K)  # PackedNibbleMatrix formats (repack.rs:4231-4236)
NIBBLE_MINS = (Q4_1, Q4_K)
ACT_IS_Q8K = {Q4_0: False, Q8_0: False, Q4_K: True, Q6_K: True, TQ1_0: True, TQ2_0: True,
              Q5_0: False, Q5_K: True}

# quant_q8.rs:37-44 and :62-71
BLOCK_Q8_0 = np.dtype([("d", "<f4"), ("qs", "i1", (32,))])
BLOCK_Q8_K = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsums", "<i2", (16,))])
assert BLOCK_Q8_0.itemsize == 36 and BLOCK_Q8_K.itemsize == 292


def build() -> str:
    """Compile the oracle with its Makefile (gcc only) if the shared object is missing/stale."""
    src = os.path.join(HERE, "jkb_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        P, S, I, F, U64 = C.c_void_p, C.c_size_t, C.c_int, C.c_float, C.c_uint64
        sig = {
            "or_f16_to_f32_ieee": (F, [C.c_uint16]),
            "or_f16_to_f32_finite": (F, [C.c_uint16]),
            "or_f32_to_f16": (C.c_uint16, [F]),
            "or_quantize_row_q8_0": (I, [P, S, P, S]),
            "or_quantize_row_q8_k": (I, [P, S, P, S]),
            "or_quantize_rows_q8_0": (I, [P, S, S, P]),
            "or_quantize_rows_q8_k": (I, [P, S, S, P]),
            "or_quantize_block32": (None, [P, P, P, P]),
            "or_act_q8_quantize": (I, [P, S, S, P, P, P, P, P]),
            "or_subln_quantize_absmax_i8": (I, [P, P, P, S, F, P]),
            "or_relu_squared_gate_f32": (I, [P, P, P, S]),
            "or_block_dots": (I, [I, P, S, S, P, P, P, P]),
            "or_gemv": (I, [I, P, P, S, S, P]),
            "or_gemv_rows_mt": (I, [I, P, P, S, S, P, S, S, I]),
            "or_vec_dot": (F, [I, P, P, S]),
            "or_dequantize_block": (None, [I, P, F, P]),
            "or_dot_product_f32": (F, [P, P, S]),
            "or_dequantize_rows": (I, [I, P, S, S, P]),
            "or_vec_dot_f32": (I, [I, P, P, S, S, S, P]),
            "or_bitlinear_i8": (I, [P, I, P, S, S, S, P, F]),
            "or_bitlinear_i8_rows_mt": (I, [P, I, P, S, S, S, P, F, S, P, I]),
            "or_repack_scale_groups": (S, [I, S]),
            "or_repack_has_mins": (I, [I]),
            "or_repack_block_scaled": (I, [I, P, S, S, S, P, P, P]),
            "or_gemm_repacked": (I, [P, I, P, P, P, S, S, P, P, P, P, S, S, S, I]),
            "or_fill_normal": (None, [P, S, U64, F]),
            "or_fill_ternary": (None, [P, S, U64]),
            "or_quantize_weights": (I, [I, P, S, S, P]),
            "or_pack_ternary": (I, [I, P, S, S, F, P]),
            "or_weight_bytes": (S, [I, S, S]),
            "or_nibble_supported": (I, [I]),
            "or_nibble_pack_tiles": (I, [I, P, S, S, S, P, P, P, P]),
            "or_nibble_decode_tiles": (I, [I, S, S, P, P, P, P, P, P, P]),
            "or_nibble_dequantize_row": (I, [I, P, P, P, S, S, P]),
            "or_gemm_nibble": (I, [P, I, P, P, P, S, S, P, P, P, S, S, S, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def weight_bytes(quant: int, rows: int, cols: int) -> int:
    return int(lib().or_weight_bytes(quant, rows, cols))


def normal(n: int, seed: int, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_fill_normal(_p(out), n, seed, sigma)
    return out


def ternary(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.int8)
    lib().or_fill_ternary(_p(out), n, seed)
    return out


def quantize_weights(quant: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros(weight_bytes(quant, rows, cols), np.uint8)
    assert lib().or_quantize_weights(quant, _p(w), rows, cols, _p(out)) == 0
    return out


def pack_ternary(quant: int, t: np.ndarray, rows: int, cols: int, scale: float) -> np.ndarray:
    t = np.ascontiguousarray(t, np.int8)
    out = np.zeros(weight_bytes(quant, rows, cols), np.uint8)
    assert lib().or_pack_ternary(quant, _p(t), rows, cols, scale, _p(out)) == 0
    return out


def quantize_row_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size // 32, BLOCK_Q8_0)
    if lib().or_quantize_row_q8_0(_p(x), x.size, _p(out), out.size) != 0:
        raise ValueError("quantize_row_q8_0: bad length")
    return out


def quantize_row_q8_k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size // 256, BLOCK_Q8_K)
    if lib().or_quantize_row_q8_k(_p(x), x.size, _p(out), out.size) != 0:
        raise ValueError("quantize_row_q8_k: bad length")
    return out


def quantize_act(quant: int, x: np.ndarray) -> np.ndarray:
    return quantize_row_q8_k(x) if ACT_IS_Q8K[quant] else quantize_row_q8_0(x)


def gemv(quant: int, w: np.ndarray, rows: int, cols: int, xq: np.ndarray) -> np.ndarray:
    out = np.zeros(rows, np.float32)
    assert lib().or_gemv(quant, _p(out), _p(w), rows, cols, _p(xq)) == 0
    return out


def gemv_mt(quant, w, rows, cols, xq, nthreads, row_begin=0, row_end=None):
    row_end = rows if row_end is None else row_end
    out = np.zeros(row_end - row_begin, np.float32)
    assert lib().or_gemv_rows_mt(quant, _p(out), _p(w), rows, cols, _p(xq), row_begin, row_end,
                                 nthreads) == 0
    return out


def block_dots(quant, w, rows, cols, xq):
    nb = cols // BLOCK[quant][0]
    sumi = np.zeros((rows, nb), np.int32)
    summins = np.zeros((rows, nb), np.int32)
    contrib = np.zeros((rows, nb), np.float32)
    assert lib().or_block_dots(quant, _p(w), rows, cols, _p(xq), _p(sumi), _p(summins),
                               _p(contrib)) == 0
    return sumi, summins, contrib


def vec_dot(quant, w_row, xq) -> float:
    return float(lib().or_vec_dot(quant, _p(w_row), _p(xq), xq.size))


def vec_dot_f32(quant, w, rows, cols, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(rows, np.float32)
    assert lib().or_vec_dot_f32(quant, _p(out), _p(w), w.size, rows, cols, _p(x)) == 0
    return out


def dequantize_block(quant, blk, i2s_scale=0.0) -> np.ndarray:
    out = np.zeros(BLOCK[quant][0], np.float32)
    lib().or_dequantize_block(quant, _p(blk), i2s_scale, _p(out))
    return out


def dequantize_rows(quant, w, rows, cols) -> np.ndarray:
    out = np.zeros((rows, cols), np.float32)
    assert lib().or_dequantize_rows(quant, _p(w), rows, cols, _p(out)) == 0
    return out


def subln_quantize_absmax_i8(x, norm_w, eps):
    x = np.ascontiguousarray(x, np.float32)
    norm_w = np.ascontiguousarray(norm_w, np.float32)
    out = np.zeros(x.size, np.int8)
    scale = np.zeros(1, np.float32)
    if lib().or_subln_quantize_absmax_i8(_p(out), _p(x), _p(norm_w), x.size, eps, _p(scale)):
        raise ValueError("subln: bad length")
    return out, float(scale[0])


def relu_squared_gate_f32(gate, up) -> np.ndarray:
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    if gate.size == 0 or up.size != gate.size:
        raise ValueError("relu_squared: dimension mismatch")
    out = np.zeros(gate.size, np.float32)
    assert lib().or_relu_squared_gate_f32(_p(out), _p(gate), _p(up), gate.size) == 0
    return out


def bitnet_ffn(x, norm1, norm2, eps, gate_q, w_gate, up_q, w_up, down_q, w_down, hidden, inter):
    """The BitNet FFN chain of tests/empirical_challenge_m3_bitnet.rs:582-686 (PATH A) for one
    token: SubLN -> gate/up BitLinear -> ReLU^2 gating -> SubLN -> down BitLinear. Returns every
    intermediate: act1, scale1, gate, up, relu, act2, scale2, out."""
    act1, s1 = subln_quantize_absmax_i8(x, norm1, eps)
    g = bitlinear_i8(gate_q, w_gate, inter, hidden, act1, s1)
    u = bitlinear_i8(up_q, w_up, inter, hidden, act1, s1)
    h = relu_squared_gate_f32(g, u)
    act2, s2 = subln_quantize_absmax_i8(h, norm2, eps)
    out = bitlinear_i8(down_q, w_down, hidden, inter, act2, s2)
    return dict(act1=act1, scale1=s1, gate=g, up=u, relu=h, act2=act2, scale2=s2, out=out)


def bitlinear_i8(quant, w, rows, cols, act, act_scale) -> np.ndarray:
    act = np.ascontiguousarray(act, np.int8)
    out = np.zeros(rows, np.float32)
    rc = lib().or_bitlinear_i8(_p(out), quant, _p(w), w.size, rows, cols, _p(act), act_scale)
    if rc != 0:
        raise ValueError(f"bitlinear_i8 rc={rc}")
    return out


def bitlinear_i8_batch(quant, w, rows, cols, act, act_scales, nthreads=1) -> np.ndarray:
    act = np.ascontiguousarray(act, np.int8)
    act_scales = np.ascontiguousarray(act_scales, np.float32)
    m = act_scales.size
    out = np.zeros((m, rows), np.float32)
    assert lib().or_bitlinear_i8_rows_mt(_p(out), quant, _p(w), w.size, rows, cols, _p(act), 0.0,
                                         m, _p(act_scales), nthreads) == 0
    return out


def act_q8_quantize(act: np.ndarray, m: int, k: int):
    act = np.ascontiguousarray(act, np.float32)
    kp = (k + 31) // 32 * 32
    q = np.zeros((m, kp), np.int8)
    xs = np.zeros((m, kp // 32), np.float32)
    xsum = np.zeros((m, kp // 32), np.float32)
    xs16 = np.zeros((m, kp // 16), np.float32)
    sup = np.zeros((m, (k + 255) // 256), np.float32)
    assert lib().or_act_q8_quantize(_p(act), m, k, _p(q), _p(xs), _p(xsum), _p(xs16),
                                    _p(sup)) == 0
    return q, xs, xsum, xs16, sup


def repack_block_scaled(quant, raw, rows, cols):
    kp = (cols + 31) // 32 * 32
    sg = int(lib().or_repack_scale_groups(quant, cols))
    q = np.zeros((rows, kp), np.int8)
    s = np.zeros((rows, sg), np.float32)
    m = np.zeros((rows, sg), np.float32) if lib().or_repack_has_mins(quant) else None
    assert lib().or_repack_block_scaled(quant, _p(raw), raw.size, rows, cols, _p(q), _p(s),
                                        _p(m)) == 0
    return q, s, m


def gemm_repacked(quant, wq, ws, wm, rows, cols, xq, xs, xsum, xs16, m, row_begin=0,
                  row_end=None, nthreads=1):
    row_end = rows if row_end is None else row_end
    out = np.zeros((m, row_end - row_begin), np.float32)
    assert lib().or_gemm_repacked(_p(out), quant, _p(wq), _p(ws), _p(wm), rows, cols, _p(xq),
                                  _p(xs), _p(xsum), _p(xs16), m, row_begin, row_end,
                                  nthreads) == 0
    return out


# ---- compact nibble matrices (PackedNibbleMatrix) ----

def nibble_pack_tiles(quant, raw, rows, cols):
    """The reference's tile layout (repack_nibble_into_tile_range): (tiles u8 [n_tiles*kb*128],
    scales_f16 or None, mins_f16 or None, headers u8 [n_tiles*(cols/256)*8*16] or None)."""
    nt, kb = (rows + 7) // 8, cols // 32
    tiles = np.zeros(nt * kb * 128, np.uint8)
    sc = mn = hd = None
    if quant == Q4_K:
        hd = np.zeros(nt * (cols // 256) * 8 * 16, np.uint8)
    else:
        sc = np.zeros(nt * kb * 8, np.uint16)
        if quant == Q4_1:
            mn = np.zeros(nt * kb * 8, np.uint16)
    raw = np.ascontiguousarray(raw, np.uint8)
    assert lib().or_nibble_pack_tiles(quant, _p(raw), raw.size, rows, cols, _p(tiles), _p(sc),
                                      _p(mn), _p(hd)) == 0
    return tiles, sc, mn, hd


def nibble_decode_tiles(quant, rows, cols, tiles, sc, mn, hd):
    """decode_tile_scales + unpack_nibble_tile_to_chunks, row-major: (q [rows][cols] i8,
    ws [rows][cols/32], wm [rows][cols/32] or None)."""
    kb = cols // 32
    q = np.zeros((rows, cols), np.int8)
    ws = np.zeros((rows, kb), np.float32)
    wm = np.zeros((rows, kb), np.float32) if quant in NIBBLE_MINS else None
    assert lib().or_nibble_decode_tiles(quant, rows, cols, _p(tiles), _p(sc), _p(mn), _p(hd),
                                        _p(q), _p(ws), _p(wm)) == 0
    return q, ws, wm


def nibble_decode(quant, raw, rows, cols):
    return nibble_decode_tiles(quant, rows, cols, *nibble_pack_tiles(quant, raw, rows, cols))


def nibble_dequantize_row(quant, q, ws, wm, cols, row):
    out = np.zeros(cols, np.float32)
    assert lib().or_nibble_dequantize_row(quant, _p(q), _p(ws), _p(wm), cols, row, _p(out)) == 0
    return out


def gemm_nibble(quant, q, ws, wm, rows, cols, xq, xs, xsum, m, row_begin=0, row_end=None,
                nthreads=1):
    row_end = rows if row_end is None else row_end
    out = np.zeros((m, row_end - row_begin), np.float32)
    assert lib().or_gemm_nibble(_p(out), quant, _p(q), _p(ws), _p(wm), rows, cols, _p(xq),
                                _p(xs), _p(xsum), m, row_begin, row_end, nthreads) == 0
    return out
