"""Generates the committed golden fixtures under tests/golden/.

kats.json -- known-answer tests restated from the jero-kernels-rvv test suite. The Rust crate
cannot be built in this environment (no cargo/rustc, its jero-core dependency is not vendored),
so the expected values are the ones its tests assert, written here as data with the file:line
of each assertion. Block bytes are hex strings.

oracle_fixtures.npz -- small seeded cases (every covered format, ragged row counts) evaluated
by the CPU oracle (oracle/jkb_oracle.c): weights, quantized activations, per-block integer
sums, block values and row outputs. The GPU tests compare against these fixed arrays, and the
CPU tests re-derive them from the live oracle so an oracle change cannot go unnoticed.

Run: python tests/golden/make_golden.py
"""
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def h16(v):
    return struct.pack("<H", v)


def kats():
    out = {}
    # quant.rs:2593-2629: Q8_0 d = 2.0 (0x4000), quants 1..=32, input ones -> 1056.
    blk = h16(0x4000) + bytes(range(1, 33))
    out["q8_0_vec_dot_f32"] = {"ref": "src/quant.rs:2593-2629", "quant": 8, "rows": 1,
                               "cols": 32, "block_hex": blk.hex(), "input": [1.0] * 32,
                               "expected": [1056.0], "abs_tol": 1e-4}
    # quant.rs:2632-2663: Q6_K d = 1.0, scales 1, ql 0x22, qh 0 -> every element -30,
    # dot with ones = -7680.
    blk = bytes([0x22] * 128) + bytes(64) + bytes([1] * 16) + h16(0x3C00)
    out["q6_k_vec_dot_f32"] = {"ref": "src/quant.rs:2632-2663", "quant": 14, "rows": 1,
                               "cols": 256, "block_hex": blk.hex(), "input": [1.0] * 256,
                               "expected": [-7680.0], "abs_tol": 1e-3,
                               "dequant_each": -30.0}
    # quant.rs:2727-2748: Q4_0 d = 0.5, nibbles lo 0xA (+2) hi 0x5 (-3), input 2s -> -16.
    blk = h16(0x3800) + bytes([0x5A] * 16)
    out["q4_0_vec_dot_f32"] = {"ref": "src/quant.rs:2727-2748", "quant": 2, "rows": 1,
                               "cols": 32, "block_hex": blk.hex(), "input": [2.0] * 32,
                               "expected": [-16.0], "abs_tol": 1e-4,
                               "dequant_lo": 1.0, "dequant_hi": -1.5}
    # lib.rs:1365-1396: two Q4_K_M blocks, d = 1.0, dmin = 0, scales[0..4] = 1, nibbles
    # lo = blk+1, hi = blk+2, shape [256, 2]; the test asserts out[0] > 0 and out[1] > out[0].
    # With sc[0..4] = 1 and sc[4..8] = 0 the exact values are 2*(32*1+32*2) = 192 and
    # 2*(32*2+32*3) = 320.
    raw = b""
    for b in range(2):
        blk = h16(0x3C00) + h16(0x0000) + bytes([1, 1, 1, 1]) + bytes(8)
        blk += bytes([((b + 2) << 4) | (b + 1)] * 128)
        raw += blk
    out["q4_k_m_two_block"] = {"ref": "src/lib.rs:1365-1396", "quant": 12, "shape": [256, 2],
                               "rows": 2, "cols": 256, "block_hex": raw.hex(),
                               "input": [1.0] * 256, "expected": [192.0, 320.0],
                               "abs_tol": 1e-4}
    # tests/empirical_challenge_m3_bitnet.rs:512-575: trit KATs.
    out["tq1_0_trits"] = {"ref": "tests/empirical_challenge_m3_bitnet.rs:512-556",
                          "cases": [{"fill": 0, "last": 0, "value": -1},
                                    {"fill": 121, "last": 1, "value": 0},
                                    {"fill": 242, "last": 2, "value": 1}],
                          "scale_hex": "003c", "scale": 1.0}
    out["tq2_0_trits"] = {"ref": "tests/empirical_challenge_m3_bitnet.rs:558-575",
                          "cases": [{"fill": 0x00, "value": -1}, {"fill": 0x55, "value": 0},
                                    {"fill": 0xAA, "value": 1}],
                          "scale_hex": "003c", "scale": 1.0}
    # tests/empirical_challenge_m3_bitnet.rs:39-163: SubLN absmax quantizer edge cases.
    out["subln"] = {
        "ref": "tests/empirical_challenge_m3_bitnet.rs:39-163,165-201",
        "len": 256, "eps": 1e-5,
        "cases": [
            {"name": "all_zero", "input": "zeros", "weight": "ones", "scale": 1.0 / 127.0,
             "q": 0},
            {"name": "zero_weight", "input": "iota1", "weight": "zeros", "scale": 1.0 / 127.0,
             "q": 0},
            {"name": "large_pos", "input": "const:1e6", "weight": "ones",
             "scale_approx": 1.0 / 127.0, "q": 127},
            {"name": "large_neg", "input": "const:-1e6", "weight": "ones",
             "scale_approx": 1.0 / 127.0, "q": -127},
            {"name": "alternating", "input": "alt:2.5", "weight": "ones",
             "scale_approx": 1.0 / 127.0, "q_even": 127, "q_odd": -127},
            {"name": "heterogeneous", "input": "ones", "weight": "alt_w:0.5:-2.0",
             "scale_approx": 2.0 / 127.0, "q_even": 32, "q_odd": -127},
            {"name": "nan", "input": "ones_nan13", "weight": "ones", "scale": 1.0 / 127.0,
             "q": 0},
            {"name": "inf", "input": "ones_inf42", "weight": "ones", "scale": 1.0 / 127.0,
             "q": 0},
            {"name": "tiny", "input": "const:1e-20", "weight": "ones", "q": 0},
        ]}
    # quant.rs:2836-2853: Q4_1 d = 0.5, m = -0.25, bytes 0xF0 -> lo nibble 0 gives -0.25, hi
    # nibble 15 gives 7.25; a zero d with m = -0.5 dequantizes to -0.5 everywhere.
    out["q4_1_dequant"] = {"ref": "src/quant.rs:2836-2853",
                           "cases": [{"block_hex": (h16(0x3800) + h16(0xB400) +
                                                    bytes([0xF0] * 16)).hex(),
                                      "lo": -0.25, "hi": 7.25},
                                     {"block_hex": (h16(0x0000) + h16(0xB800) + bytes(16)).hex(),
                                      "lo": -0.5, "hi": -0.5}]}
    # quant.rs:2895-2905: IQ4_NL d = 1.0, qs[0] = 0xF0, qs[1] = 0x08 -> out[0] = -127,
    # out[16] = 113, out[1] = 1, out[17] = -127.
    out["iq4_nl_dequant"] = {"ref": "src/quant.rs:2895-2905",
                             "block_hex": (h16(0x3C00) + bytes([0xF0, 0x08]) + bytes(14)).hex(),
                             "expect": {"0": -127.0, "16": 113.0, "1": 1.0, "17": -127.0}}
    # quant.rs:2665-2697: Q5_K d = 1.0, dmin = 0.5, scales[0..8] = 2,3,4,5,1,2,3,4, qh = 0x09,
    # qs[0..32] = 0x53, qs[32..64] = 0x24: the 256 dequantized values sum to 4928, and the f32
    # matvec against ones gives 4928.
    raw = bytearray(176)
    raw[0:2] = h16(0x3C00)
    raw[2:4] = h16(0x3800)
    for i, v in ((4, 2), (8, 1), (5, 3), (9, 2), (6, 4), (10, 3), (7, 5), (11, 4)):
        raw[i] = v
    raw[16:48] = bytes([0x09] * 32)
    raw[48:80] = bytes([0x53] * 32)
    raw[80:112] = bytes([0x24] * 32)
    out["q5_k_dequant_sum"] = {"ref": "src/quant.rs:2665-2697", "quant": 13, "rows": 1,
                               "cols": 256, "block_hex": bytes(raw).hex(), "input": [1.0] * 256,
                               "expected": [4928.0], "abs_tol": 1e-3, "sum": 4928.0}
    # quant.rs:2855-2862: Q5_0 d = 0.5, qh bit 0 set, qs[0] = 0x21: element 0 is
    # (1 | 16) - 16 = 1 -> 0.5, element 16 is (2 | 0) - 16 = -14 -> -7.
    blk = h16(0x3800) + bytes([1, 0, 0, 0]) + bytes([0x21]) + bytes(15)
    out["q5_0_dequant"] = {"ref": "src/quant.rs:2855-2862", "block_hex": blk.hex(),
                           "expect": {"0": 0.5, "16": -7.0}}
    # quant.rs:2910-2966: a two-block Q5_0 row (d = 0.5 / 1.0, qh 0xAAAA5555 / 0x0F0FF0F0, the
    # nibble patterns below) against x = (i - 31) / 16 (f32 path) and against the Q8_0 blocks of
    # d = 1.0, q = i - 31 (Q8 path): both within 1e-4 of the f32 dot with the dequantized row.
    row = bytearray(44)
    row[0:2] = h16(0x3800)
    row[2:6] = struct.pack("<I", 0xAAAA5555)
    for i in range(16):
        row[6 + i] = (i & 0x0F) | (((15 - i) & 0x0F) << 4)
    row[22:24] = h16(0x3C00)
    row[24:28] = struct.pack("<I", 0x0F0FF0F0)
    row[28:44] = bytes([0x5A] * 16)
    out["q5_0_two_block_row"] = {"ref": "src/quant.rs:2910-2966", "row_hex": bytes(row).hex(),
                                 "abs_tol": 1e-4}
    # quant.rs:2864-2873: Q5_1 d = 0.5, m = 1.0, qh bits 0 and 16 set, qs[0] = 0x32: element 0
    # is 0.5 * (2 + 16) + 1 = 10, element 16 is 0.5 * (3 + 16) + 1 = 10.5.
    blk = h16(0x3800) + h16(0x3C00) + struct.pack("<I", 0x00010001) + bytes([0x32]) + bytes(15)
    out["q5_1_dequant"] = {"ref": "src/quant.rs:2864-2873", "block_hex": blk.hex(),
                           "expect": {"0": 10.0, "16": 10.5}}
    # quant.rs:2875-2884: Q2_K sub-block 0 scale 2, min 1, code 3, d = 1.0, dmin = 0.5:
    # element 0 is 1 * 2 * 3 - 0.5 * 1 = 5.5.
    raw = bytearray(84)
    raw[0] = (1 << 4) | 2
    raw[16] = 0x03
    raw[80:82] = h16(0x3C00)
    raw[82:84] = h16(0x3800)
    out["q2_k_dequant"] = {"ref": "src/quant.rs:2875-2884", "block_hex": bytes(raw).hex(),
                           "expect": {"0": 5.5}}
    # quant.rs:2886-2893: Q3_K hmask 0, every 6-bit scale 33 (scales[0..8] = 0x11,
    # scales[8..12] = 0xAA), qs[0] = 3, d = 0.5: element 0 is 0.5 * (33 - 32) * (3 - 4) = -0.5.
    raw = bytearray(110)
    raw[96:104] = bytes([0x11] * 8)
    raw[104:108] = bytes([0xAA] * 4)
    raw[32] = 0x03
    raw[108:110] = h16(0x3800)
    out["q3_k_dequant"] = {"ref": "src/quant.rs:2886-2893", "block_hex": bytes(raw).hex(),
                           "expect": {"0": -0.5}}
    # quant_q8.rs:3414-3482: quantizer sanitization on test_f32_row inputs.
    out["q8_sanitize"] = {"ref": "src/quant_q8.rs:3388-3395,3414-3482"}
    return out


def test_f32_row(n, seed):
    """quant_q8.rs:3388-3395 generator: ((i*37 + seed*13) % 29 - 14) * 0.125."""
    return np.array([(((i * 37 + seed * 13) % 29) - 14) * 0.125 for i in range(n)], np.float32)


def fixtures():
    import pyoracle as O

    data = {}
    cases = [
        ("q4_0", O.Q4_0, 5, 256), ("q4_0_b", O.Q4_0, 17, 1024),
        ("q8_0", O.Q8_0, 5, 256), ("q8_0_b", O.Q8_0, 33, 512),
        ("q4_k", O.Q4_K, 5, 512), ("q4_k_b", O.Q4_K, 19, 1024),
        ("q6_k", O.Q6_K, 5, 512), ("q6_k_b", O.Q6_K, 21, 768),
        ("tq2_0", O.TQ2_0, 7, 512),
        ("q5_0", O.Q5_0, 9, 512), ("q5_k", O.Q5_K, 7, 768),
    ]
    for name, q, rows, cols in cases:
        seed = sum(map(ord, name))
        if q == O.TQ2_0:
            t = O.ternary(rows * cols, 0x5EED0000 + seed)
            w = O.pack_ternary(q, t, rows, cols, 0.0125)
        else:
            W = O.normal(rows * cols, 0x5EED0000 + seed, 0.02)
            w = O.quantize_weights(q, W, rows, cols)
        x = O.normal(cols, 0xAC70000 + seed, 1.0)
        xq = O.quantize_act(q, x)
        sumi, summins, contrib = O.block_dots(q, w, rows, cols, xq)
        y = O.gemv(q, w, rows, cols, xq)
        data[f"{name}__meta"] = np.array([q, rows, cols], np.int64)
        data[f"{name}__w"] = w
        data[f"{name}__x"] = x
        data[f"{name}__xq"] = xq.view(np.uint8).reshape(-1)
        data[f"{name}__sumi"] = sumi
        data[f"{name}__summins"] = summins
        data[f"{name}__contrib"] = contrib
        data[f"{name}__y"] = y
    # compact nibble GEMM (PackedNibbleMatrix) of the formats without a GEMV here: weights,
    # activation and the oracle's output
    for name, q, rows, cols, m in (("nib_q4_1", O.Q4_1, 13, 256, 5),
                                   ("nib_iq4_nl", O.IQ4_NL, 11, 512, 3)):
        seed = sum(map(ord, name))
        w = O.quantize_weights(q, O.normal(rows * cols, 0x5EED0000 + seed, 0.02), rows, cols)
        x = O.normal(m * cols, 0xAC70000 + seed, 1.0)
        xq, xs, xsum, _, _ = O.act_q8_quantize(x, m, cols)
        nq, ws, wm = O.nibble_decode(q, w, rows, cols)
        data[f"{name}__nmeta"] = np.array([q, rows, cols, m], np.int64)
        data[f"{name}__w"] = w
        data[f"{name}__x"] = x
        data[f"{name}__out"] = O.gemm_nibble(q, nq, ws, wm, rows, cols, xq, xs, xsum, m)
    return data


def main():
    with open(os.path.join(HERE, "kats.json"), "w") as f:
        json.dump(kats(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "oracle_fixtures.npz"), **fixtures())
    print("wrote kats.json and oracle_fixtures.npz")


if __name__ == "__main__":
    main()
