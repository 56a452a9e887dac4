"""Pins the CPU oracle (oracle/jkb_oracle.c) to the jero-kernels-rvv test suite: its
known-answer tests, exhaustive decode tests, sanitization cases and the tolerance contracts of
its GEMV/GEMM tests, plus the committed golden fixtures. CPU only."""
import json
import os
import struct

import numpy as np
import pytest

import refgen as R

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def kats():
    with open(os.path.join(GOLDEN, "kats.json")) as f:
        return json.load(f)


def _u8(hexs):
    return np.frombuffer(bytes.fromhex(hexs), np.uint8).copy()


@pytest.mark.parametrize("name", ["q8_0_vec_dot_f32", "q6_k_vec_dot_f32", "q4_0_vec_dot_f32",
                                  "q4_k_m_two_block"])
def test_vec_dot_f32_kats(oracle, kats, name):
    k = kats[name]
    w = _u8(k["block_hex"])
    out = oracle.vec_dot_f32(k["quant"], w, k["rows"], k["cols"], np.array(k["input"], np.float32))
    assert np.allclose(out, k["expected"], atol=k["abs_tol"], rtol=0), (name, out)
    if name == "q6_k_vec_dot_f32":
        assert np.all(oracle.dequantize_block(14, w) == -30.0)
    if name == "q4_0_vec_dot_f32":
        d = oracle.dequantize_block(2, w)
        assert np.all(d[:16] == 1.0) and np.all(d[16:] == -1.5)
    if name == "q4_k_m_two_block":  # lib.rs:1393-1395
        assert out[0] > 0.0 and out[1] > out[0]


def test_zero_scale_block_dequantizes_to_zero(oracle):
    """quant.rs:2614-2618: all-zero Q8_0 block (d = 0) dequantizes to 0."""
    assert np.all(oracle.dequantize_block(8, np.zeros(34, np.uint8)) == 0.0)


def test_tq_trit_kats(oracle, kats):
    for c in kats["tq1_0_trits"]["cases"]:
        blk = np.full(54, c["fill"], np.uint8)
        blk[0:2] = [0x00, 0x3C]
        blk[53] = c["last"]
        assert np.all(oracle.dequantize_block(34, blk) == c["value"])
    for c in kats["tq2_0_trits"]["cases"]:
        blk = np.full(66, c["fill"], np.uint8)
        blk[0:2] = [0x00, 0x3C]
        assert np.all(oracle.dequantize_block(35, blk) == c["value"])
    # out-of-range base-3 bytes stay in {-1, 0, 1} (bitnet.rs:544-556)
    for bad in range(243, 256):
        blk = np.full(54, bad, np.uint8)
        blk[0:2] = [0x00, 0x3C]
        assert set(np.unique(oracle.dequantize_block(34, blk))) <= {-1.0, 0.0, 1.0}


def test_exhaustive_tq1_0_base3_decode(oracle):
    """tests/empirical_challenge_m3_bitlinear.rs:65-135 (scale 1.0, one byte set at a time)."""
    for val in range(256):
        exp = []
        b = val
        for _ in range(5):
            exp.append(b % 3 - 1)
            b //= 3
        for chunk in (0, 17, 50):
            blk = np.zeros(54, np.uint8)
            blk[0:2] = [0x00, 0x3C]
            blk[2 + chunk] = val
            out = oracle.dequantize_block(34, blk)
            assert list(out[chunk * 5:chunk * 5 + 5]) == exp
            mask = np.ones(256, bool)
            mask[chunk * 5:chunk * 5 + 5] = False
            assert np.all(out[mask] == -1.0)
        blk = np.zeros(54, np.uint8)
        blk[0:2] = [0x00, 0x3C]
        blk[53] = val
        assert oracle.dequantize_block(34, blk)[255] == val % 3 - 1


def test_exhaustive_tq2_0_2bit_decode(oracle):
    """tests/empirical_challenge_m3_bitlinear.rs:141-181 (scale 2.5)."""
    for val in range(256):
        exp = [((val >> (2 * j)) & 3) - 1 for j in range(4)]
        for idx in (0, 31, 63):
            blk = np.zeros(66, np.uint8)
            blk[0:2] = [0x00, 0x41]
            blk[2 + idx] = val
            out = oracle.dequantize_block(35, blk) / 2.5
            assert list(out[4 * idx:4 * idx + 4]) == exp
            mask = np.ones(256, bool)
            mask[4 * idx:4 * idx + 4] = False
            assert np.all(out[mask] == -1.0)


def test_f16_exhaustive(oracle):
    """tests/wave1_rope_swiglu_fidelity.rs:186-246: every f16 bit pattern; finite values match
    IEEE bit for bit, non-finite ones decode to Inf/NaN and clamp to +0.0 in the finite form."""
    L = oracle.lib()
    bits = np.arange(65536, dtype=np.uint16)
    ieee = np.array([L.or_f16_to_f32_ieee(int(b)) for b in bits], np.float32)
    fin = np.array([L.or_f16_to_f32_finite(int(b)) for b in bits], np.float32)
    np_ref = bits.view(np.float16).astype(np.float32)
    finite = np.isfinite(np_ref)
    assert np.array_equal(ieee[finite].view(np.uint32), np_ref[finite].view(np.uint32))
    assert np.array_equal(fin[finite].view(np.uint32), np_ref[finite].view(np.uint32))
    assert np.all(fin[~finite].view(np.uint32) == 0)
    inf = np.isinf(np_ref)
    assert np.all(np.isinf(ieee[inf])) and np.all(np.isnan(ieee[np.isnan(np_ref)]))


def test_q8_quantizer_sanitization(oracle):
    """src/quant_q8.rs:3414-3482 restated on the oracle."""
    with pytest.raises(ValueError):
        oracle.quantize_row_q8_0(np.zeros(31, np.float32))
    x96 = R.test_f32_row(96, 1)
    x96[3] = np.nan
    x96[11] = -np.nan
    x96[32 + 7] = np.inf
    x96[32 + 19] = -np.inf
    x96[64:96] = np.nan
    x96[64] = np.inf
    x96[95] = 0.0
    q = oracle.quantize_row_q8_0(x96)
    assert q[0]["d"] > 0 and q[0]["qs"][3] == 0 and q[0]["qs"][11] == 0
    assert np.any(q[0]["qs"] != 0)
    assert q[1]["d"] > 0 and q[1]["qs"][7] == 0 and q[1]["qs"][19] == 0
    assert q[2]["d"] == 0 and np.all(q[2]["qs"] == 0)
    x768 = R.test_f32_row(768, 2)
    x768[3] = np.nan
    x768[16 + 9] = -np.nan
    x768[256 + 5] = -np.inf
    x768[256 + 37] = np.inf
    x768[512:768] = np.nan
    x768[512] = -np.inf
    k = oracle.quantize_row_q8_k(x768)
    assert k[0]["d"] > 0 and k[0]["qs"][3] == 0 and k[0]["qs"][25] == 0
    assert k[1]["d"] > 0 and k[1]["qs"][5] == 0 and k[1]["qs"][37] == 0
    assert k[2]["d"] == 0 and np.all(k[2]["qs"] == 0) and np.all(k[2]["bsums"] == 0)
    for blk in k:
        assert np.array_equal(blk["bsums"], blk["qs"].reshape(16, 16).astype(np.int32).sum(1))


def _subln_input(spec, n):
    if spec == "zeros":
        return np.zeros(n, np.float32)
    if spec == "ones":
        return np.ones(n, np.float32)
    if spec == "iota1":
        return np.arange(1, n + 1, dtype=np.float32)
    if spec.startswith("const:"):
        return np.full(n, float(spec[6:]), np.float32)
    if spec.startswith("alt:"):
        v = float(spec[4:])
        return np.array([v if i % 2 == 0 else -v for i in range(n)], np.float32)
    if spec.startswith("alt_w:"):
        _, a, b = spec.split(":")
        return np.array([float(a) if i % 2 == 0 else float(b) for i in range(n)], np.float32)
    if spec == "ones_nan13":
        x = np.ones(n, np.float32)
        x[13] = np.nan
        return x
    if spec == "ones_inf42":
        x = np.ones(n, np.float32)
        x[42] = np.inf
        return x
    raise ValueError(spec)


def subln_case_check(case, q, scale):
    if "scale" in case:
        assert scale == np.float32(case["scale"]), (case["name"], scale)
    if "scale_approx" in case:
        assert abs(scale - case["scale_approx"]) < 1e-5, (case["name"], scale)
    if "q" in case:
        assert np.all(q == case["q"]), case["name"]
    if "q_even" in case:
        assert np.all(q[0::2] == case["q_even"]) and np.all(q[1::2] == case["q_odd"]), case["name"]


def test_subln_kats(oracle, kats):
    s = kats["subln"]
    for c in s["cases"]:
        x = _subln_input(c["input"], s["len"])
        w = _subln_input(c["weight"], s["len"])
        q, scale = oracle.subln_quantize_absmax_i8(x, w, s["eps"])
        subln_case_check(c, q, scale)
    with pytest.raises(ValueError):
        oracle.subln_quantize_absmax_i8(np.zeros(0, np.float32), np.zeros(0, np.float32), 1e-5)


@pytest.mark.parametrize("k", [128, 896, 2048])
def test_wave4_q4_0_q8_0_gemv_cosine(oracle, k):
    """tests/wave4_quant_gemv_and_argmax.rs:254-348 (Q4_0, Q8_0) on the oracle."""
    x = R.gen_activation(k, 100 + k)
    xq = oracle.quantize_row_q8_0(x)
    for n in (1, 3, 4, 17):
        for quant, fill, seed in ((2, R.fill_q4_0_bytes, 200), (8, R.fill_q8_0_bytes, 400)):
            w = fill(n, k, seed + k + n)
            o = oracle.gemv(quant, w, n, k, xq)
            o_mt = oracle.gemv_mt(quant, w, n, k, xq, 3)
            assert np.array_equal(np.abs(o), np.abs(o_mt))  # gemv == gemv_4x up to -0.0
            of32 = oracle.vec_dot_f32(quant, w, n, k, x)
            ref = R.ref_matvec(oracle, quant, w, n, k, x)
            if n == 1:
                assert abs(o[0] - ref[0]) <= abs(ref[0]) * 0.03 + 0.25
            else:
                assert R.cosine(o, of32) > 0.9995 and R.cosine(o, ref) > 0.9995


@pytest.mark.parametrize("k", [256, 1536, 2048, 3584, 5120])
def test_wave4_k_quants_ternary_rel_err(oracle, k):
    """tests/wave4_quant_gemv_and_argmax.rs:361-542: l2_rel_err(gemv, f64 over the Q8_K-
    dequantized input) < 1e-5 and cosine > 0.999 against the f64 product on the f32 input."""
    rows = 5
    x = R.gen_activation(k, 700 + k)
    xq = oracle.quantize_row_q8_k(x)
    xd = R.dequant_q8(xq)
    for quant, fill, seed in ((12, R.fill_q4_k_m_bytes, 11), (14, R.fill_q6_k_bytes, 33),
                              (34, R.fill_tq1_0_bytes, 44), (35, R.fill_tq2_0_bytes, 55)):
        w = fill(rows, k, seed + k)
        o = oracle.gemv(quant, w, rows, k, xq)
        r = R.ref_matvec(oracle, quant, w, rows, k, x)
        rq = R.ref_matvec(oracle, quant, w, rows, k, xd)
        assert R.cosine(o, r) > 0.999, (quant, k)
        assert R.l2_rel_err(o, rq) < 1e-5, (quant, k, R.l2_rel_err(o, rq))
        assert R.l2_rel_err(o, r) < 1.5e-2, (quant, k)
        if quant in (12, 14):
            of32 = oracle.vec_dot_f32(quant, w, rows, k, x)
            assert R.cosine(of32, r) > 0.999


def test_golden_fixtures_match_live_oracle(oracle):
    """The committed oracle fixtures are reproduced bit for bit by the current oracle."""
    f = np.load(os.path.join(GOLDEN, "oracle_fixtures.npz"))
    names = sorted({k.split("__")[0] for k in f.files if k.endswith("__meta")})
    assert len(names) >= 9
    for name in names:
        q, rows, cols = (int(v) for v in f[f"{name}__meta"])
        w = f[f"{name}__w"]
        dt = oracle.BLOCK_Q8_K if oracle.ACT_IS_Q8K[q] else oracle.BLOCK_Q8_0
        xq = oracle.quantize_act(q, f[f"{name}__x"])
        assert np.array_equal(xq.view(np.uint8).reshape(-1), f[f"{name}__xq"])
        sumi, summins, contrib = oracle.block_dots(q, w, rows, cols, f[f"{name}__xq"].view(dt))
        assert np.array_equal(sumi, f[f"{name}__sumi"])
        assert np.array_equal(summins, f[f"{name}__summins"])
        assert np.array_equal(contrib.view(np.uint32), f[f"{name}__contrib"].view(np.uint32))
        y = oracle.gemv(q, w, rows, cols, xq)
        assert np.array_equal(y.view(np.uint32), f[f"{name}__y"].view(np.uint32))


def test_bitlinear_tq1_tq2_same_trits_bit_identical(oracle):
    """tests/empirical_challenge_m3_bitnet.rs:414-505: the same ternary matrix packed as TQ1_0
    and TQ2_0 gives bit-identical BitLinear outputs."""
    rows, cols = 37, 1024
    t = oracle.ternary(rows * cols, 7)
    w1 = oracle.pack_ternary(34, t, rows, cols, 0.03125)
    w2 = oracle.pack_ternary(35, t, rows, cols, 0.03125)
    act = oracle.ternary(cols, 9) * 40
    o1 = oracle.bitlinear_i8(34, w1, rows, cols, act.astype(np.int8), 0.0123)
    o2 = oracle.bitlinear_i8(35, w2, rows, cols, act.astype(np.int8), 0.0123)
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
    with pytest.raises(ValueError):
        oracle.bitlinear_i8(12, np.zeros(144, np.uint8), 1, 256, np.zeros(256, np.int8), 1.0)


def test_relu_squared_gate_oracle(oracle):
    """lib.rs:1130-1137: (relu * relu) * up with relu = g > 0 ? g : 0, each product rounded to
    f32; NaN and -0 gates give +0, so the product's sign is the sign of up."""
    rng = np.random.default_rng(3)
    g = rng.normal(0, 3, 4099).astype(np.float32)
    u = rng.normal(0, 3, 4099).astype(np.float32)
    g[:6] = [np.nan, -0.0, 0.0, np.inf, -np.inf, 1e20]
    u[:6] = [-1.0, -2.0, 3.0, 2.0, 5.0, 1.0]
    got = oracle.relu_squared_gate_f32(g, u)
    r = np.where(g > 0, g, np.float32(0)).astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        want = ((r * r).astype(np.float32) * u).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert got[0] == 0 and np.signbit(got[0]) and np.signbit(got[1])
    assert got[3] == np.inf and got[4] == 0 and got[5] == np.inf
    with pytest.raises(ValueError, match="dimension mismatch"):
        oracle.relu_squared_gate_f32(g, u[:-1])


def test_bitnet_chain_reference_scenarios(oracle):
    """tests/empirical_challenge_m3_bitnet.rs:582-686 on the oracle: the reference's synthetic
    weights (gate = up = all +1 at scale 1; down TQ1_0 bytes 0x55) and its three inputs. The
    reference asserts finite outputs; the weights also fix the values in closed form: every
    gate / up output is sum(act1) * scale1, every intermediate element equals the same h, act2
    is +-127 (or 0), and each down row is two TQ1_0 blocks with 102 trits of -1 each."""
    hidden, inter, eps = 256, 512, 1e-5
    wg, wd = R.bitnet_chain_weights(hidden, inter)
    n1, n2 = np.ones(hidden, np.float32), np.ones(inter, np.float32)
    deq = oracle.dequantize_rows(34, wd, hidden, inter)
    assert np.all(deq.reshape(hidden, 2, 256).astype(np.int32).sum(axis=2) == -102)
    for name, x in R.bitnet_chain_scenarios(hidden):
        r = oracle.bitnet_ffn(x, n1, n2, eps, 35, wg, 35, wg, 34, wd, hidden, inter)
        assert np.all(np.isfinite(r["out"])), name
        g0 = np.float32(np.float32(r["act1"].astype(np.int32).sum()) * np.float32(r["scale1"]))
        assert np.all(r["gate"] == g0) and np.array_equal(r["gate"], r["up"]), name
        assert np.all(r["relu"] == np.float32(np.float32(max(g0, 0) * max(g0, 0)) * g0)), name
        if name == "all_zeros":
            assert not r["act1"].any() and r["scale1"] == np.float32(1) / np.float32(127)
        if r["relu"][0] > 0:
            assert np.all(r["act2"] == 127)
            v = np.float32(-102 * 127) * np.float32(r["scale2"])
            assert np.all(r["out"] == np.float32(np.float32(0) + v) + v), name
        else:
            assert not r["act2"].any() and not r["out"].any(), name


@pytest.mark.parametrize("quant", [2, 8, 12, 14, 35, 36])
def test_repack_lossless_and_gemm_rows_stitch(oracle, quant):
    """tests/test_repack_gemv_gemm.rs:619-700 (repacked values reproduce the dequantizer) and
    :805-826 (row-slice outputs stitch to the full GEMM)."""
    rows, cols = 19, 512
    if quant in (35, 36):
        w = oracle.pack_ternary(quant, oracle.ternary(rows * cols, 3), rows, cols, 0.02)
    else:
        w = oracle.quantize_weights(quant, oracle.normal(rows * cols, 5, 0.02), rows, cols)
    q, s, mn = oracle.repack_block_scaled(quant, w, rows, cols)
    g = 16 if quant == 14 else 32
    deq = q.astype(np.float32).reshape(rows, -1, g) * s[:, :, None]
    if mn is not None:
        deq = deq - mn[:, :, None]
    assert np.allclose(deq.reshape(rows, -1), oracle.dequantize_rows(quant, w, rows, cols),
                       rtol=1e-6, atol=1e-7)
    m = 5
    act = oracle.normal(m * cols, 11, 1.0)
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(act, m, cols)
    full = oracle.gemm_repacked(quant, q, s, mn, rows, cols, xq, xs, xsum, xs16, m, nthreads=2)
    parts = [oracle.gemm_repacked(quant, q, s, mn, rows, cols, xq, xs, xsum, xs16, m, a, b)
             for a, b in ((0, 7), (7, 8), (8, 19))]
    assert np.array_equal(np.concatenate(parts, axis=1), full)
    ref = oracle.dequantize_rows(quant, w, rows, cols).astype(np.float64) @ \
        act.reshape(m, cols).astype(np.float64).T
    assert R.cosine(full.reshape(-1), ref.T.reshape(-1)) > 0.9995


# ---------------------------------------------------------------- compact nibble matrices

def test_q4_1_iq4_nl_dequant_kats(oracle, kats):
    """quant.rs:2836-2853 (Q4_1, including a zero d with a non-zero min) and :2895-2905
    (IQ4_NL code book)."""
    for c in kats["q4_1_dequant"]["cases"]:
        d = oracle.dequantize_block(oracle.Q4_1, _u8(c["block_hex"]))
        assert np.allclose(d[:16], c["lo"], atol=1e-6) and np.allclose(d[16:], c["hi"], atol=1e-6)
    k = kats["iq4_nl_dequant"]
    d = oracle.dequantize_block(oracle.IQ4_NL, _u8(k["block_hex"]))
    for idx, v in k["expect"].items():
        assert abs(d[int(idx)] - v) < 1e-6, (idx, d[int(idx)])


def _q4_0_kat_tensor(rows, cols):
    """repack.rs:5902-5918: Q4_0 d = 0.5 and an index-derived nibble pattern."""
    nb = cols // 32
    raw = np.zeros((rows, nb, 18), np.uint8)
    raw[..., 0:2] = [0x00, 0x38]
    r = np.arange(rows)[:, None, None]
    b = np.arange(nb)[None, :, None]
    i = np.arange(16)[None, None, :]
    raw[..., 2:] = (((r + i + b * 3) & 0x0F) | (((r * 3 + i + 5) & 0x0F) << 4)).astype(np.uint8)
    return raw.reshape(-1)


def test_nibble_q4_0_footprint_dequant_and_gemm_kat(oracle):
    """repack.rs:5899-5988 (wave3_packed_nibble_footprint_and_gemm_parity): the tile layout is
    exactly the GGUF size, dequantize_row reproduces the Q4_0 dequantizer, and the nibble GEMM
    tracks the f32 dot product of the dequantized row and the activation."""
    rows, cols, m = 16, 64, 4
    raw = _q4_0_kat_tensor(rows, cols)
    tiles, sc, mn, hd = oracle.nibble_pack_tiles(oracle.Q4_0, raw, rows, cols)
    assert tiles.nbytes + sc.nbytes == raw.nbytes
    q, ws, wm = oracle.nibble_decode_tiles(oracle.Q4_0, rows, cols, tiles, sc, mn, hd)
    deq = oracle.dequantize_rows(oracle.Q4_0, raw, rows, cols).reshape(rows, cols)
    for r in range(rows):
        row = oracle.nibble_dequantize_row(oracle.Q4_0, q, ws, wm, cols, r)
        assert np.array_equal(row, deq[r])
    x = ((np.arange(m * cols) % 19).astype(np.float32) - 9.0) * 0.25
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(x, m, cols)
    out = oracle.gemm_nibble(oracle.Q4_0, q, ws, wm, rows, cols, xq, xs, xsum, m)
    ref = x.reshape(m, cols) @ deq.T
    assert np.all(np.abs(out - ref) < 0.05 * np.maximum(np.abs(ref), 1.0) + 0.25)
    rq, rs, rm = oracle.repack_block_scaled(oracle.Q4_0, raw, rows, cols)
    rep = oracle.gemm_repacked(oracle.Q4_0, rq, rs, rm, rows, cols, xq, xs, xsum, xs16, m)
    assert np.all(np.abs(out - rep) < 1e-4)


@pytest.mark.parametrize("quant", [2, 3, 20, 12])
def test_nibble_all_formats_match_repacked(oracle, quant):
    """tests/wave3_prefill_gqa_and_gemm.rs:233-279: every nibble format (Q4_0, Q4_1, IQ4_NL,
    Q4_K_M) at [256, 512] on the suite's pseudo-quant tensors: the tile layout is exactly the
    GGUF size and the nibble GEMM equals the repacked GEMM (the suite allows 1e-4; the
    arithmetic is identical, so the oracle's two paths agree bit for bit)."""
    rows, cols, m = 256, 512, 17
    raw = R.fill_pseudo_quant_tensor(quant, rows, cols)
    tiles, sc, mn, hd = oracle.nibble_pack_tiles(quant, raw, rows, cols)
    meta = sum(a.nbytes for a in (sc, mn, hd) if a is not None)
    assert tiles.nbytes + meta == raw.nbytes
    q, ws, wm = oracle.nibble_decode_tiles(quant, rows, cols, tiles, sc, mn, hd)
    x = np.float32(0.5) + R.small_f32(np.arange(m * cols), 13, 5.0, 0.25)
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(x, m, cols)
    out = oracle.gemm_nibble(quant, q, ws, wm, rows, cols, xq, xs, xsum, m, nthreads=4)
    rq, rs, rm = oracle.repack_block_scaled(quant, raw, rows, cols)
    rep = oracle.gemm_repacked(quant, rq, rs, rm, rows, cols, xq, xs, xsum, xs16, m, nthreads=4)
    assert np.all(np.abs(out - rep) < 1e-4)
    assert np.array_equal(out.view(np.uint32), rep.view(np.uint32))
    # the decoded nibble matrix reproduces the block dequantizer row by row
    deq = oracle.dequantize_rows(quant, raw, rows, cols).reshape(rows, cols)
    for r in (0, 7, 8, 255):
        assert np.array_equal(oracle.nibble_dequantize_row(quant, q, ws, wm, cols, r), deq[r])


def test_nibble_unaligned_rows_footprint(oracle):
    """tests/wave3_prefill_gqa_and_gemm.rs:270-278: 203 Q4_K_M rows (tiles of 8 rows pad to
    208) stay within 1.05x of the GGUF bytes."""
    rows, cols = 203, 512
    raw = R.fill_pseudo_quant_tensor(12, rows, cols)
    tiles, _, _, hd = oracle.nibble_pack_tiles(12, raw, rows, cols)
    assert (tiles.nbytes + hd.nbytes) * 100 <= raw.nbytes * 105


def test_nibble_zero_scale_blocks(oracle):
    """repack.rs:4458-4500: Q4_0 / IQ4_NL blocks whose scale decodes to zero (0, NaN, Inf) keep
    zero scale bits and zero nibbles in the tiles; they contribute nothing to the GEMM."""
    rows, cols = 9, 64
    for quant in (2, 20):
        raw = R.fill_pseudo_quant_tensor(quant, rows, cols).reshape(rows, 2, 18).copy()
        raw[1, 0, 0:2] = [0x00, 0x7C]  # +Inf
        raw[4, 1, 0:2] = [0x01, 0x7E]  # NaN
        raw[8, 0, 0:2] = [0x00, 0x00]  # 0
        raw = raw.reshape(-1)
        tiles, sc, _, _ = oracle.nibble_pack_tiles(quant, raw, rows, cols)
        assert sc.reshape(2, 2, 8)[0, 0, 1] == 0 and sc.reshape(2, 2, 8)[0, 1, 4] == 0
        assert sc.reshape(2, 2, 8)[1, 0, 0] == 0
        q, ws, wm = oracle.nibble_decode_tiles(quant, rows, cols, tiles, sc, None, None)
        zero = oracle.Q4_0 == quant and -8 or -127
        assert np.all(q[1, 0:32] == zero) and np.all(q[4, 32:64] == zero)
        assert ws[1, 0] == 0.0 and ws[4, 1] == 0.0 and ws[8, 0] == 0.0
        deq = oracle.dequantize_rows(quant, raw, rows, cols).reshape(rows, cols)
        assert np.all(deq[1, 0:32] == 0.0)


def test_nibble_golden_fixtures_match_live_oracle(oracle):
    """The committed nibble GEMM fixtures (Q4_1, IQ4_NL) are reproduced bit for bit."""
    f = np.load(os.path.join(GOLDEN, "oracle_fixtures.npz"))
    names = sorted({k.split("__")[0] for k in f.files if k.endswith("__nmeta")})
    assert len(names) == 2
    for name in names:
        q, rows, cols, m = (int(v) for v in f[f"{name}__nmeta"])
        xq, xs, xsum, _, _ = oracle.act_q8_quantize(f[f"{name}__x"], m, cols)
        nq, ws, wm = oracle.nibble_decode(q, f[f"{name}__w"], rows, cols)
        out = oracle.gemm_nibble(q, nq, ws, wm, rows, cols, xq, xs, xsum, m)
        assert np.array_equal(out.view(np.uint32), f[f"{name}__out"].view(np.uint32))


# ---------------------------------------------------------------- Q5_0 / Q5_K

def test_q5_k_kat_4928(oracle, kats):
    """quant.rs:2665-2697: the Q5_K block dequantizes to values summing to 4928, and the f32
    matvec with ones returns 4928."""
    k = kats["q5_k_dequant_sum"]
    w = _u8(k["block_hex"])
    assert abs(float(oracle.dequantize_block(oracle.Q5_K, w).astype(np.float64).sum()) - 4928.0) < 1e-3
    out = oracle.vec_dot_f32(oracle.Q5_K, w, 1, 256, np.ones(256, np.float32))
    assert abs(out[0] - 4928.0) < 1e-3


def test_q5_0_kats(oracle, kats):
    """quant.rs:2855-2862 (block dequantization) and :2910-2966 (a two-block row through the f32
    path and through Q8_0 activations, both within 1e-4 of the dequantized f32 dot)."""
    k = kats["q5_0_dequant"]
    d = oracle.dequantize_block(oracle.Q5_0, _u8(k["block_hex"]))
    for idx, v in k["expect"].items():
        assert abs(d[int(idx)] - v) < 1e-6
    k = kats["q5_0_two_block_row"]
    row = _u8(k["row_hex"])
    deq = oracle.dequantize_rows(oracle.Q5_0, row, 1, 64).reshape(-1)
    x = (np.arange(64, dtype=np.float32) - 31.0) * np.float32(0.0625)
    ref = float(np.float32(sum(np.float32(a) * np.float32(b) for a, b in zip(deq, x))))
    got = oracle.vec_dot_f32(oracle.Q5_0, row, 1, 64, x)[0]
    assert abs(got - ref) < k["abs_tol"]
    q8 = np.zeros(2, oracle.BLOCK_Q8_0)
    q8["d"] = 1.0
    q8["qs"] = (np.arange(64) - 31).reshape(2, 32)
    exact = float(np.dot(deq.astype(np.float64), (np.arange(64) - 31).astype(np.float64)))
    assert abs(oracle.vec_dot(oracle.Q5_0, row, q8) - exact) < k["abs_tol"]


@pytest.mark.parametrize("quant", [6, 13])
def test_q5_gemv_tolerance_and_repack(oracle, quant):
    """The Q5 GEMVs meet the suite's l2 contract against the f64 product over the dequantized
    blocks, and their repacked form reproduces the dequantizer (tests/test_repack_gemv_gemm.rs:
    619-700)."""
    rows, cols = 33, 1024
    w = oracle.quantize_weights(quant, oracle.normal(rows * cols, 8, 0.02), rows, cols)
    x = oracle.normal(cols, 9, 1.0)
    xq = oracle.quantize_act(quant, x)
    o = oracle.gemv(quant, w, rows, cols, xq)
    rq = R.ref_matvec(oracle, quant, w, rows, cols, R.dequant_q8(xq))
    assert R.l2_rel_err(o, rq) < 1e-5
    assert R.cosine(o, R.ref_matvec(oracle, quant, w, rows, cols, x)) > 0.999
    q, s, mn = oracle.repack_block_scaled(quant, w, rows, cols)
    deq = q.astype(np.float32).reshape(rows, -1, 32) * s[:, :, None]
    if mn is not None:
        deq = deq - mn[:, :, None]
    assert np.allclose(deq.reshape(rows, -1), oracle.dequantize_rows(quant, w, rows, cols),
                       rtol=1e-6, atol=1e-7)


def test_q5_1_q2_k_q3_k_dequant_kats(oracle, kats):
    """quant.rs:2864-2893: Q5_1 (high bits from qh), Q2_K (sub-block scale and min), Q3_K
    (6-bit scale 33 split over the scale bytes, cleared hmask bit subtracts 4)."""
    for key, quant in (("q5_1_dequant", oracle.Q5_1), ("q2_k_dequant", oracle.Q2_K),
                       ("q3_k_dequant", oracle.Q3_K)):
        k = kats[key]
        d = oracle.dequantize_block(quant, _u8(k["block_hex"]))
        for idx, v in k["expect"].items():
            assert abs(d[int(idx)] - v) < 1e-6, (key, idx, d[int(idx)])


WAVE2 = [(3, 256, 19, 1.5e-2), (6, 256, 21, 1.2e-2), (7, 256, 17, 1.5e-2), (10, 512, 15, 2.0e-2),
         (11, 512, 19, 1.5e-2), (20, 256, 23, 1.5e-2), (36, 256, 17, 1.5e-2)]


@pytest.mark.parametrize("q_idx", range(len(WAVE2)))
def test_wave2_repack_gemm_contract(oracle, q_idx):
    """tests/test_repack_gemv_gemm.rs:919-997 on the oracle, with the test's own synthetic
    tensors and activations: the repacked weight's rows (scale * q - min, repack.rs:2529-2598)
    within 1e-4 of the block dequantizers, and the repacked GEMM over Q8 activations against the
    f32 product: cosine > 0.999 and relative l2 error below the test's per-format bound, for
    M in {1, 5, 8, 17, 64}."""
    quant, cols, rows, max_rel = WAVE2[q_idx]
    raw = R.build_synthetic_quant_tensor(quant, rows, cols, q_idx + 17)
    q, s, mn = oracle.repack_block_scaled(quant, raw, rows, cols)
    gsz = q.shape[1] // s.shape[1]
    deq = oracle.dequantize_rows(quant, raw, rows, cols)
    rep = np.repeat(s, gsz, axis=1) * q.astype(np.float32)
    if mn is not None:
        rep = rep - np.repeat(mn, gsz, axis=1)
    assert np.all(np.abs(rep[:, :cols] - deq) < 1e-4)
    for m in (1, 5, 8, 17, 64):
        x = R.make_activations(m, cols, 300 + q_idx * 10 + m)
        xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(x, m, cols)
        got = oracle.gemm_repacked(quant, q, s, mn, rows, cols, xq, xs, xsum, xs16, m)
        want = x.reshape(m, cols).astype(np.float64) @ deq.astype(np.float64).T
        cos, rel = R.cosine_and_rel_l2(got, want)
        assert cos > 0.999 and rel < max_rel, (quant, m, cos, rel)
