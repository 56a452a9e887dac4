"""Input generators and metrics restated from the jero-kernels-rvv test suite.

These are test data generators (not arithmetic under test); each cites the Rust test it
restates so the parity tests here can apply the same properties as the crate's own tests.
"""
import numpy as np

MASK64 = (1 << 64) - 1
LCG_A = 6364136223846793005
LCG_C = 1442695040888963407


def lcg_seq(seed: int, n: int) -> np.ndarray:
    """Successive states of lcg_next (tests/wave4_quant_gemv_and_argmax.rs:31-36):
    s = s * 6364136223846793005 + 1442695040888963407 (mod 2^64), returned after each step.
    Vectorised by leapfrogging blocks of B steps."""
    B = 4096
    first = np.empty(min(n, B), np.uint64)
    s = seed & MASK64
    for i in range(first.size):
        s = (s * LCG_A + LCG_C) & MASK64
        first[i] = s
    if n <= B:
        return first
    # s_{k+B} = A s_k + C with A = a^B, C = c (a^{B-1} + ... + 1)
    A, Cc = 1, 0
    for _ in range(B):
        A, Cc = (A * LCG_A) & MASK64, (Cc * LCG_A + LCG_C) & MASK64
    out = np.empty(((n + B - 1) // B) * B, np.uint64)
    out[:B] = first
    A64, C64 = np.uint64(A), np.uint64(Cc)
    with np.errstate(over="ignore"):
        for k in range(1, out.size // B):
            out[k * B:(k + 1) * B] = out[(k - 1) * B:k * B] * A64 + C64
    return out[:n]


def gen_activation(n: int, seed: int) -> np.ndarray:
    """tests/wave4_quant_gemv_and_argmax.rs:38-48."""
    s = lcg_seq(seed, n)
    r = ((s >> np.uint64(32)).astype(np.uint32)).astype(np.float32) / np.float32(4294967295.0)
    i = np.arange(n, dtype=np.float32)
    return ((r - np.float32(0.35)) * np.float32(1.4) +
            np.sin(i * np.float32(0.013)).astype(np.float32) * np.float32(0.2)).astype(np.float32)


def test_f32_row(n: int, seed: int) -> np.ndarray:
    """src/quant_q8.rs:3388-3395."""
    i = np.arange(n)
    return ((((i * 37 + seed * 13) % 29) - 14) * 0.125).astype(np.float32)


def _hi32(s):
    return (s >> np.uint64(32))


def fill_q4_0_bytes(rows, cols, seed):
    """tests/wave4_quant_gemv_and_argmax.rs:77-96."""
    nb = cols // 32
    s = lcg_seq(seed, rows * nb * 32).reshape(rows, nb, 16, 2)
    lo = (_hi32(s[..., 0]) % np.uint64(16)).astype(np.uint8)
    hi = ((s[..., 1] >> np.uint64(40)) % np.uint64(16)).astype(np.uint8)
    scales = np.array([0x3000, 0x3200, 0x3400, 0x3600], np.uint16)
    r = np.arange(rows)[:, None]
    b = np.arange(nb)[None, :]
    sc = scales[(r + b) % 4]
    out = np.zeros((rows, nb, 18), np.uint8)
    out[..., 0:2] = sc[..., None].view(np.uint8).reshape(rows, nb, 2)
    out[..., 2:] = (hi << 4) | lo
    return out.reshape(-1)


def fill_q8_0_bytes(rows, cols, seed):
    """tests/wave4_quant_gemv_and_argmax.rs:118-135."""
    nb = cols // 32
    s = lcg_seq(seed, rows * nb * 32).reshape(rows, nb, 32)
    q = ((_hi32(s) % np.uint64(127)).astype(np.int16) - 63).astype(np.int8)
    scales = np.array([0x2800, 0x2C00, 0x3000, 0x3200], np.uint16)
    r = np.arange(rows)[:, None]
    b = np.arange(nb)[None, :]
    sc = scales[(r + b) % 4]
    out = np.zeros((rows, nb, 34), np.uint8)
    out[..., 0:2] = sc[..., None].view(np.uint8).reshape(rows, nb, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(-1)


def fill_q4_k_m_bytes(rows, cols, seed):
    """tests/wave4_quant_gemv_and_argmax.rs:137-154."""
    nb = cols // 256
    s = lcg_seq(seed, rows * nb * 140).reshape(rows, nb, 140)
    out = np.zeros((rows, nb, 144), np.uint8)
    out[..., 0:2] = np.frombuffer(np.uint16(0x3000).tobytes(), np.uint8)
    out[..., 2:4] = np.frombuffer(np.uint16(0x2800).tobytes(), np.uint8)
    out[..., 4:16] = (_hi32(s[..., :12]) % np.uint64(31) + np.uint64(1)).astype(np.uint8)
    out[..., 16:] = (_hi32(s[..., 12:]) & np.uint64(0xFF)).astype(np.uint8)
    return out.reshape(-1)


def fill_q6_k_bytes(rows, cols, seed):
    """tests/wave4_quant_gemv_and_argmax.rs:175-192."""
    nb = cols // 256
    s = lcg_seq(seed, rows * nb * 208).reshape(rows, nb, 208)
    out = np.zeros((rows, nb, 210), np.uint8)
    out[..., 0:192] = (_hi32(s[..., :192]) & np.uint64(0xFF)).astype(np.uint8)
    out[..., 192:208] = ((_hi32(s[..., 192:]) % np.uint64(15)).astype(np.int16) - 7).astype(
        np.int8).view(np.uint8)
    out[..., 208:210] = np.frombuffer(np.uint16(0x3000).tobytes(), np.uint8)
    return out.reshape(-1)


def fill_tq1_0_bytes(rows, cols, seed):
    """tests/wave4_quant_gemv_and_argmax.rs:194-209."""
    nb = cols // 256
    s = lcg_seq(seed, rows * nb * 52).reshape(rows, nb, 52)
    out = np.zeros((rows, nb, 54), np.uint8)
    out[..., 0:2] = np.frombuffer(np.uint16(0x3400).tobytes(), np.uint8)
    out[..., 2:] = (_hi32(s) % np.uint64(243)).astype(np.uint8)
    return out.reshape(-1)


def fill_tq2_0_bytes(rows, cols, seed):
    """tests/wave4_quant_gemv_and_argmax.rs:211-226."""
    nb = cols // 256
    s = lcg_seq(seed, rows * nb * 64).reshape(rows, nb, 64)
    out = np.zeros((rows, nb, 66), np.uint8)
    out[..., 0:2] = np.frombuffer(np.uint16(0x3400).tobytes(), np.uint8)
    out[..., 2:] = (_hi32(s) & np.uint64(0xFF)).astype(np.uint8)
    return out.reshape(-1)


def cosine(a, b) -> float:
    """tests/wave4_quant_gemv_and_argmax.rs:50-65 (f64 accumulation)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / (np.sqrt(a @ a) * np.sqrt(b @ b)))


def l2_rel_err(got, ref) -> float:
    """tests/wave4_quant_gemv_and_argmax.rs:67-75."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(((got - ref) ** 2).sum()) / np.sqrt((ref ** 2).sum()))


def ref_matvec(oracle, quant, w, rows, cols, x) -> np.ndarray:
    """ref_matvec_blocks (tests/wave4_quant_gemv_and_argmax.rs:228-251): f64 sum over the
    dequantized blocks (the dequantizers are the oracle's restatement of quant.rs/lib.rs)."""
    deq = oracle.dequantize_rows(quant, w, rows, cols).astype(np.float64)
    return (deq @ np.asarray(x, np.float64)).astype(np.float32)


def dequant_q8(xq) -> np.ndarray:
    """dequantize_q8_k_row (tests/wave4_quant_gemv_and_argmax.rs:350-358) and its Q8_0 twin."""
    return (xq["qs"].astype(np.float32) * xq["d"][:, None]).reshape(-1)


def gemv_tolerance_ok(got, oracle_out, contrib, rel=1e-5):
    """f32 outputs: the GPU sums a row's (bit-exact) block values in a different order than
    the reference's sequential loop, so each output may differ by rounding only. Bound per
    element: |got - ref| <= rel * sum_b |block value_b| (+ the smallest normal), and the
    vector-level l2 relative error must stay under rel."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(oracle_out, np.float64)
    bound = rel * np.abs(np.asarray(contrib, np.float64)).sum(axis=-1) + 1.2e-38
    ok = np.abs(got - ref) <= bound
    return bool(ok.all()), float(np.max(np.abs(got - ref) / bound))


def small_f32(i, modulo, offset, scale):
    """tests/wave3_prefill_gqa_and_gemm.rs:17-20, vectorised over an index array."""
    return ((np.asarray(i) % modulo).astype(np.float32) - np.float32(offset)) * np.float32(scale)


def fill_pseudo_quant_tensor(quant, rows, cols):
    """tests/wave3_prefill_gqa_and_gemm.rs:22-100 (the nibble formats and Q8_0): block b of the
    flattened tensor gets fixed scale bits and index-derived payload bytes."""
    be, bb = {2: (32, 18), 20: (32, 18), 3: (32, 20), 12: (256, 144), 8: (32, 34)}[quant]
    nblk = rows * cols // be
    b = np.arange(nblk)[:, None]
    out = np.zeros((nblk, bb), np.uint8)
    if quant == 8:
        out[:, 0:2] = [0x00, 0x34]
        k = np.arange(32)[None, :]
        out[:, 2:] = (((b * 7 + k * 5) % 21) - 10).astype(np.int8).view(np.uint8)
    elif quant in (2, 20):
        out[:, 0:2] = [0x00, 0x38]
        k = np.arange(16)[None, :]
        out[:, 2:] = (((b + k * 3) & 0x0F) | (((b * 3 + k * 5 + 1) & 0x0F) << 4)).astype(np.uint8)
    elif quant == 3:
        out[:, 0:2] = [0x00, 0x38]
        out[:, 2:4] = [0x00, 0x34]
        k = np.arange(16)[None, :]
        out[:, 4:] = (((b + k * 3) & 0x0F) | (((b * 5 + k + 2) & 0x0F) << 4)).astype(np.uint8)
    else:
        out[:, 0:2] = [0x00, 0x34]
        out[:, 2:4] = [0x00, 0x30]
        k = np.arange(12)[None, :]
        out[:, 4:16] = ((b * 5 + k * 3 + 1) & 0x3F).astype(np.uint8)
        k = np.arange(128)[None, :]
        out[:, 16:] = ((b * 7 + k * 11 + 3) & 0xFF).astype(np.uint8)
    return out.reshape(-1)


def bitnet_chain_weights(hidden: int, inter: int):
    """The synthetic FFN weights of tests/empirical_challenge_m3_bitnet.rs:602-622: gate and up
    are TQ2_0 [inter, hidden] of bytes 0xAA with every block's f16 scale (bytes 0..2) 1.0, down
    is TQ1_0 [hidden, inter] of bytes 0x55 with scale 1.0. Returns (gate_up_bytes, down_bytes)."""
    gate = np.full(inter * hidden // 256 * 66, 0xAA, np.uint8).reshape(-1, 66)
    gate[:, 0:2] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)
    down = np.full(hidden * inter // 256 * 54, 0x55, np.uint8).reshape(-1, 54)
    down[:, 0:2] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)
    return gate.reshape(-1), down.reshape(-1)


def bitnet_chain_scenarios(hidden: int):
    """The three inputs of tests/empirical_challenge_m3_bitnet.rs:588-596: sin(0.05 i) * 2 (f32
    arithmetic; numpy's float32 sin stands in for Rust's), all zeros, all 1e5."""
    i = np.arange(hidden, dtype=np.float32)
    return [("normal_random", (np.sin(i * np.float32(0.05)) * np.float32(2.0)).astype(np.float32)),
            ("all_zeros", np.zeros(hidden, np.float32)),
            ("extreme_large", np.full(hidden, 1e5, np.float32))]


# ---- tests/test_repack_gemv_gemm.rs generators ----

def f16_bits_trunc(v) -> int:
    """f32_to_f16_bits of tests/test_repack_gemv_gemm.rs:31-45: the mantissa truncated (no
    rounding), exponents below the f16 range flushed to a signed zero, above it clamped to
    0x7BFF."""
    bits = int(np.float32(v).view(np.uint32))
    sign = (bits >> 16) & 0x8000
    exp = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    if exp <= 127 - 15:
        return sign
    if exp >= 127 + 16:
        return sign | 0x7BFF
    return sign | ((exp - 112) << 10) | (mant >> 13)


def make_activations(m: int, k: int, seed: int) -> np.ndarray:
    """make_activations (tests/test_repack_gemv_gemm.rs:51-63): xorshift64 states, each
    multiplied by 0x2545F4914F6CDD1D, top 24 bits as a unit float, mapped to [-1, 1)."""
    out = np.empty(m * k, np.float32)
    s = ((seed * 0x9E3779B97F4A7C15) & MASK64) | 1
    for i in range(m * k):
        s ^= s >> 12
        s ^= (s << 25) & MASK64
        s ^= s >> 27
        u = (s * 0x2545F4914F6CDD1D) & MASK64
        out[i] = np.float32(u >> 40) / np.float32(1 << 24)
    return (out * np.float32(2.0) - np.float32(1.0)).astype(np.float32)


def build_synthetic_quant_tensor(quant: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """build_synthetic_quant_tensor (tests/test_repack_gemv_gemm.rs:86-390) for the formats of
    its wave-2 test: Q4_1 (3), Q5_0 (6), Q5_1 (7), Q2_K (10), Q3_K (11), IQ4_NL (20), I2_S (36).
    Scales are f32 expressions rounded through f16_bits_trunc, as there."""
    f = np.float32
    h = lambda v: int(f16_bits_trunc(v)).to_bytes(2, "little")
    u32 = lambda v: (v & 0xFFFFFFFF).to_bytes(4, "little")
    out = bytearray()
    if quant == 36:
        nb = cols // 128
        for r in range(rows):
            for b in range(nb):
                for gp in range(32):
                    t0 = (r + gp + seed) % 3
                    t1 = (b + gp + 1 + seed) % 3
                    t2 = (r + b + gp + 2) % 3
                    t3 = (r * 3 + gp + 1) % 3
                    out.append((t0 << 6) | (t1 << 4) | (t2 << 2) | t3)
        trailer = bytearray(32)
        trailer[0:4] = np.float32(0.125).tobytes()
        return np.frombuffer(bytes(out + trailer), np.uint8).copy()
    for r in range(rows):
        for b in range(cols // (256 if quant in (10, 11) else 32)):
            if quant == 3:
                d = f(0.0625) * (f(1.0) + f((r + b) % 4) * f(0.5))
                m = f(-0.25) + f((r * 3 + b) % 5) * f(0.125)
                out += h(d) + h(m)
                out += bytes(((r * 7 + b * 3 + i + seed) & 15) |
                             (((r * 11 + b * 5 + i * 3 + seed) & 15) << 4) for i in range(16))
            elif quant == 6:
                d = f(0.0625) * (f(1.0) + f((r + b) % 4) * f(0.25))
                qh = (r * 0x9E3779B1) ^ (b * 0x85EBCA77) ^ (seed * 0x01010101)
                out += h(d) + u32(qh)
                out += bytes(((r * 5 + b * 9 + i + seed) & 15) |
                             (((r * 13 + b * 3 + i * 5 + seed) & 15) << 4) for i in range(16))
            elif quant == 7:
                d = f(0.0625) * (f(1.0) + f((r + b) % 3) * f(0.25))
                m = f(-0.25) + f((r * 2 + b * 3) % 7) * f(0.0625)
                qh = (r * 0x517CC1B7) ^ (b * 0x27220A95) ^ seed
                out += h(d) + h(m) + u32(qh)
                out += bytes(((r * 9 + b * 7 + i + seed) & 15) |
                             (((r * 3 + b * 11 + i * 7 + seed) & 15) << 4) for i in range(16))
            elif quant == 10:
                sc = [((r * 5 + b * 3 + s + 1) % 15) + 1 for s in range(16)]
                mn = [(r * 3 + b * 7 + s + 2) % 13 for s in range(16)]
                out += bytes((sc[s] & 15) | ((mn[s] & 15) << 4) for s in range(16))
                out += bytes((r * 17 + b * 11 + i * 5 + seed) & 0xFF for i in range(64))
                out += h(0.0625) + h(0.03125)
            elif quant == 11:
                out += bytes((r * 13 + b * 7 + i * 9 + seed) & 0xFF for i in range(96))
                out += bytes((r * 19 + b * 23 + s * 11 + seed + 7) & 0xFF for s in range(12))
                out += h(0.0625)
            elif quant == 20:
                d = f(0.03125) * (f(1.0) + f((r + b) % 4) * f(0.25))
                out += h(d)
                out += bytes(((r * 5 + b * 3 + i + seed) & 15) |
                             (((r * 7 + b * 9 + i * 3 + seed) & 15) << 4) for i in range(16))
            else:
                raise ValueError(f"no generator for quant {quant}")
    return np.frombuffer(bytes(out), np.uint8).copy()


def cosine_and_rel_l2(actual, reference):
    """cosine_similarity_and_rel_l2 (tests/test_repack_gemv_gemm.rs:65-84), in f64."""
    a = np.asarray(actual, np.float64).ravel()
    r = np.asarray(reference, np.float64).ravel()
    denom = max(np.linalg.norm(a) * np.linalg.norm(r), 1e-12)
    return float(a @ r / denom), float(np.linalg.norm(a - r) / max(np.linalg.norm(r), 1e-12))
