"""GPU decode GEMV / block dots vs the CPU oracle.

Contract (the north star's): per-block integer sums (sumi, and summins for Q4_K) are
bit-exact, the f32 block values (the reference's separately rounded block formula) are
bit-exact, and row outputs -- whose block values the GPU sums in a different order than the
reference's sequential loop -- stay within |err| <= 1e-5 * sum_b |block value| per element and
l2 relative error < 1e-5 (tests/wave4_quant_gemv_and_argmax.rs:397 uses the same 1e-5)."""
import os

import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import bits, dev, host, upload

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REL = 1e-5

GEMV_FN = {2: "gemv_q4_0_q8_0", 8: "gemv_q8_0_q8_0", 12: "gemv_q4_k_q8_k",
           14: "gemv_q6_k_q8_k", 34: "gemv_tq1_0_q8_k", 35: "gemv_tq2_0_q8_k",
           6: "gemv_q5_0_q8_0", 13: "gemv_q5_k_q8_k"}
VEC_DOT_FN = {2: "vec_dot_q4_0_q8_0", 8: "vec_dot_q8_0_q8_0", 12: "vec_dot_q4_k_q8_k",
              14: "vec_dot_q6_k_q8_k", 34: "vec_dot_tq1_0_q8_k", 35: "vec_dot_tq2_0_q8_k",
              6: "vec_dot_q5_0_q8_0_blocks", 13: "vec_dot_q5_k_q8_k"}


def run_gemv(jkb, quant, w, xq_bytes):
    out = torch.empty(w.rows, dtype=torch.float32, device="cuda")
    getattr(jkb, GEMV_FN[quant])(out, w, xq_bytes)
    return host(out)


def check_case(jkb, oracle, quant, wbytes, rows, cols, x, orient="rc"):
    xq = oracle.quantize_act(quant, x)
    shape = [rows, cols] if orient == "rc" else [cols, rows]
    w = upload(jkb, quant, wbytes, rows, cols, shape=shape)
    xd = dev(xq)
    sumi, summins, vals = (host(t) for t in jkb.gemv_block_dots(w, xd))
    s_ref, m_ref, v_ref = oracle.block_dots(quant, wbytes, rows, cols, xq)
    assert np.array_equal(sumi, s_ref), "per-block integer sums differ"
    if quant in (12, 13):
        assert np.array_equal(summins, m_ref), "per-block min sums differ"
    assert np.array_equal(bits(vals), bits(v_ref)), "per-block f32 values differ"
    y = run_gemv(jkb, quant, w, xd)
    y_ref = oracle.gemv(quant, wbytes, rows, cols, xq)
    ok, worst = R.gemv_tolerance_ok(y, y_ref, v_ref, REL)
    assert ok, f"row tolerance exceeded (worst {worst:.3g} of bound)"
    if np.linalg.norm(y_ref) > 0:
        assert R.l2_rel_err(y, y_ref) < REL
    w.destroy()
    return y, y_ref


def test_golden_fixtures(jkb, oracle):
    f = np.load(os.path.join(GOLDEN, "oracle_fixtures.npz"))
    names = sorted({k.split("__")[0] for k in f.files if k.endswith("__meta")})
    for name in names:
        q, rows, cols = (int(v) for v in f[f"{name}__meta"])
        wb = f[f"{name}__w"]
        w = upload(jkb, q, wb, rows, cols)
        xd = dev(f[f"{name}__xq"])
        sumi, summins, vals = (host(t) for t in jkb.gemv_block_dots(w, xd))
        assert np.array_equal(sumi, f[f"{name}__sumi"]), name
        if q in (12, 13):
            assert np.array_equal(summins, f[f"{name}__summins"]), name
        assert np.array_equal(bits(vals), bits(f[f"{name}__contrib"])), name
        y = run_gemv(jkb, q, w, xd)
        ok, worst = R.gemv_tolerance_ok(y, f[f"{name}__y"], f[f"{name}__contrib"], REL)
        assert ok, (name, worst)
        w.destroy()


@pytest.mark.parametrize("quant", [2, 8, 12, 14, 35, 6, 13])
@pytest.mark.parametrize("rows,cols", [(1, 256), (5, 4096), (67, 1024), (300, 14336)])
def test_gemv_random_normal(jkb, oracle, quant, rows, cols):
    if quant == 35:
        wb = oracle.pack_ternary(35, oracle.ternary(rows * cols, rows + cols), rows, cols, 0.02)
    else:
        wb = oracle.quantize_weights(quant, oracle.normal(rows * cols, 0x5EED0000 + rows, 0.02),
                                     rows, cols)
    x = oracle.normal(cols, 0xAC70000 + cols, 1.0)
    check_case(jkb, oracle, quant, wb, rows, cols, x)


@pytest.mark.parametrize("k", [256, 1536, 3584, 5120])
def test_wave4_generators_k_quants(jkb, oracle, k):
    """tests/wave4_quant_gemv_and_argmax.rs:361-542 inputs (LCG-filled blocks, incl. Q6_K
    negative scales and TQ2_0 code 3) on the GPU: bit-exact blocks and the 1e-5 contract
    against the f64 product over the Q8_K-dequantized input."""
    rows = 5
    x = R.gen_activation(k, 700 + k)
    xq = oracle.quantize_row_q8_k(x)
    xdq = R.dequant_q8(xq)
    for quant, fill, seed in ((12, R.fill_q4_k_m_bytes, 11), (14, R.fill_q6_k_bytes, 33),
                              (34, R.fill_tq1_0_bytes, 44), (35, R.fill_tq2_0_bytes, 55)):
        wb = fill(rows, k, seed + k)
        y, _ = check_case(jkb, oracle, quant, wb, rows, k, x, orient="cr")
        rq = R.ref_matvec(oracle, quant, wb, rows, k, xdq)
        assert R.l2_rel_err(y, rq) < 1e-5
        assert R.cosine(y, R.ref_matvec(oracle, quant, wb, rows, k, x)) > 0.999


@pytest.mark.parametrize("k", [128, 896, 4096])
def test_wave4_generators_q4_0_q8_0(jkb, oracle, k):
    """tests/wave4_quant_gemv_and_argmax.rs:254-348 inputs on the GPU."""
    x = R.gen_activation(k, 100 + k)
    for n in (1, 3, 4, 17, 1024):
        for quant, fill, seed in ((2, R.fill_q4_0_bytes, 200), (8, R.fill_q8_0_bytes, 400)):
            wb = fill(n, k, seed + k + n)
            y, _ = check_case(jkb, oracle, quant, wb, n, k, x, orient="cr")
            if n > 1 and (n <= 17 or k <= 896):
                assert R.cosine(y, R.ref_matvec(oracle, quant, wb, n, k, x)) > 0.9995


def test_zero_and_nonfinite_scales(jkb, oracle):
    """f16_to_f32_finite (lib.rs:714-717): NaN/Inf block scales act as 0; zero-scale and
    zero-activation blocks contribute exactly 0 (quant_q8.rs:675-677, :1837-1839)."""
    rows, cols = 9, 512
    for quant in (2, 8, 12, 14, 35, 6, 13):
        wb = oracle.quantize_weights(quant, oracle.normal(rows * cols, 3, 0.02), rows, cols) \
            if quant != 35 else oracle.pack_ternary(35, oracle.ternary(rows * cols, 3), rows,
                                                   cols, 0.02)
        be, bb = oracle.BLOCK[quant]
        blk = wb.reshape(rows, cols // be, bb)
        doff = 208 if quant == 14 else 0
        blk[0, 0, doff:doff + 2] = [0x00, 0x7C]  # +Inf
        blk[1, 0, doff:doff + 2] = [0x01, 0x7E]  # NaN
        blk[2, 1, doff:doff + 2] = [0x00, 0x00]  # zero
        if quant in (12, 13):
            blk[3, 1, 0:4] = 0  # d = dmin = 0
        x = oracle.normal(cols, 4, 1.0)
        x[:be] = 0.0  # first activation block all zero -> xd = 0
        check_case(jkb, oracle, quant, blk.reshape(-1), rows, cols, x)


@pytest.mark.parametrize("quant", [2, 8, 12, 14, 34, 35, 6, 13])
def test_vec_dot_single_row_bit_exact(jkb, oracle, quant):
    """vec_dot_*_q8_* on raw GGUF bytes: block values in parallel, then the reference's
    sequential `.sum()` -- bit-exact with the oracle."""
    cols = 4096
    if quant in (34, 35):
        wb = oracle.pack_ternary(quant, oracle.ternary(cols, 1), 1, cols, 0.02)
    else:
        wb = oracle.quantize_weights(quant, oracle.normal(cols, 2, 0.02), 1, cols)
    x = oracle.normal(cols, 5, 1.0)
    xq = oracle.quantize_act(quant, x)
    res = torch.empty(1, dtype=torch.float32, device="cuda")
    getattr(jkb, VEC_DOT_FN[quant])(dev(wb), dev(xq), res)
    assert bits(host(res))[0] == bits(np.float32(oracle.vec_dot(quant, wb, xq)))
    with pytest.raises(jkb.TensorBoundsError):
        getattr(jkb, VEC_DOT_FN[quant])(dev(wb[:-1]), dev(xq), res)


@pytest.mark.parametrize("quant,fn", [(12, "vec_dot_q4_k_m"), (8, "vec_dot_q8_0"),
                                      (14, "vec_dot_q6_k"), (2, "vec_dot_q4_0"),
                                      (36, "vec_dot_i2_s"), (6, "vec_dot_q5_0"),
                                      (13, "vec_dot_q5_k")])
def test_vec_dot_f32_activation_bit_exact(jkb, oracle, quant, fn):
    """VectorKernel f32-activation entries: dequantize -> sequential f32 dot (lib.rs:1268,
    quant.rs:899/1012/1401/2199), reproduced bit for bit."""
    rows, cols = 37, 1024
    if quant == 36:
        wb = oracle.pack_ternary(36, oracle.ternary(rows * cols, 9), rows, cols, 0.0173)
    else:
        wb = oracle.quantize_weights(quant, oracle.normal(rows * cols, 8, 0.02), rows, cols)
    x = oracle.normal(cols, 6, 1.0)
    w = upload(jkb, quant, wb, rows, cols)
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    getattr(jkb, fn)(out, w, dev(x))
    assert np.array_equal(bits(host(out)), bits(oracle.vec_dot_f32(quant, wb, rows, cols, x)))


def test_kats_through_gpu(jkb, oracle):
    """The vec_dot KATs (quant.rs:2593-2748, lib.rs:1365-1396) through the GPU f32 entries."""
    import json

    with open(os.path.join(GOLDEN, "kats.json")) as f:
        kats = json.load(f)
    fns = {8: "vec_dot_q8_0", 14: "vec_dot_q6_k", 2: "vec_dot_q4_0", 12: "vec_dot_q4_k_m",
           13: "vec_dot_q5_k"}
    for name in ("q8_0_vec_dot_f32", "q6_k_vec_dot_f32", "q4_0_vec_dot_f32", "q4_k_m_two_block",
                 "q5_k_dequant_sum"):
        k = kats[name]
        wb = np.frombuffer(bytes.fromhex(k["block_hex"]), np.uint8).copy()
        shape = k.get("shape", [k["rows"], k["cols"]])
        w = jkb.Weight(jkb.TensorView(name, k["quant"], shape, wb), k["rows"], k["cols"])
        out = torch.empty(k["rows"], dtype=torch.float32, device="cuda")
        getattr(jkb, fns[k["quant"]])(out, w, dev(np.array(k["input"], np.float32)))
        assert np.allclose(host(out), k["expected"], atol=k["abs_tol"], rtol=0), name


def test_row_range_stitching_and_device_upload(jkb, oracle):
    rows, cols, quant = 103, 2048, 12
    wb = oracle.quantize_weights(quant, oracle.normal(rows * cols, 1, 0.02), rows, cols)
    x = oracle.normal(cols, 2, 1.0)
    xd = dev(oracle.quantize_act(quant, x))
    w = upload(jkb, quant, wb, rows, cols, on_device=True)
    full = run_gemv(jkb, quant, w, xd)
    parts = []
    for a, b in ((0, 1), (1, 40), (40, 40), (40, 103)):
        o = torch.empty(b - a, dtype=torch.float32, device="cuda")
        jkb.gemv_rows(o, w, xd, range(a, b))
        parts.append(host(o))
    assert np.array_equal(bits(np.concatenate(parts)), bits(full))
    with pytest.raises(jkb.TensorBoundsError):
        jkb.gemv_rows(torch.empty(5, device="cuda"), w, xd, range(100, 105))


def test_gemv_validation_errors(jkb, oracle):
    rows, cols = 8, 512
    wb = oracle.quantize_weights(12, oracle.normal(rows * cols, 1, 0.02), rows, cols)
    w = upload(jkb, 12, wb, rows, cols)
    xq = dev(oracle.quantize_row_q8_k(oracle.normal(cols, 1)))
    with pytest.raises(jkb.TensorBoundsError, match="does not match output len 7"):
        jkb.gemv_q4_k_q8_k(torch.empty(7, device="cuda"), w, xq)
    with pytest.raises(jkb.TensorBoundsError, match="expected Q6_K quant type"):
        jkb.gemv_q6_k_q8_k(torch.empty(8, device="cuda"), w, xq)
    with pytest.raises(jkb.TensorBoundsError):
        jkb.gemv_q4_k_q8_k(torch.empty(8, device="cuda"), w, xq[:292])
    w.destroy()
    with pytest.raises(jkb.InvalidHandle):
        jkb.gemv_q4_k_q8_k(torch.empty(8, device="cuda"), w, xq)


@pytest.mark.parametrize("quant,rows,cols", [(12, 28672, 8192), (12, 8192, 28672),
                                             (14, 128256, 8192)])
def test_gemv_batch16_70b_shapes(jkb, oracle, quant, rows, cols):
    """BASELINE configs[4] at batch 16 (Llama-3-70B Q4_K_M gate/up, down and the Q6_K lm_head, full
    size): one jkb_gemv_batch launch equals the 16 single-token calls bit for bit, and sampled
    rows of the first and last token match the oracle within the row tolerance."""
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench  # seeded synthetic GGUF matrices at full size

    m = 16
    wb = bench.synth_matrix(quant, rows, cols, 77 + rows)
    w = upload(jkb, quant, wb, rows, cols)
    xs = [oracle.normal(cols, 900 + t, 1.0) for t in range(m)]
    xq = [oracle.quantize_act(quant, x) for x in xs]
    xall = dev(np.concatenate([q.view(np.uint8).reshape(-1) for q in xq]))
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    jkb.gemv_batch(out, w, xall, m)
    got = host(out).reshape(m, rows)
    for t in range(m):
        single = run_gemv(jkb, quant, w, dev(xq[t]))
        assert np.array_equal(bits(got[t]), bits(single)), f"token {t}"
    row_bytes = wb.size // rows
    sample = np.unique(np.concatenate([np.arange(8), np.arange(rows - 8, rows),
                                       np.random.default_rng(5).integers(0, rows, 48)]))
    for t in (0, m - 1):
        for r in sample:
            part = wb[r * row_bytes:(r + 1) * row_bytes]
            y_ref = oracle.gemv(quant, part, 1, cols, xq[t])
            _, _, v_ref = oracle.block_dots(quant, part, 1, cols, xq[t])
            ok, worst = R.gemv_tolerance_ok(got[t, r:r + 1], y_ref, v_ref, REL)
            assert ok, f"token {t} row {r}: worst {worst:.3g} of bound"
    w.destroy()

