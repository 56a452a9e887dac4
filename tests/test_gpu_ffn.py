"""GPU BitNet FFN pieces vs the CPU oracle: relu_squared_gate_f32 (lib.rs:1111-1148), the fused
ReLU^2 + SubLN quantizer, and the whole chain of tests/empirical_challenge_m3_bitnet.rs:582-686
(jkb_bitnet_ffn_*).

Contract per step: the elementwise ReLU^2 gating, the SubLN i8 activations and their scales
are bit-exact given the same input; BitLinear rows follow the GEMV contract (exact block
integers, 1e-5 on the row sums). The chain is checked step by step (each GPU step against the
oracle fed with the GPU's own previous step) and against the separate single-call kernels."""
import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import bits, dev, host, upload

pytestmark = pytest.mark.gpu

EPS = 1e-5


def _special_gate_up(n, seed):
    rng = np.random.default_rng(seed)
    g = rng.normal(0, 3, n).astype(np.float32)
    u = rng.normal(0, 3, n).astype(np.float32)
    k = min(n, 6)
    g[:k] = np.array([np.nan, -0.0, 0.0, np.inf, -np.inf, 1e20], np.float32)[:k]
    u[:k] = np.array([-1.0, -2.0, 3.0, 2.0, 5.0, 1.0], np.float32)[:k]
    return g, u


@pytest.mark.parametrize("n", [1, 6, 1000, 6912, (1 << 20) + 3])
def test_relu_squared_gate_bit_exact(jkb, oracle, n):
    g, u = _special_gate_up(n, n)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    jkb.relu_squared_gate_f32(out, dev(g), dev(u))
    ref = oracle.relu_squared_gate_f32(g, u)
    assert np.array_equal(bits(host(out)), bits(ref))


def test_relu_squared_gate_validation(jkb):
    a = torch.zeros(8, device="cuda")
    with pytest.raises(jkb.TensorBoundsError, match="dimension mismatch: gate=8, up=7, out=8"):
        jkb.relu_squared_gate_f32(a, a, a[:7])
    with pytest.raises(jkb.TensorBoundsError, match="relu_squared"):
        jkb.relu_squared_gate_f32(a[:0], a[:0], a[:0])


@pytest.mark.parametrize("m,length", [(1, 512), (3, 6912), (2, 7), (5, 2560)])
@pytest.mark.parametrize("keep_relu", [True, False])
def test_relu_squared_subln_rows_bit_exact(jkb, oracle, m, length, keep_relu):
    g, u = _special_gate_up(m * length, m + length)
    g[~np.isfinite(g)] = 0.5  # SubLN of an inf / NaN row is all-zero; keep rows informative
    g[np.abs(g) > 1e10] = 2.0
    if m > 1:
        g[length:2 * length] = -1.0  # a row whose ReLU^2 is all zero: the guarded branch
    w = (0.5 + np.random.default_rng(1).random(length)).astype(np.float32)
    out = torch.empty(m * length, dtype=torch.int8, device="cuda")
    relu = torch.empty(m * length, dtype=torch.float32, device="cuda") if keep_relu else None
    sc = torch.empty(m, dtype=torch.float32, device="cuda")
    jkb.relu_squared_subln_quantize_i8_rows(out, relu, dev(g), dev(u), dev(w), m, length, EPS,
                                            sc)
    q, s = host(out).reshape(m, length), host(sc)
    for r in range(m):
        h = oracle.relu_squared_gate_f32(g[r * length:(r + 1) * length],
                                         u[r * length:(r + 1) * length])
        qr, sr = oracle.subln_quantize_absmax_i8(h, w, EPS)
        assert np.array_equal(q[r], qr) and bits(np.float32(s[r])) == bits(np.float32(sr))
        if keep_relu:
            assert np.array_equal(bits(host(relu).reshape(m, length)[r]), bits(h))


def _ffn(jkb, wg, wu, wd, gq, uq, dq, hidden, inter, m_cap=1, n1=None, n2=None):
    Wg = upload(jkb, gq, wg, inter, hidden, name="gate")
    Wu = upload(jkb, uq, wu, inter, hidden, name="up")
    Wd = upload(jkb, dq, wd, hidden, inter, name="down")
    n1 = np.ones(hidden, np.float32) if n1 is None else n1
    n2 = np.ones(inter, np.float32) if n2 is None else n2
    return jkb.BitNetFFN(Wg, Wu, Wd, dev(n1), dev(n2), EPS, m_cap), (Wg, Wu, Wd), (n1, n2)


def test_chain_reference_scenarios(jkb, oracle):
    """The reference chain test's weights and inputs: every intermediate and the output equal
    the oracle chain bit for bit (one and two blocks per row, so the row sums have a single
    order)."""
    hidden, inter = 256, 512
    wg, wd = R.bitnet_chain_weights(hidden, inter)
    ffn, _, (n1, n2) = _ffn(jkb, wg, wg, wd, 35, 35, 34, hidden, inter)
    for name, x in R.bitnet_chain_scenarios(hidden):
        out = torch.empty(hidden, dtype=torch.float32, device="cuda")
        ffn.forward(out, dev(x))
        ref = oracle.bitnet_ffn(x, n1, n2, EPS, 35, wg, 35, wg, 34, wd, hidden, inter)
        a1, s1, g, u, h, a2, s2 = [host(t) for t in ffn.buffers()]
        assert np.array_equal(a1[0], ref["act1"]), name
        assert bits(np.float32(s1[0])) == bits(np.float32(ref["scale1"])), name
        for got, key in ((g[0], "gate"), (u[0], "up"), (h[0], "relu")):
            assert np.array_equal(bits(got), bits(ref[key])), (name, key)
        assert np.array_equal(a2[0], ref["act2"]), name
        assert bits(np.float32(s2[0])) == bits(np.float32(ref["scale2"])), name
        y = host(out)
        assert np.all(np.isfinite(y)), name
        assert np.array_equal(bits(y), bits(ref["out"])), name


def _ternary(oracle, quant, rows, cols, seed, scale):
    return oracle.pack_ternary(quant, oracle.ternary(rows * cols, seed), rows, cols, scale)


def _rows_close(got, ref, quant, w, rows, cols, act, scale, oracle):
    deq = oracle.dequantize_rows(quant, w, rows, cols).astype(np.float64)
    bound = np.abs(deq) @ (np.abs(act.astype(np.float64)) * abs(scale))
    assert np.all(np.abs(got.astype(np.float64) - ref) <= 1e-5 * bound + 1e-30)


@pytest.mark.parametrize("gq,dq,scales", [
    (35, 35, (0.0173, 0.0173, 0.021)),   # TQ2_0 throughout (gate and up in one launch)
    (35, 34, (0.0173, 0.0173, 0.021)),   # TQ2_0 gate / up, TQ1_0 down (the reference test)
    (36, 36, (0.0173, 0.0191, 0.021)),   # I2_S with different per-tensor scales: two launches
    (36, 36, (0.0173, 0.0173, 0.021)),   # I2_S, equal scales: one launch
])
def test_chain_bitnet_2b_shapes(jkb, oracle, gq, dq, scales):
    """BitNet-b1.58-2B FFN shapes (hidden 2560, intermediate 6912): step-wise parity and
    agreement with the separate single-call kernels."""
    hidden, inter = 2560, 6912
    wg = _ternary(oracle, gq, inter, hidden, 11, scales[0])
    wu = _ternary(oracle, gq, inter, hidden, 12, scales[1])
    wd = _ternary(oracle, dq, hidden, inter, 13, scales[2])
    rng = np.random.default_rng(5)
    n1 = (0.5 + rng.random(hidden)).astype(np.float32)
    n2 = (0.5 + rng.random(inter)).astype(np.float32)
    ffn, (Wg, Wu, Wd), _ = _ffn(jkb, wg, wu, wd, gq, gq, dq, hidden, inter, 1, n1, n2)
    x = oracle.normal(hidden, 7, 1.0)
    out = torch.empty(hidden, dtype=torch.float32, device="cuda")
    ffn.forward(out, dev(x))
    y = host(out)
    a1, s1, g, u, h, a2, s2 = [host(t)[0] for t in ffn.buffers()]
    # step 1: SubLN, bit-exact
    ra1, rs1 = oracle.subln_quantize_absmax_i8(x, n1, EPS)
    assert np.array_equal(a1, ra1) and bits(np.float32(s1)) == bits(np.float32(rs1))
    # step 2: gate / up BitLinear within the GEMV contract, equal to the single calls
    for got, w, q in ((g, wg, gq), (u, wu, gq)):
        ref = oracle.bitlinear_i8(q, w, inter, hidden, a1, float(s1))
        _rows_close(got, ref, q, w, inter, hidden, a1, float(s1), oracle)
    for got, W in ((g, Wg), (u, Wu)):
        one = torch.empty(inter, dtype=torch.float32, device="cuda")
        jkb.bitlinear_i8(one, W, dev(a1), float(s1))
        assert np.array_equal(bits(host(one)), bits(got))
    # step 3: ReLU^2 + SubLN on the GPU's gate / up, bit-exact
    rh = oracle.relu_squared_gate_f32(g, u)
    assert np.array_equal(bits(h), bits(rh))
    ra2, rs2 = oracle.subln_quantize_absmax_i8(rh, n2, EPS)
    assert np.array_equal(a2, ra2) and bits(np.float32(s2)) == bits(np.float32(rs2))
    # step 4: down BitLinear on the GPU's act2
    ref = oracle.bitlinear_i8(dq, wd, hidden, inter, a2, float(s2))
    _rows_close(y, ref, dq, wd, hidden, inter, a2, float(s2), oracle)
    one = torch.empty(hidden, dtype=torch.float32, device="cuda")
    jkb.bitlinear_i8(one, Wd, dev(a2), float(s2))
    assert np.array_equal(bits(host(one)), bits(y))
    # end to end against the oracle chain: the i8 activations may differ only where a row sum's
    # order moved an element across a rounding boundary, so compare the outputs loosely
    full = oracle.bitnet_ffn(x, n1, n2, EPS, gq, wg, gq, wu, dq, wd, hidden, inter)
    assert np.mean(full["act2"] != a2) < 1e-3
    assert R.l2_rel_err(y, full["out"]) < 1e-3


def test_chain_token_batch_matches_single_token(jkb, oracle):
    hidden, inter, m = 2560, 6912, 5
    wg = _ternary(oracle, 35, inter, hidden, 21, 0.0173)
    wu = _ternary(oracle, 35, inter, hidden, 22, 0.0173)
    wd = _ternary(oracle, 35, hidden, inter, 23, 0.021)
    ffn, _, _ = _ffn(jkb, wg, wu, wd, 35, 35, 35, hidden, inter, m_cap=m)
    X = np.stack([oracle.normal(hidden, 30 + t, 1.0) for t in range(m)])
    X[2] = 0.0  # an all-zero token inside the batch
    out = torch.empty(m * hidden, dtype=torch.float32, device="cuda")
    ffn.forward(out, dev(X.reshape(-1)), m)
    yb = host(out).reshape(m, hidden)
    for t in range(m):
        one = torch.empty(hidden, dtype=torch.float32, device="cuda")
        ffn.forward(one, dev(X[t]), 1)
        assert np.array_equal(bits(host(one)), bits(yb[t])), t
    assert not yb[2].any()


def test_chain_validation(jkb, oracle):
    hidden, inter = 256, 512
    wg, wd = R.bitnet_chain_weights(hidden, inter)
    ffn, (Wg, Wu, Wd), _ = _ffn(jkb, wg, wg, wd, 35, 35, 34, hidden, inter, m_cap=2)
    x = torch.zeros(3 * hidden, device="cuda")
    out = torch.empty(3 * hidden, device="cuda")
    with pytest.raises(jkb.TensorBoundsError, match="capacity"):
        ffn.forward(out, x, 3)
    with pytest.raises(jkb.TensorBoundsError, match="dimension mismatch"):
        ffn.forward(out[:hidden], x[:hidden - 1], 1)
    with pytest.raises(jkb.TensorBoundsError, match="output length"):
        ffn.forward(out[:hidden + 1], x[:hidden], 1)
    n1, n2 = torch.ones(hidden, device="cuda"), torch.ones(inter, device="cuda")
    with pytest.raises(jkb.TensorBoundsError):  # down given as the gate: shapes do not chain
        jkb.BitNetFFN(Wg, Wu, Wg, n1, n2, EPS)
    with pytest.raises(jkb.TensorBoundsError, match="norm weights"):
        jkb.BitNetFFN(Wg, Wu, Wd, n2, n2, EPS)
    q4 = upload(jkb, 2, np.zeros(inter * hidden // 32 * 18, np.uint8), inter, hidden)
    with pytest.raises(jkb.TensorBoundsError, match="unsupported quantization format"):
        jkb.BitNetFFN(q4, Wu, Wd, n1, n2, EPS)


@pytest.mark.parametrize("quant,dq", [(35, 35), (36, 36), (35, 34)])
def test_chain_tensor_core_batch(jkb, oracle, quant, dq):
    """Batches of at least 32 tokens with RepackedWeights: the three projections on the tensor
    cores (one accumulator per BitLinear block). With the exact epilogue every projection output
    is the reference's bitlinear_i8 of the GPU's own activations bit for bit; by default the
    chain stays within tolerance of the GEMV chain."""
    hidden, inter, m = 2560, 6912, 48
    wg = _ternary(oracle, quant, inter, hidden, 41, 0.0173)
    wu = _ternary(oracle, quant, inter, hidden, 42, 0.0173)
    wd = _ternary(oracle, dq, hidden, inter, 43, 0.021)
    rng = np.random.default_rng(9)
    n1 = (0.5 + rng.random(hidden)).astype(np.float32)
    n2 = (0.5 + rng.random(inter)).astype(np.float32)
    Wg = upload(jkb, quant, wg, inter, hidden, name="gate")
    Wu = upload(jkb, quant, wu, inter, hidden, name="up")
    Wd = upload(jkb, dq, wd, hidden, inter, name="down")
    rep = tuple(jkb.RepackedWeight.from_tensor(jkb.TensorView(n, q, [r, c], b), r, c)
                for n, q, b, r, c in (("gate", quant, wg, inter, hidden),
                                      ("up", quant, wu, inter, hidden),
                                      ("down", dq, wd, hidden, inter)))
    d1, d2 = dev(n1), dev(n2)
    tc = jkb.BitNetFFN(Wg, Wu, Wd, d1, d2, EPS, m, repacked=rep)
    gv = jkb.BitNetFFN(Wg, Wu, Wd, d1, d2, EPS, m)
    X = np.stack([oracle.normal(hidden, 60 + t, 1.0) for t in range(m)])
    x = dev(X.reshape(-1))
    out = torch.empty(m * hidden, dtype=torch.float32, device="cuda")
    with jkb.gemm_exact(True):
        tc.forward(out, x, m)
    y = host(out).reshape(m, hidden)
    a1, s1, g, u, h, a2, s2 = [host(t) for t in tc.buffers()]
    for t in (0, 17, m - 1):
        ra1, rs1 = oracle.subln_quantize_absmax_i8(X[t], n1, EPS)
        assert np.array_equal(a1[t], ra1) and bits(np.float32(s1[t])) == bits(np.float32(rs1))
        for got, w in ((g[t], wg), (u[t], wu)):
            ref = oracle.bitlinear_i8(quant, w, inter, hidden, a1[t], float(s1[t]))
            assert np.array_equal(bits(got), bits(ref))
        rh = oracle.relu_squared_gate_f32(g[t], u[t])
        assert np.array_equal(bits(h[t]), bits(rh))
        ra2, rs2 = oracle.subln_quantize_absmax_i8(rh, n2, EPS)
        assert np.array_equal(a2[t], ra2) and bits(np.float32(s2[t])) == bits(np.float32(rs2))
        ref = oracle.bitlinear_i8(dq, wd, hidden, inter, a2[t], float(s2[t]))
        assert np.array_equal(bits(y[t]), bits(ref))
    # default epilogue against the GEMV chain
    out2 = torch.empty(m * hidden, dtype=torch.float32, device="cuda")
    tc.forward(out, x, m)
    gv.forward(out2, x, m)
    assert R.l2_rel_err(host(out), host(out2)) < 1e-3
    with pytest.raises(jkb.TensorBoundsError, match="does not match"):
        jkb.BitNetFFN(Wg, Wu, Wd, d1, d2, EPS, m, repacked=(rep[0], rep[1], rep[0]))
