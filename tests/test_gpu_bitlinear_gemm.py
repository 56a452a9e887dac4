"""GPU BitLinear (ime.rs:882-938) and repacked GEMM (repack.rs:2718-3093) vs the CPU oracle.

BitLinear outputs follow the GEMV contract (bit-exact block integers, 1e-5 on the row sums);
the repacked GEMM accumulates its scale groups in K order per output exactly like
accumulate_scaled_tile_scalar, so its outputs are compared bit for bit."""
import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import assert_gemm_close, gemm_abs_bound, bits, dev, host, upload

pytestmark = pytest.mark.gpu


def bitnet_act(oracle, k, seed):
    x = oracle.normal(k, seed, 1.0)
    return oracle.subln_quantize_absmax_i8(x, np.ones(k, np.float32), 1e-5)


def ternary_weights(oracle, quant, rows, cols, seed, scale=0.0173):
    t = oracle.ternary(rows * cols, seed)
    return oracle.pack_ternary(quant, t, rows, cols, scale)


@pytest.mark.parametrize("quant", [34, 35, 8, 36])
@pytest.mark.parametrize("rows,cols", [(37, 256), (2560, 6912), (6912, 2560)])
def test_bitlinear_i8_vs_oracle(jkb, oracle, quant, rows, cols):
    if quant == 8:
        wb = oracle.quantize_weights(8, oracle.normal(rows * cols, 5, 0.02), rows, cols)
    else:
        if cols % oracle.BLOCK[quant][0]:
            pytest.skip("shape not a multiple of the block")
        wb = ternary_weights(oracle, quant, rows, cols, rows + cols)
    act, scale = bitnet_act(oracle, cols, cols)
    w = upload(jkb, quant, wb, rows, cols)
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    jkb.bitlinear_i8(out, w, dev(act), scale)
    y = host(out)
    ref = oracle.bitlinear_i8(quant, wb, rows, cols, act, scale)
    # per-element bound from the block values (integer dots exact, scale product rounded once)
    deq = oracle.dequantize_rows(quant, wb, rows, cols).astype(np.float64)
    absb = np.abs(deq) @ (np.abs(act.astype(np.float64)) * abs(scale))
    assert np.all(np.abs(y.astype(np.float64) - ref) <= 1e-5 * absb + 1e-30)
    assert R.l2_rel_err(y, ref) < 1e-5
    for alias in (jkb.bitlinear_i8_rvv, jkb.bitlinear_i8_ime):
        o2 = torch.empty(rows, dtype=torch.float32, device="cuda")
        alias(o2, w, dev(act), scale)
        assert np.array_equal(bits(host(o2)), bits(y))


@pytest.mark.parametrize("quant,m", [(35, 16), (34, 11), (36, 9), (8, 3)])
def test_bitlinear_batch_matches_single_calls(jkb, oracle, quant, m):
    """Token batches (up to eight tokens per CTA share each weight load, each with its own
    scale) equal the single-token calls bit for bit."""
    rows, cols = 640, 2560
    if quant == 8:
        wb = oracle.quantize_weights(8, oracle.normal(rows * cols, 3, 0.02), rows, cols)
    else:
        wb = ternary_weights(oracle, quant, rows, cols, 3)
    w = upload(jkb, quant, wb, rows, cols)
    acts, scales = [], []
    for t in range(m):
        a, s = bitnet_act(oracle, cols, 100 + t)
        acts.append(a)
        scales.append(s)
    A = np.concatenate(acts)
    S = np.array(scales, np.float32)
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    jkb.bitlinear_i8_batch(out, w, dev(A), dev(S))
    ob = host(out).reshape(m, rows)
    ref = oracle.bitlinear_i8_batch(quant, wb, rows, cols, A, S, nthreads=4)
    for t in range(m):
        one = torch.empty(rows, dtype=torch.float32, device="cuda")
        jkb.bitlinear_i8(one, w, dev(acts[t]), scales[t])
        assert np.array_equal(bits(host(one)), bits(ob[t]))
        assert R.l2_rel_err(ob[t], ref[t]) < 1e-5


def test_bitlinear_validation(jkb, oracle):
    rows, cols = 8, 256
    wb = oracle.quantize_weights(12, oracle.normal(rows * cols, 1, 0.02), rows, cols)
    w = upload(jkb, 12, wb, rows, cols)
    with pytest.raises(jkb.TensorBoundsError, match="unsupported quantization format"):
        jkb.bitlinear_i8(torch.empty(rows, device="cuda"), w,
                         torch.zeros(cols, dtype=torch.int8, device="cuda"), 1.0)
    wt = upload(jkb, 35, ternary_weights(oracle, 35, rows, cols, 1), rows, cols)
    with pytest.raises(jkb.TensorBoundsError):
        jkb.bitlinear_i8(torch.empty(rows, device="cuda"), wt,
                         torch.zeros(cols - 1, dtype=torch.int8, device="cuda"), 1.0)


def _weights(oracle, quant, rows, cols, seed):
    if quant in (34, 35, 36):
        return ternary_weights(oracle, quant, rows, cols, seed)
    return oracle.quantize_weights(quant, oracle.normal(rows * cols, seed, 0.02), rows, cols)


@pytest.mark.parametrize("quant", [8, 2, 12, 14, 35, 36, 6, 13])
def test_repacked_weight_buffers_bit_exact(jkb, oracle, quant):
    rows, cols = 29, 1024
    wb = _weights(oracle, quant, rows, cols, 4)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], wb), rows, cols)
    q, s, m = (None if t is None else host(t) for t in rw.buffers())
    q_ref, s_ref, m_ref = oracle.repack_block_scaled(quant, wb, rows, cols)
    assert np.array_equal(q, q_ref)
    assert np.array_equal(bits(s), bits(s_ref))
    if m_ref is not None:
        assert np.array_equal(bits(m), bits(m_ref))


def _oracle_gemm(oracle, quant, wb, rows, cols, act, m, r0=0, r1=None):
    q, s, mn = oracle.repack_block_scaled(quant, wb, rows, cols)
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(act, m, cols)
    return oracle.gemm_repacked(quant, q, s, mn, rows, cols, xq, xs, xsum, xs16, m, r0, r1,
                                nthreads=8)


@pytest.mark.parametrize("quant", [8, 2, 12, 14, 35, 36, 6, 13])
@pytest.mark.parametrize("m", [1, 5, 17, 64])
def test_gemm_repacked_bit_exact(jkb, oracle, quant, m):
    """tests/test_repack_gemv_gemm.rs:751-829 shapes (M in {1,5,8,17,64}) on the GPU,
    compared bit for bit with the scalar GEMM branch."""
    rows, cols = 72, 1024
    wb = _weights(oracle, quant, rows, cols, 6)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [cols, rows], wb), rows, cols)
    act = oracle.normal(m * cols, 100 + m, 1.0)
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    ref = _oracle_gemm(oracle, quant, wb, rows, cols, act, m)
    with jkb.gemm_exact():  # the tensor-core path (m = 64) with the reference's roundings
        rw.gemm(out, a)
        assert np.array_equal(bits(host(out).reshape(m, rows)), bits(ref))
        if m == 1:
            o1 = torch.empty(rows, dtype=torch.float32, device="cuda")
            rw.gemv(o1, a)
            assert np.array_equal(bits(host(o1)), bits(ref[0]))
        parts = []
        for r0, r1 in ((0, 9), (9, 64), (64, 72)):
            o = torch.empty(m * (r1 - r0), dtype=torch.float32, device="cuda")
            rw.gemm_rows(o, a, range(r0, r1))
            parts.append(host(o).reshape(m, r1 - r0))
        assert np.array_equal(bits(np.concatenate(parts, axis=1)), bits(ref))
    rw.gemm(out, a)  # default epilogue: bit-exact on the dp4a path, within tolerance on tcgen05
    assert_gemm_close(host(out).reshape(m, rows), ref,
                      gemm_abs_bound(oracle, quant, wb, rows, cols, act, m))


@pytest.mark.parametrize("m,rows,cols", [(128, 512, 4096), (256, 384, 2048)])
def test_gemm_repacked_q8_0_prefill_shapes(jkb, oracle, m, rows, cols):
    """Q8_0 x Q8_0 prefill GEMM (BASELINE config 3 kind) at a size the oracle finishes quickly."""
    wb = _weights(oracle, 8, rows, cols, 9)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [rows, cols], wb), rows, cols)
    act = oracle.normal(m * cols, 10, 1.0)
    scratch = jkb.QuantizedActQ8(m, cols)
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    ref = _oracle_gemm(oracle, 8, wb, rows, cols, act, m)
    with jkb.gemm_exact():
        jkb.gemm_repacked_f32(out, rw, dev(act), m, scratch)
    assert np.array_equal(bits(host(out).reshape(m, rows)), bits(ref))
    jkb.gemm_repacked_f32(out, rw, dev(act), m, scratch)
    assert_gemm_close(host(out).reshape(m, rows), ref,
                      gemm_abs_bound(oracle, 8, wb, rows, cols, act, m))


def test_gemm_validation(jkb, oracle):
    rows, cols = 16, 256
    wb = _weights(oracle, 8, rows, cols, 1)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [rows, cols], wb), rows, cols)
    a = jkb.QuantizedActQ8.quantize(dev(oracle.normal(2 * cols, 1)), 2, cols)
    with pytest.raises(jkb.TensorBoundsError, match="act.m"):
        rw.gemv(torch.empty(rows, device="cuda"), a)
    with pytest.raises(jkb.TensorBoundsError):
        rw.gemm(torch.empty(rows, device="cuda"), a)
    with pytest.raises(jkb.TensorBoundsError):
        rw.gemm_rows(torch.empty(2 * 4, device="cuda"), a, range(14, 18))
    b = jkb.QuantizedActQ8.quantize(dev(oracle.normal(512, 2)), 1, 512)
    with pytest.raises(jkb.TensorBoundsError):
        rw.gemm(torch.empty(rows, device="cuda"), b)


@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("rows,cols,m", [(640, 2560, 128), (2560, 6912, 40), (6912, 2560, 64),
                                         (256, 1024, 8), (384, 512, 33), (6912, 2560, 128)])
@pytest.mark.parametrize("quant", [35, 34, 36, 8])
def test_bitlinear_gemm_tensor_cores(jkb, oracle, quant, rows, cols, m, exact):
    """jkb_bitlinear_i8_gemm against the reference's per-token bitlinear_i8 (ime.rs:882-938).
    From 32 tokens every BitLinear block is one tensor-core accumulator and its value
    (f32)c * (d * s) is added in K order: the exact epilogue gives the reference's row sums bit
    for bit, the default one stays within the 1e-5 contract. Below 32 tokens the repacked
    GEMM's 32-element groups run (within the contract)."""
    wb = _weights(oracle, quant, rows, cols, rows + cols + m)
    acts, scales = zip(*[bitnet_act(oracle, cols, 500 + t) for t in range(m)])
    A = np.concatenate(acts)
    S = np.array(scales, np.float32)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], wb), rows, cols)
    scratch = jkb.QuantizedActQ8(m + 3, cols)
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    with jkb.gemm_exact(exact):
        jkb.bitlinear_i8_gemm(out, rw, dev(A), dev(S), m, scratch)
    y = host(out).reshape(m, rows)
    ref = oracle.bitlinear_i8_batch(quant, wb, rows, cols, A, S, nthreads=8)
    if exact and m >= 32:
        assert np.array_equal(bits(y), bits(ref))
    else:
        deq = np.abs(oracle.dequantize_rows(quant, wb, rows, cols).astype(np.float64))
        xa = np.abs(A.reshape(m, cols).astype(np.float64)) * S.astype(np.float64)[:, None]
        bound = xa @ deq.T
        assert np.all(np.abs(y.astype(np.float64) - ref) <= 1e-5 * bound + 1e-30)
    rw.destroy()
    scratch.destroy()


def test_bitlinear_gemm_validation(jkb, oracle):
    rows, cols, m = 128, 512, 32
    wq = oracle.quantize_weights(12, oracle.normal(rows * cols, 1, 0.02), rows, cols)
    rq = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 12, [rows, cols], wq), rows, cols)
    scratch = jkb.QuantizedActQ8(m, cols)
    A = torch.zeros(m * cols, dtype=torch.int8, device="cuda")
    S = torch.ones(m, device="cuda")
    out = torch.empty(m * rows, device="cuda")
    with pytest.raises(jkb.TensorBoundsError, match="unsupported quantization format"):
        jkb.bitlinear_i8_gemm(out, rq, A, S, m, scratch)
    wt = ternary_weights(oracle, 35, rows, cols, 2)
    rt = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 35, [rows, cols], wt), rows, cols)
    with pytest.raises(jkb.TensorBoundsError, match="capacity"):
        jkb.bitlinear_i8_gemm(torch.empty((m + 1) * rows, device="cuda"), rt,
                              torch.zeros((m + 1) * cols, dtype=torch.int8, device="cuda"),
                              torch.ones(m + 1, device="cuda"), m + 1, scratch)
    with pytest.raises(jkb.TensorBoundsError, match="k 256 != weight cols 512"):
        jkb.bitlinear_i8_gemm(out, rt, A, S, m, jkb.QuantizedActQ8(m, 256))
