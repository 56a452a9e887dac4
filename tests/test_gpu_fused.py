"""GPU f32-input integer GEMV paths (vec_dot_*_rvv) and the grouped launch vs the CPU oracle.

The riscv64 entries vec_dot_q4_k_m_rvv / vec_dot_q6_k_rvv / vec_dot_q8_0_rvv / vec_dot_q4_0_rvv
(lib.rs:1313, quant.rs:1056/999/1445) quantize the f32 input with quantize_row_q8_k /
quantize_row_q8_0_f32 and run the Q8 GEMV (quant_q8.rs:3280-3317, :1712-1750). On the GPU the
quantization happens inside the GEMV launch, while every CTA stages the input, so:
  * the output equals jkb.quantize_row_q8_* followed by jkb.gemv_* bit for bit (same quantized
    bytes, same block arithmetic, same per-row summation order);
  * against the oracle it meets the GEMV contract over the oracle's own Q8 quantization of x
    (bit-exact block values, 1e-5 row tolerance);
  * a grouped launch returns, for every item, exactly its single call's output."""
import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import bits, dev, host, upload

pytestmark = pytest.mark.gpu
REL = 1e-5

RVV_FN = {2: "vec_dot_q4_0_rvv", 8: "vec_dot_q8_0_rvv", 12: "vec_dot_q4_k_m_rvv",
          14: "vec_dot_q6_k_rvv", 6: "vec_dot_q5_0_rvv", 13: "vec_dot_q5_k_rvv"}
GEMV_FN = {2: "gemv_q4_0_q8_0", 8: "gemv_q8_0_q8_0", 12: "gemv_q4_k_q8_k", 14: "gemv_q6_k_q8_k",
           6: "gemv_q5_0_q8_0", 13: "gemv_q5_k_q8_k"}


def weights(oracle, quant, rows, cols, seed):
    return oracle.quantize_weights(quant, oracle.normal(rows * cols, seed, 0.02), rows, cols)


def quantize_then_gemv(jkb, quant, w, x_dev):
    cols = x_dev.numel()
    if quant in (2, 8, 6):
        xq = jkb.empty_q8_0_blocks(cols // 32)
        jkb.quantize_row_q8_0(x_dev, xq)
    else:
        xq = jkb.empty_q8_k_blocks(cols // 256)
        jkb.quantize_row_q8_k(x_dev, xq)
    out = torch.empty(w.rows, dtype=torch.float32, device="cuda")
    getattr(jkb, GEMV_FN[quant])(out, w, xq)
    return host(out)


def fused(jkb, quant, w, x_dev):
    out = torch.empty(w.rows, dtype=torch.float32, device="cuda")
    getattr(jkb, RVV_FN[quant])(out, w, x_dev)
    return host(out)


def check_against_oracle(oracle, quant, wb, rows, cols, x, y):
    xq = oracle.quantize_act(quant, x)
    _, _, v_ref = oracle.block_dots(quant, wb, rows, cols, xq)
    y_ref = oracle.gemv(quant, wb, rows, cols, xq)
    ok, worst = R.gemv_tolerance_ok(y, y_ref, v_ref, REL)
    assert ok, f"row tolerance exceeded (worst {worst:.3g} of bound)"
    if np.linalg.norm(y_ref) > 0:
        assert R.l2_rel_err(y, y_ref) < REL


# Shapes cover every cluster size the launcher picks (1, 2, 4 and 8 CTAs), CTAs of 2, 4 and 8
# warps, a partial last Q8_0 unit (96 columns) and a single block (32 columns).
CASES = [(12, 37, 1024), (12, 64, 768), (12, 300, 14336), (12, 2048, 8192), (14, 33, 512),
         (14, 129, 4096), (8, 17, 96), (8, 70, 4096), (8, 40, 14336), (2, 5, 32), (2, 200, 2048),
         (6, 33, 1024), (6, 300, 14336), (13, 37, 1024), (13, 129, 4096)]


@pytest.mark.parametrize("quant,rows,cols", CASES)
def test_rvv_equals_quantize_then_gemv(jkb, oracle, quant, rows, cols):
    wb = weights(oracle, quant, rows, cols, 0xF00 + rows)
    w = upload(jkb, quant, wb, rows, cols)
    x = oracle.normal(cols, 0xF10 + cols, 1.0)
    xd = dev(x)
    y = fused(jkb, quant, w, xd)
    assert np.array_equal(bits(y), bits(quantize_then_gemv(jkb, quant, w, xd)))
    check_against_oracle(oracle, quant, wb, rows, cols, x, y)
    w.destroy()


@pytest.mark.parametrize("quant", [2, 8, 12, 14, 6, 13])
def test_rvv_special_inputs(jkb, oracle, quant):
    """Non-finite inputs quantize to 0 (round_scaled_to_i8, quant_q8.rs:102-108) and do not
    enter the block absmax; all-zero and -0.0 blocks give a zero scale; extreme magnitudes."""
    rows, cols = 11, 1024
    wb = weights(oracle, quant, rows, cols, 77)
    w = upload(jkb, quant, wb, rows, cols)
    x = oracle.normal(cols, 78, 1.0)
    x[3], x[40], x[300] = np.nan, np.inf, -np.inf
    x[256:512] = 0.0
    x[512:544] = -0.0
    x[600] = 3.0e38
    x[700:710] = 1.0e-40  # subnormal
    xd = dev(x)
    y = fused(jkb, quant, w, xd)
    assert np.array_equal(bits(y), bits(quantize_then_gemv(jkb, quant, w, xd)))
    xq_ref = oracle.quantize_act(quant, x)
    y_ref = oracle.gemv(quant, wb, rows, cols, xq_ref)
    _, _, v_ref = oracle.block_dots(quant, wb, rows, cols, xq_ref)
    ok, worst = R.gemv_tolerance_ok(y, y_ref, v_ref, REL)
    assert ok, f"row tolerance exceeded (worst {worst:.3g} of bound)"
    w.destroy()


@pytest.mark.parametrize("quant", [8, 12])
def test_rvv_input_not_16_byte_aligned(jkb, oracle, quant):
    """A 4-byte aligned input that is not 16-byte aligned takes the scalar staging loads."""
    rows, cols = 23, 2048
    wb = weights(oracle, quant, rows, cols, 91)
    w = upload(jkb, quant, wb, rows, cols)
    x = oracle.normal(cols, 92, 1.0)
    buf = torch.empty(cols + 4, dtype=torch.float32, device="cuda")
    buf[1:cols + 1].copy_(dev(x))
    xs = buf[1:cols + 1]
    assert xs.data_ptr() % 16 != 0
    y = fused(jkb, quant, w, xs)
    assert np.array_equal(bits(y), bits(fused(jkb, quant, w, dev(x))))
    w.destroy()


@pytest.mark.parametrize("quant,cols,rows_list", [
    (12, 1024, [64, 16, 16]),                      # q / k / v of a small layer
    (12, 4096, [14336 // 8, 14336 // 8]),          # gate / up
    (14, 512, [7, 1, 40]),
    (8, 256, [3, 5]),
    (2, 64, [1, 2, 3, 5, 7, 31, 33, 100]),          # eight items, ragged row counts
])
def test_grouped_equals_single_calls(jkb, oracle, quant, cols, rows_list):
    x = oracle.normal(cols, 0x6A0 + cols, 1.0)
    xd = dev(x)
    ws, wbs = [], []
    for i, rows in enumerate(rows_list):
        wb = weights(oracle, quant, rows, cols, 0x6B0 + 13 * i)
        wbs.append(wb)
        ws.append(upload(jkb, quant, wb, rows, cols, name=f"w{i}"))
    outs = [torch.full((w.rows,), float("nan"), device="cuda") for w in ws]
    jkb.vec_dot_grouped_rvv(list(zip(outs, ws)), xd)
    for i, (w, o) in enumerate(zip(ws, outs)):
        y = host(o)
        assert np.array_equal(bits(y), bits(fused(jkb, quant, w, xd))), f"item {i}"
        if i < 3:
            check_against_oracle(oracle, quant, wbs[i], w.rows, cols, x, y)
    for w in ws:
        w.destroy()


def test_grouped_validation(jkb, oracle):
    cols = 512
    x = dev(oracle.normal(cols, 1, 1.0))
    a = upload(jkb, 12, weights(oracle, 12, 8, cols, 1), 8, cols, name="a")
    b = upload(jkb, 14, weights(oracle, 14, 8, cols, 2), 8, cols, name="b")
    c = upload(jkb, 12, weights(oracle, 12, 8, 2 * cols, 3), 8, 2 * cols, name="c")
    t = upload(jkb, 35, oracle.pack_ternary(35, oracle.ternary(8 * cols, 4), 8, cols, 0.02),
               8, cols, name="t")
    o = lambda n=8: torch.empty(n, device="cuda")  # noqa: E731
    with pytest.raises(jkb.TensorBoundsError, match="expected Q4_K_M quant type"):
        jkb.vec_dot_grouped_rvv([(o(), a), (o(), b)], x)
    with pytest.raises(jkb.TensorBoundsError):
        jkb.vec_dot_grouped_rvv([(o(), a), (o(), c)], x)  # width differs from the input
    with pytest.raises(jkb.TensorBoundsError, match="does not match output len 7"):
        jkb.vec_dot_grouped_rvv([(o(), a), (o(7), a)], x)
    with pytest.raises(jkb.TensorBoundsError):
        jkb.vec_dot_grouped_rvv([], x)
    with pytest.raises(jkb.TensorBoundsError):
        jkb.vec_dot_grouped_rvv([(o(), a)] * 9, x)
    with pytest.raises(jkb.CapabilityMismatch):
        jkb.vec_dot_grouped_rvv([(o(), t)], x)
    with pytest.raises(jkb.TensorBoundsError, match="expected Q6_K quant type"):
        jkb.vec_dot_q6_k_rvv(o(), a, x)
    with pytest.raises(jkb.TensorBoundsError):
        jkb.vec_dot_q4_k_m_rvv(o(), a, x[:256])
    for w in (a, b, c, t):
        w.destroy()
