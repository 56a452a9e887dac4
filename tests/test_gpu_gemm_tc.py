"""The tcgen05 tensor-core path of the repacked GEMM (32-element scale groups without mins:
Q8_0, Q4_0, TQ2_0, I2_S weights; batches of at least 32 tokens; K a multiple of 128) vs the CPU
oracle, bit for bit: every output accumulates its groups in K order as
accumulate_scaled_tile_scalar does (repack.rs:3045-3093), acc += (f32)c * (xs * ws).

Shapes cover one tile (32 x 128 x 128: one K stage, a partial M tile), ragged M and N tiles,
K = 14336 (448 groups), a row range that starts inside a tile, and every format the path
takes. The device error word (bounded waits inside the kernel) must stay clear."""
import numpy as np
import pytest
import torch

from gpuutil import bits, dev, host

pytestmark = pytest.mark.gpu


def _weights(oracle, quant, rows, cols, seed):
    if quant in (34, 35, 36):
        return oracle.pack_ternary(quant, oracle.ternary(rows * cols, seed), rows, cols, 0.0173)
    return oracle.quantize_weights(quant, oracle.normal(rows * cols, seed, 0.02), rows, cols)


def _oracle_gemm(oracle, quant, wb, rows, cols, act, m, r0=0, r1=None):
    q, s, mn = oracle.repack_block_scaled(quant, wb, rows, cols)
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(act, m, cols)
    return oracle.gemm_repacked(quant, q, s, mn, rows, cols, xq, xs, xsum, xs16, m, r0, r1,
                                nthreads=8)


@pytest.mark.parametrize("quant,m,rows,cols", [
    (8, 32, 128, 128),      # one tile, one K stage
    (8, 200, 300, 4096),    # ragged M (72 of 128) and N (44 of 128) tiles
    (8, 129, 257, 14336),   # K = 14336, one row past an M tile, one past an N tile
    (8, 512, 1024, 4096),   # several tiles per CTA on small grids
    (2, 64, 640, 1024),     # Q4_0
    (35, 96, 256, 512),     # TQ2_0
    (36, 40, 384, 2560),    # I2_S (per-tensor scale)
])
def test_tc_gemm_bit_exact(jkb, oracle, quant, m, rows, cols):
    wb = _weights(oracle, quant, rows, cols, 40 + rows)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], wb), rows, cols)
    act = oracle.normal(m * cols, 50 + m, 1.0)
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    out = torch.full((m * rows,), float("nan"), dtype=torch.float32, device="cuda")
    rw.gemm(out, a)
    assert jkb.device_status() == 0
    ref = _oracle_gemm(oracle, quant, wb, rows, cols, act, m)
    assert np.array_equal(bits(host(out).reshape(m, rows)), bits(ref))
    rw.destroy()


def test_tc_gemm_row_range(jkb, oracle):
    """gemm_repacked_rows (repack.rs:4087) over [100, 333) of 384 rows: the tiles start at a
    weight row that is not a multiple of 128, and the last tile is partial."""
    m, rows, cols = 70, 384, 2048
    wb = _weights(oracle, 8, rows, cols, 7)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [rows, cols], wb), rows, cols)
    act = oracle.normal(m * cols, 8, 1.0)
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    out = torch.empty(m * 233, dtype=torch.float32, device="cuda")
    rw.gemm_rows(out, a, range(100, 333))
    assert jkb.device_status() == 0
    ref = _oracle_gemm(oracle, 8, wb, rows, cols, act, m)
    assert np.array_equal(bits(host(out).reshape(m, 233)), bits(ref[:, 100:333]))
    rw.destroy()


def test_tc_gemm_special_activations(jkb, oracle):
    """Zero and non-finite activation blocks (absmax < 1e-30 -> zero scale; non-finite
    sanitized to 0, repack.rs:175-204) through the tensor-core path."""
    m, rows, cols = 48, 256, 1024
    wb = _weights(oracle, 8, rows, cols, 11)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [rows, cols], wb), rows, cols)
    act = oracle.normal(m * cols, 12, 1.0).reshape(m, cols)
    act[0, :] = 0.0
    act[1, 32:64] = np.nan
    act[2, 100] = np.inf
    act[3, :32] = 1e-35
    act = act.reshape(-1)
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    rw.gemm(out, a)
    assert jkb.device_status() == 0
    ref = _oracle_gemm(oracle, 8, wb, rows, cols, act, m)
    assert np.array_equal(bits(host(out).reshape(m, rows)), bits(ref))
    rw.destroy()
