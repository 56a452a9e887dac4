"""The tcgen05 tensor-core path of the repacked GEMM (32-element scale groups: Q8_0, Q4_0,
TQ2_0, I2_S and Q4_K_M weights, the last with their min terms; 16-element groups: Q6_K;
batches of at least 16 tokens, 16 to 32 of them on the 32-token tile;
K a multiple of 128) vs the CPU oracle. Every output accumulates its groups in K order as
accumulate_scaled_tile_scalar does (repack.rs:3045-3093), acc += (f32)c * (xs * ws)
[- x_sum * wm]:
* with the exact epilogue (jkb.gemm_exact()) bit for bit;
* with the default fused multiply-add epilogue within the f32 tolerance contract
  (|err| <= 1e-5 * sum_k |x~||w~| per output, l2 relative error < 1e-5);
* the integer group sums c themselves are exact in both: with unit scales the default epilogue
  returns the integer dot products bit for bit.

Shapes cover one tile (32 x 128 x 128: one K stage, a partial token tile), ragged token and
weight-row tiles, K = 14336 (448 groups), a row range that starts inside a tile, batches that
select each of the four tile widths (32, 64, 96, 128 tokens; the 32-token one with 16 and 24
tokens, half or a quarter of it padding), and every format the path takes.
The device error word (bounded waits inside the kernel) must stay clear."""
import numpy as np
import pytest
import torch

from gpuutil import assert_gemm_close, bits, dev, gemm_abs_bound, host

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


SHAPES = [
    (8, 32, 128, 128),      # one tile, one K stage
    (8, 200, 300, 4096),    # ragged token and weight-row tiles
    (8, 129, 257, 14336),   # K = 14336, one row past a tile on both sides
    (8, 512, 1024, 4096),   # several tiles per CTA on small grids
    (8, 2048, 4096, 256),   # 2048 tokens x 32 weight tiles: the 64-token tile, 7 waves
    (8, 96, 12800, 256),    # 100 weight tiles, one 96-token tile each: the 96-token tile
    (8, 512, 18944, 256),   # 512 tokens x 148 weight tiles: the 128-token tile
    (8, 200, 12032, 256),   # 94 weight tiles, a partial last 64-token tile
    (12, 200, 300, 4096),   # Q4_K_M (min terms), ragged tiles
    (12, 2048, 4096, 256),  # Q4_K_M, the 64-token tile over 7 waves
    (12, 96, 12800, 256),   # Q4_K_M, the 96-token tile
    (14, 200, 300, 4096),   # Q6_K (16-element groups: masked token tiles, two MMAs a slice)
    (14, 2048, 4096, 256),  # Q6_K, the 64-token tile
    (14, 96, 12800, 256),   # Q6_K, the 96-token tile
    (2, 64, 640, 1024),     # Q4_0
    (35, 96, 256, 512),     # TQ2_0
    (36, 40, 384, 2560),    # I2_S (per-tensor scale)
    (6, 200, 300, 4096),    # Q5_0
    (13, 200, 300, 4096),   # Q5_K (min terms)
    (8, 16, 300, 4096),     # 16 tokens: the 32-token tile, half of it padding
    (8, 24, 1100, 512),     # 24 tokens, 9 weight tiles
    (12, 16, 300, 4096),    # Q4_K_M, 16 tokens
    (14, 16, 300, 4096),    # Q6_K, 16 tokens
    (12, 16, 28672, 256),   # Q4_K_M, 16 tokens over 224 weight tiles (two waves)
    (8, 16, 300, 4224),     # 3 tiles: K split over clusters of 4, 33 K stages split 8/8/8/9
    (12, 20, 1000, 2304),   # Q4_K_M, 8 tiles: K split over clusters of 4, ragged tokens
    (8, 32, 8192, 1024),    # 64 tiles: K split over clusters of 2
]


def _run(jkb, oracle, quant, m, rows, cols):
    wb = _weights(oracle, quant, rows, cols, 40 + rows)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], wb), rows, cols)
    act = oracle.normal(m * cols, 50 + m, 1.0)
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    out = torch.full((m * rows,), float("nan"), dtype=torch.float32, device="cuda")
    rw.gemm(out, a)
    assert jkb.device_status() == 0
    rw.destroy()
    return wb, act, host(out).reshape(m, rows)


@pytest.mark.parametrize("quant,m,rows,cols", SHAPES)
def test_tc_gemm_bit_exact(jkb, oracle, quant, m, rows, cols):
    with jkb.gemm_exact():
        wb, act, got = _run(jkb, oracle, quant, m, rows, cols)
    ref = _oracle_gemm(oracle, quant, wb, rows, cols, act, m)
    assert np.array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("quant,m,rows,cols", SHAPES)
def test_tc_gemm_fma_within_tolerance(jkb, oracle, quant, m, rows, cols):
    assert not jkb.gemm_get_exact()
    wb, act, got = _run(jkb, oracle, quant, m, rows, cols)
    ref = _oracle_gemm(oracle, quant, wb, rows, cols, act, m)
    assert np.all(np.isfinite(got))
    assert_gemm_close(got, ref, gemm_abs_bound(oracle, quant, wb, rows, cols, act, m))


def test_tc_gemm_integer_group_sums_exact(jkb, oracle):
    """Unit scales (Q8_0 d = 1.0; every activation block has absmax 127, so x_scale = 1.0 and
    the quantized values are the inputs): each output is the exact integer dot product, which
    the default epilogue must return bit for bit -- the int8 MMA sums are exact."""
    m, rows, cols = 96, 256, 2048
    rng = np.random.default_rng(3)
    wq = rng.integers(-127, 128, (rows, cols)).astype(np.int8)
    blk = np.zeros((rows, cols // 32, 34), np.uint8)
    blk[..., 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blk[..., 2:] = wq.reshape(rows, cols // 32, 32).view(np.uint8)
    wb = blk.reshape(-1)
    x = rng.integers(-127, 128, (m, cols)).astype(np.float32)
    x[:, ::32] = 127.0
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [rows, cols], wb), rows, cols)
    a = jkb.QuantizedActQ8.quantize(dev(x.reshape(-1)), m, cols)
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    rw.gemm(out, a)
    assert jkb.device_status() == 0
    want = x.astype(np.int64) @ wq.astype(np.int64).T
    assert np.abs(want).max() < 2 ** 24
    assert np.array_equal(host(out).reshape(m, rows), want.astype(np.float32))
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
    with jkb.gemm_exact():
        rw.gemm_rows(out, a, range(100, 333))
    assert jkb.device_status() == 0
    ref = _oracle_gemm(oracle, 8, wb, rows, cols, act, m)
    assert np.array_equal(bits(host(out).reshape(m, 233)), bits(ref[:, 100:333]))
    rw.gemm_rows(out, a, range(100, 333))
    bound = gemm_abs_bound(oracle, 8, wb, rows, cols, act, m)
    assert_gemm_close(host(out).reshape(m, 233), ref[:, 100:333], bound[:, 100:333])
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
    with jkb.gemm_exact():
        rw.gemm(out, a)
    assert jkb.device_status() == 0
    ref = _oracle_gemm(oracle, 8, wb, rows, cols, act, m)
    assert np.array_equal(bits(host(out).reshape(m, rows)), bits(ref))
    rw.gemm(out, a)
    assert_gemm_close(host(out).reshape(m, rows), ref,
                      gemm_abs_bound(oracle, 8, wb, rows, cols, act, m))
    rw.destroy()
