"""PackedNibbleMatrix on the GPU (repack.rs:4188-5545): Q4_0, Q4_1, IQ4_NL and Q4_K_M weights
kept 4-bit on the device, their GEMM, gemv, row ranges, dequantize_row and the tile-buffer
constructors, against the CPU oracle's restatement of execute_nibble_gemm_rows.

* The row kernel (batches under 32 tokens, or cols not a multiple of 128) reproduces the
  reference's sequential roundings: bit for bit in both epilogue modes.
* The tensor-core path (>= 32 tokens, cols a multiple of 128; converter warps expand the
  4-bit codes in shared memory): bit for bit under jkb.gemm_exact(), within the f32 tolerance
  contract (|err| <= 1e-5 * sum_k |x~||w~| per output, l2 relative error < 1e-5) by default.
* On the same weights the nibble GEMM and the repacked i8 GEMM agree bit for bit (the suite's
  own parity property, tests/wave3_prefill_gqa_and_gemm.rs:233-279).
* Device bytes equal the GGUF payload (the 1.00x footprint contract).
The device error word (bounded waits in the tensor-core kernel) must stay clear."""
import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import assert_gemm_close, bits, dev, host

pytestmark = pytest.mark.gpu

Q4_0, Q4_1, IQ4_NL, Q4_K = 2, 3, 20, 12
FORMATS = [Q4_0, Q4_1, IQ4_NL, Q4_K]


def _weights(oracle, quant, rows, cols, seed):
    return oracle.quantize_weights(quant, oracle.normal(rows * cols, seed, 0.02), rows, cols)


def _oracle(oracle, quant, wb, rows, cols, act, m, r0=0, r1=None):
    q, ws, wm = oracle.nibble_decode(quant, wb, rows, cols)
    xq, xs, xsum, _, _ = oracle.act_q8_quantize(act, m, cols)
    return oracle.gemm_nibble(quant, q, ws, wm, rows, cols, xq, xs, xsum, m, r0, r1, nthreads=8)


def _bound(oracle, quant, wb, rows, cols, act, m):
    """sum_k |x~[m,k]| |w~[n,k]| (+ |x_sum| |wm| for the min formats), f64."""
    q, ws, wm = oracle.nibble_decode(quant, wb, rows, cols)
    xq, xs, xsum, _, _ = oracle.act_q8_quantize(act, m, cols)
    xd = np.abs(xq.astype(np.float64) * np.repeat(xs.astype(np.float64), 32, axis=1))
    wd = np.abs(q.astype(np.float64) * np.repeat(ws.astype(np.float64), 32, axis=1))
    b = xd @ wd.T
    if wm is not None:
        b += np.abs(xsum.astype(np.float64)) @ np.abs(wm.astype(np.float64)).T
    return b


def _matrix(jkb, quant, wb, rows, cols):
    return jkb.PackedNibbleMatrix.from_tensor(jkb.TensorView("w", quant, [cols, rows], wb), rows,
                                              cols)


def _gemm(jkb, nm, act, m, cols, rows, r=None):
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    n = rows if r is None else len(r)
    out = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
    if r is None:
        nm.gemm(out, a)
    else:
        nm.gemm_rows(out, a, r)
    assert jkb.device_status() == 0
    return host(out).reshape(m, n)


# (m, rows, cols): row kernel shapes (m below the tensor-core threshold -- at most 32, from 8 on
# large matrices -- or cols % 128 != 0) and tensor-core shapes
ROWS_SHAPES = [(1, 203, 512), (5, 64, 256), (17, 256, 512), (31, 130, 1024), (40, 77, 160),
               (64, 33, 800)]
TC_SHAPES = [(32, 128, 256), (64, 300, 1024), (100, 203, 4096), (200, 256, 512),
             (512, 1024, 2048), (96, 12800, 256), (512, 18944, 256), (9, 14336, 256)]
# (96, 12800, 256) and (512, 18944, 256) select the 96- and 128-token tiles (formats without min
# terms; the min formats take 96 or 64, IQ4_NL always 64); (9, 14336, 256) is a 9-token batch
# that takes the tensor cores on a large matrix


def _cols_ok(quant, cols):
    return cols % (256 if quant == Q4_K else 32) == 0


@pytest.mark.parametrize("quant", FORMATS)
@pytest.mark.parametrize("m,rows,cols", ROWS_SHAPES)
def test_nibble_row_kernel_bit_exact(jkb, oracle, quant, m, rows, cols):
    if not _cols_ok(quant, cols):
        pytest.skip("cols not a multiple of the Q4_K_M block")
    wb = _weights(oracle, quant, rows, cols, 70 + rows)
    act = oracle.normal(m * cols, 80 + m, 1.0)
    nm = _matrix(jkb, quant, wb, rows, cols)
    got = _gemm(jkb, nm, act, m, cols, rows)
    ref = _oracle(oracle, quant, wb, rows, cols, act, m)
    assert np.array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("quant", [Q4_0, IQ4_NL])
def test_nibble_unaligned_scale_rows_take_row_kernel(jkb, oracle, quant):
    """Q4_0 / IQ4_NL with cols % 256 != 0: the f16 scale rows are not 16-byte multiples, so even
    large batches run the row kernel -- bit for bit in the default epilogue."""
    m, rows, cols = 48, 96, 384
    wb = _weights(oracle, quant, rows, cols, 61)
    act = oracle.normal(m * cols, 62, 1.0)
    got = _gemm(jkb, _matrix(jkb, quant, wb, rows, cols), act, m, cols, rows)
    assert np.array_equal(bits(got), bits(_oracle(oracle, quant, wb, rows, cols, act, m)))


@pytest.mark.parametrize("quant", FORMATS)
@pytest.mark.parametrize("m,rows,cols", TC_SHAPES)
def test_nibble_tc_bit_exact(jkb, oracle, quant, m, rows, cols):
    if not _cols_ok(quant, cols):
        pytest.skip("cols not a multiple of the Q4_K_M block")
    wb = _weights(oracle, quant, rows, cols, 90 + rows)
    act = oracle.normal(m * cols, 91 + m, 1.0)
    nm = _matrix(jkb, quant, wb, rows, cols)
    with jkb.gemm_exact():
        got = _gemm(jkb, nm, act, m, cols, rows)
    ref = _oracle(oracle, quant, wb, rows, cols, act, m)
    assert np.array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("quant", FORMATS)
@pytest.mark.parametrize("m,rows,cols", TC_SHAPES[:4])
def test_nibble_tc_default_within_tolerance(jkb, oracle, quant, m, rows, cols):
    if not _cols_ok(quant, cols):
        pytest.skip("cols not a multiple of the Q4_K_M block")
    wb = _weights(oracle, quant, rows, cols, 90 + rows)
    act = oracle.normal(m * cols, 91 + m, 1.0)
    nm = _matrix(jkb, quant, wb, rows, cols)
    got = _gemm(jkb, nm, act, m, cols, rows)
    ref = _oracle(oracle, quant, wb, rows, cols, act, m)
    assert_gemm_close(got, ref, _bound(oracle, quant, wb, rows, cols, act, m))


@pytest.mark.parametrize("quant", [Q4_0, Q4_K])
def test_nibble_matches_repacked_gemm(jkb, oracle, quant):
    """Same weights, same activation: PackedNibbleMatrix::gemm == gemm_repacked bit for bit in
    the exact epilogue (both tensor-core paths) and on the row kernel vs the dp4a path."""
    rows, cols = 300, 1024
    wb = _weights(oracle, quant, rows, cols, 11)
    nm = _matrix(jkb, quant, wb, rows, cols)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], wb), rows, cols)
    for m in (7, 64, 200):
        act = oracle.normal(m * cols, 12 + m, 1.0)
        a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
        o1 = torch.empty(m * rows, device="cuda")
        o2 = torch.empty(m * rows, device="cuda")
        with jkb.gemm_exact():
            nm.gemm(o1, a)
            rw.gemm(o2, a)
        assert np.array_equal(bits(host(o1)), bits(host(o2))), m
    assert jkb.device_status() == 0


@pytest.mark.parametrize("quant", FORMATS)
def test_nibble_gemm_rows_and_gemv(jkb, oracle, quant):
    rows, cols = 203, 512
    wb = _weights(oracle, quant, rows, cols, 21)
    nm = _matrix(jkb, quant, wb, rows, cols)
    for m in (3, 48):
        act = oracle.normal(m * cols, 22 + m, 1.0)
        for r in (range(0, 203), range(5, 200), range(130, 131), range(7, 7)):
            with jkb.gemm_exact():
                got = _gemm(jkb, nm, act, m, cols, rows, r)
            if len(r):
                ref = _oracle(oracle, quant, wb, rows, cols, act, m, r.start, r.stop)
                assert np.array_equal(bits(got), bits(ref)), (m, r)
    act = oracle.normal(cols, 5, 1.0)
    a = jkb.QuantizedActQ8.quantize(dev(act), 1, cols)
    out = torch.empty(rows, device="cuda")
    nm.gemv(out, a)
    assert np.array_equal(bits(host(out)), bits(_oracle(oracle, quant, wb, rows, cols, act, 1)[0]))
    a2 = jkb.QuantizedActQ8.quantize(dev(oracle.normal(2 * cols, 6, 1.0)), 2, cols)
    with pytest.raises(jkb.TensorBoundsError) as e:
        nm.gemv(torch.empty(2 * rows, device="cuda"), a2)
    assert "gemv requires act.m() == 1, got 2" in e.value.reason
    with pytest.raises(jkb.TensorBoundsError):
        nm.gemm_rows(torch.empty(3 * rows, device="cuda"), a2, range(0, 204))
    with pytest.raises(jkb.TensorBoundsError):
        nm.gemm(torch.empty(2 * rows + 1, device="cuda"), a2)
    a3 = jkb.QuantizedActQ8.quantize(dev(oracle.normal(2 * 256, 6, 1.0)), 2, 256)
    with pytest.raises(jkb.TensorBoundsError) as e:
        nm.gemm(torch.empty(2 * rows, device="cuda"), a3)
    assert "activation K (256) != weight cols (512)" in e.value.reason


@pytest.mark.parametrize("quant", FORMATS)
def test_nibble_footprint_and_dequantize_row(jkb, oracle, quant):
    """packed_bytes == raw_tensor_bytes (1.00x); dequantize_row matches the reference's, bit for
    bit, including blocks whose scale is 0, -0, Inf or NaN."""
    rows, cols = 203, 512
    raw = R.fill_pseudo_quant_tensor(quant, rows, cols)
    be, bb = {Q4_0: (32, 18), Q4_1: (32, 20), IQ4_NL: (32, 18), Q4_K: (256, 144)}[quant]
    blocks = raw.reshape(rows, cols // be, bb)
    for (r, b), h in zip([(1, 0), (4, 1), (8, 0), (9, 1)], [0x7C00, 0x7E01, 0x0000, 0x8000]):
        blocks[r, b, 0:2] = [h & 0xFF, h >> 8]
    raw = blocks.reshape(-1)
    nm = _matrix(jkb, quant, raw, rows, cols)
    assert nm.packed_bytes() == nm.raw_tensor_bytes() == raw.nbytes
    assert nm.n_tiles == 26 and nm.k_blocks32 == cols // 32
    q, ws, wm = oracle.nibble_decode(quant, raw, rows, cols)
    out = torch.empty(cols, device="cuda")
    for r in (0, 1, 4, 8, 9, 100, 202):
        nm.dequantize_row(r, out)
        ref = oracle.nibble_dequantize_row(quant, q, ws, wm, cols, r)
        assert np.array_equal(bits(host(out)), bits(ref)), r
    with pytest.raises(jkb.TensorBoundsError):
        nm.dequantize_row(203, out)
    with pytest.raises(jkb.TensorBoundsError):
        nm.dequantize_row(0, torch.empty(cols - 1, device="cuda"))


@pytest.mark.parametrize("quant", FORMATS)
def test_nibble_tile_buffers_roundtrip(jkb, oracle, quant):
    """Matrices built from the reference's tile buffers (the library's host packer and the
    oracle's) equal the one built from the tensor; the zero-scale blocks the packer zeroes do
    not change any output."""
    rows, cols = 203, 512
    wb = _weights(oracle, quant, rows, cols, 31)
    view = jkb.TensorView("w", quant, [cols, rows], wb)
    nm = jkb.PackedNibbleMatrix.from_tensor(view, rows, cols)
    tiles, sc, mn, hd = jkb.repack_nibble_into_tile_range(view, rows, cols, range(0, 26))
    if quant == Q4_1:
        pytest.skip("the reference has no buffer constructor for Q4_1")
    if quant == Q4_K:
        nb = jkb.PackedNibbleMatrix.from_q4_k_buffers(rows, cols, tiles, hd)
    else:
        nb = jkb.PackedNibbleMatrix.from_scale_f16_buffers(quant, rows, cols, tiles, sc)
    for m in (9, 64):
        act = oracle.normal(m * cols, 33 + m, 1.0)
        with jkb.gemm_exact():
            g1 = _gemm(jkb, nm, act, m, cols, rows)
            g2 = _gemm(jkb, nb, act, m, cols, rows)
        assert np.array_equal(bits(g1), bits(g2))


def test_gemm_ime_entry_points_check_format(jkb, oracle):
    """gemm_q4_0_ime / gemm_q4_k_ime (repack.rs:5140-5175, :5983-5986): the GEMM on the right
    format, CapabilityMismatch on the other."""
    rows, cols, m = 64, 512, 33
    act = oracle.normal(m * cols, 3, 1.0)
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    out = torch.empty(m * rows, device="cuda")
    for quant, right, wrong in ((Q4_0, jkb.gemm_q4_0_ime, jkb.gemm_q4_k_ime),
                                (Q4_K, jkb.gemm_q4_k_ime, jkb.gemm_q4_0_ime)):
        wb = _weights(oracle, quant, rows, cols, 4)
        nm = _matrix(jkb, quant, wb, rows, cols)
        with jkb.gemm_exact():
            right(out, nm, a)
        ref = _oracle(oracle, quant, wb, rows, cols, act, m)
        assert np.array_equal(bits(host(out).reshape(m, rows)), bits(ref))
        with pytest.raises(jkb.CapabilityMismatch):
            wrong(out, nm, a)
