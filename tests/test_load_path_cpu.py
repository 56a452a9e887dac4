"""The parallel load path's host side, which needs no GPU: block_scaled_layout
(repack.rs:2372, BlockScaledTileLayout::for_tensor :1308-1366), repack_into_tile_range (:1579)
and repack_q4_k_m_parallel_slices (:1659), through the C ABI.

* Every one of the 14 block-scaled formats, on a row count that leaves the last 8-row tile
  ragged: the tiles, scales and mins equal the oracle's repacked values (repack.rs:1724-2103,
  restated row-major in oracle/) placed in the reference's tile layout -- tiles
  [n_tile][k_chunk][8 rows][16 K values], scales and mins [n_tile][scale_group][8] -- bit for bit,
  with zero rows past the matrix.
* Tile ranges stitch: disjoint ranges filled separately (as the reference's worker threads do,
  tests/wave3_prefill_gqa_and_gemm.rs:281-363) concatenate to the whole range.
* Validation fails closed like the reference: ranges past n_tiles, wrong slice lengths, a
  missing mins slice, dense or non-Q4_K_M formats.
* QuantizedActQ8View::scratch_bytes_for_row (repack.rs:827) on the host."""
import ctypes as C

import numpy as np
import pytest

import refgen as R

ALL = [2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 20, 34, 35, 36]
NAMES = {2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 10: "Q2_K", 11: "Q3_K",
         12: "Q4_K_M", 13: "Q5_K", 14: "Q6_K", 20: "IQ4_NL", 34: "TQ1_0", 35: "TQ2_0",
         36: "I2_S"}


@pytest.fixture(scope="module")
def jkb():
    import jkb200

    return jkb200


def weights(oracle, quant, rows, cols, seed):
    if quant in (34, 35):
        return oracle.pack_ternary(quant, oracle.ternary(rows * cols, seed), rows, cols, 0.0173)
    if quant in (7, 10, 11, 36):
        return R.build_synthetic_quant_tensor(quant, rows, cols, seed)
    return oracle.quantize_weights(quant, oracle.normal(rows * cols, seed, 0.02), rows, cols)


def tiles_of(q, s, mn, rows, t0, t1):
    """The oracle's row-major repack in the reference's tile layout, tiles t0..t1."""
    kp, sg = q.shape[1], s.shape[1]
    n = t1 - t0
    qp = np.zeros((n * 8, kp), np.int8)
    sp = np.zeros((n * 8, sg), np.float32)
    mp = np.zeros((n * 8, sg), np.float32)
    r0, r1 = t0 * 8, min(t1 * 8, rows)
    qp[:r1 - r0] = q[r0:r1]
    sp[:r1 - r0] = s[r0:r1]
    if mn is not None:
        mp[:r1 - r0] = mn[r0:r1]
    tiles = qp.reshape(n, 8, kp // 16, 16).transpose(0, 2, 1, 3).reshape(n * (kp // 16), 128)
    sc = sp.reshape(n, 8, sg).transpose(0, 2, 1).reshape(-1)
    mins = mp.reshape(n, 8, sg).transpose(0, 2, 1).reshape(-1) if mn is not None else None
    return tiles.view(np.uint8), sc, mins


@pytest.mark.parametrize("quant", ALL, ids=[NAMES[q] for q in ALL])
def test_layout_and_tile_ranges_match_oracle(jkb, oracle, quant):
    rows, cols = 37, 512
    raw = weights(oracle, quant, rows, cols, 3 + quant)
    view = jkb.TensorView("w", quant, [rows, cols], raw)
    L = jkb.block_scaled_layout(view, rows, cols)
    ge = 16 if quant in (10, 11, 14) else 32
    assert (L.rows, L.cols, L.k_padded, L.n_tiles, L.k_chunks) == (rows, cols, 512, 5, 32)
    assert (L.chunks_per_scale, L.scale_groups) == (ge // 16, 512 // ge)
    assert L.has_mins == (quant in (3, 7, 10, 12, 13))
    assert L.total_tiles == 5 * 32 and L.total_scales == 5 * (512 // ge) * 8
    assert L.total_mins == (L.total_scales if L.has_mins else 0)
    assert L.row_bytes == raw[:rows * L.row_bytes].size // rows
    q, s, mn = oracle.repack_block_scaled(quant, raw, rows, cols)
    full = jkb.repack_into_tile_range(view, rows, cols, range(0, 5))
    want = tiles_of(q, s, mn, rows, 0, 5)
    assert np.array_equal(full[0], want[0])
    assert np.array_equal(full[1].view(np.uint32), want[1].view(np.uint32))
    if L.has_mins:
        assert np.array_equal(full[2].view(np.uint32), want[2].view(np.uint32))
    else:
        assert full[2] is None
    # disjoint ranges stitch to the whole, the empty range writes nothing
    parts = [jkb.repack_into_tile_range(view, rows, cols, r)
             for r in (range(0, 2), range(2, 2), range(2, 5))]
    assert np.array_equal(np.concatenate([p[0] for p in parts]), full[0])
    assert np.array_equal(np.concatenate([p[1] for p in parts]), full[1])


def test_q4_k_m_parallel_slices(jkb, oracle):
    rows, cols = 21, 1024
    raw = weights(oracle, 12, rows, cols, 9)
    view = jkb.TensorView("w", 12, [rows, cols], raw)
    L = jkb.block_scaled_layout(view, rows, cols)
    tiles = np.full(2 * L.k_chunks * 128, 0x55, np.int8)
    sc = np.full(2 * L.scale_groups * 8, np.nan, np.float32)
    mn = np.full(2 * L.scale_groups * 8, np.nan, np.float32)
    jkb.repack_q4_k_m_parallel_slices(view, rows, cols, range(1, 3), tiles, sc, mn)
    q, s, m = oracle.repack_block_scaled(12, raw, rows, cols)
    want = tiles_of(q, s, m, rows, 1, 3)
    assert np.array_equal(tiles.view(np.uint8).reshape(-1, 128), want[0])
    assert np.array_equal(sc.view(np.uint32), want[1].view(np.uint32))
    assert np.array_equal(mn.view(np.uint32), want[2].view(np.uint32))
    other = jkb.TensorView("w8", 8, [rows, cols], weights(oracle, 8, rows, cols, 1))
    with pytest.raises(jkb.CapabilityMismatch):
        jkb.repack_q4_k_m_parallel_slices(other, rows, cols, range(0, 1), tiles, sc, mn)
    with pytest.raises(jkb.TensorBoundsError, match="parallel slice lengths"):
        jkb.repack_q4_k_m_parallel_slices(view, rows, cols, range(0, 1), tiles, sc, mn)


def test_tile_range_validation_fails_closed(jkb, oracle):
    rows, cols = 37, 512
    view = jkb.TensorView("w", 12, [rows, cols], weights(oracle, 12, rows, cols, 4))
    with pytest.raises(jkb.TensorBoundsError, match="exceeds n_tiles"):
        jkb.repack_into_tile_range(view, rows, cols, range(3, 6))
    tiles = np.full((32, 128), 7, np.uint8)
    sc = np.zeros(16 * 8, np.float32)
    with pytest.raises(jkb.TensorBoundsError, match="tile/scale slice lengths"):
        jkb.repack_into_tile_range(view, rows, cols, range(0, 2), tiles, sc, np.zeros(128))
    with pytest.raises(jkb.TensorBoundsError, match="requires out_mins"):
        from jkb200 import _lib

        v = view._c()
        rc = _lib.load().jkb_repack_into_tile_range(C.byref(v), rows, cols, 0, 1,
                                                    tiles.ctypes.data, 32, sc.ctypes.data, 128,
                                                    None, 0)
        from jkb200.api import _check

        _check(rc)
    assert np.all(tiles == 7)  # nothing written on failure
    dense = jkb.TensorView("f", 0, [4, 32], np.zeros(4 * 32 * 4, np.uint8))
    with pytest.raises(jkb.CapabilityMismatch):
        jkb.block_scaled_layout(dense, 4, 32)
    with pytest.raises(jkb.TensorBoundsError):
        jkb.block_scaled_layout(view, rows + 1, cols)  # byte length does not match


def test_view_scratch_bytes_for_row(jkb):
    from jkb200 import _lib

    f = _lib.load().jkb_act_q8_view_scratch_bytes_for_row
    assert f(0) == 0

    def up(n):
        return (n + 127) // 128 * 128

    for k in (1, 31, 32, 256, 4096, 4100, 14336):
        kp = (k + 31) // 32 * 32
        assert f(k) == 128 + up(kp) + 2 * up(kp // 32 * 4) + up(kp // 16 * 4) + \
            up((k + 255) // 256 * 4)
