"""The public repack.rs / quant_q8.rs entry points around the repacked GEMM, on the GPU against
the CPU oracle (every comparison bit for bit unless it says otherwise):

* RepackedWeight::from_tile_buffers (repack.rs:2386) on the tiles of repack_into_tile_range
  (:1579) equals RepackedWeight::from_tensor for all 14 formats -- planes and exact GEMM -- and
  rejects buffers that do not match the layout;
* quantize_row_f32_to_q8_32 (repack.rs:441) equals quantize_block32_scalar per block
  (quants, scales, sequential sums; ragged tail, non-finite inputs, an unaligned quant buffer);
* scratch arenas: quantize_row_q8_0 / q8_k _in_scratch / _in_scope (quant_q8.rs:405-444,
  :602-641) equal quantize_row_q8_0 / q8_k, failures leave the cursor untouched, scopes rewind
  (the reference's own contract, quant_q8.rs:3771-3826);
* QuantizedActQ8View::quantize_row_in_scratch / _in_scope (repack.rs:870, :969) equal
  QuantizedActQ8::quantize_row, fit in scratch_bytes_for_row, and feed gemv_repacked_view /
  _view_rows (:4030, :4045) and RepackedWeight::gemv_view(_rows), which equal the oracle's
  gemm_repacked at m = 1; QuantizedActQ8::as_view (:708) gives the same result;
* gemv_repacked_f32 / _rows (:4101, :4114) and gemm_repacked_f32_rows (:4143) equal the oracle
  on their row ranges (exact epilogue for the tensor-core batch)."""
import numpy as np
import pytest
import torch

from gpuutil import bits, dev, host
from test_load_path_cpu import ALL, NAMES, weights

pytestmark = pytest.mark.gpu


def _oracle_rows(oracle, quant, raw, rows, cols, x, m, r0=0, r1=None):
    q, s, mn = oracle.repack_block_scaled(quant, raw, rows, cols)
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(x, m, cols)
    return oracle.gemm_repacked(quant, q, s, mn, rows, cols, xq, xs, xsum, xs16, m, r0, r1,
                                nthreads=8)


@pytest.mark.parametrize("quant", ALL, ids=[NAMES[q] for q in ALL])
def test_from_tile_buffers_equals_from_tensor(jkb, oracle, quant):
    rows, cols = 45, 1024
    raw = weights(oracle, quant, rows, cols, 11 + quant)
    view = jkb.TensorView("w", quant, [rows, cols], raw)
    L = jkb.block_scaled_layout(view, rows, cols)
    # two "workers" fill disjoint tile ranges of the same host buffers
    tiles = np.zeros((L.total_tiles, 128), np.uint8)
    sc = np.zeros(L.total_scales, np.float32)
    mn = np.zeros(L.total_mins, np.float32) if L.has_mins else None
    for r in (range(0, 2), range(2, L.n_tiles)):
        t0, t1 = r.start * L.k_chunks, r.stop * L.k_chunks
        s0, s1 = r.start * L.scale_groups * 8, r.stop * L.scale_groups * 8
        jkb.repack_into_tile_range(view, rows, cols, r, tiles[t0:t1], sc[s0:s1],
                                   None if mn is None else mn[s0:s1])
    a = jkb.RepackedWeight.from_tile_buffers(L, tiles, sc, mn)
    b = jkb.RepackedWeight.from_tensor(view, rows, cols)
    for pa, pb in zip(a.buffers(), b.buffers()):
        assert (pa is None) == (pb is None)
        if pa is not None:
            assert np.array_equal(host(pa).view(np.uint8), host(pb).view(np.uint8))
    m = 40
    x = oracle.normal(m * cols, 21, 1.0)
    act = jkb.QuantizedActQ8.quantize(dev(x), m, cols)
    out = torch.full((m * rows,), float("nan"), dtype=torch.float32, device="cuda")
    with jkb.gemm_exact():
        a.gemm(out, act)
    ref = _oracle_rows(oracle, quant, raw, rows, cols, x, m)
    assert np.array_equal(bits(host(out).reshape(m, rows)), bits(ref))
    assert jkb.device_status() == 0
    a.destroy()
    b.destroy()


def test_from_tile_buffers_validation(jkb, oracle):
    rows, cols = 16, 512
    view = jkb.TensorView("w", 12, [rows, cols], weights(oracle, 12, rows, cols, 2))
    L = jkb.block_scaled_layout(view, rows, cols)
    tiles, sc, mn = jkb.repack_into_tile_range(view, rows, cols, range(0, L.n_tiles))
    with pytest.raises(jkb.TensorBoundsError, match="buffer lengths"):
        jkb.RepackedWeight.from_tile_buffers(L, tiles[:-1], sc, mn)
    with pytest.raises(jkb.TensorBoundsError, match="requires mins buffer"):
        jkb.RepackedWeight.from_tile_buffers(L, tiles, sc, None)
    v8 = jkb.TensorView("w8", 8, [rows, cols], weights(oracle, 8, rows, cols, 3))
    L8 = jkb.block_scaled_layout(v8, rows, cols)
    t8, s8, _ = jkb.repack_into_tile_range(v8, rows, cols, range(0, L8.n_tiles))
    with pytest.raises(jkb.TensorBoundsError, match="does not use mins"):
        jkb.RepackedWeight.from_tile_buffers(L8, t8, s8, np.zeros(L8.total_scales, np.float32))
    L8._c.k_chunks += 1  # a layout no block_scaled_layout call produced
    with pytest.raises(jkb.TensorBoundsError, match="layout fields"):
        jkb.RepackedWeight.from_tile_buffers(L8, t8, s8)


@pytest.mark.parametrize("n", [32, 77, 4096, 14336])
def test_quantize_row_f32_to_q8_32(jkb, oracle, n):
    x = oracle.normal(n, 31 + n, 1.0)
    x[3] = np.nan
    x[n // 2] = np.inf
    x[n - 1] = -np.inf
    blocks = (n + 31) // 32
    q_all = torch.full((blocks * 32 + 1,), 99, dtype=torch.int8, device="cuda")
    q = q_all[1:]  # an unaligned quant buffer (byte stores)
    sc = torch.empty(blocks, dtype=torch.float32, device="cuda")
    sm = torch.empty(blocks, dtype=torch.float32, device="cuda")
    jkb.quantize_row_f32_to_q8_32(dev(x), q, sc, sm)
    xq, xs, xsum, _, _ = oracle.act_q8_quantize(x, 1, n)
    assert np.array_equal(host(q), xq[0])
    assert np.array_equal(bits(host(sc)), bits(xs[0]))
    assert np.array_equal(bits(host(sm)), bits(xsum[0]))
    with pytest.raises(jkb.TensorBoundsError, match="insufficient Q8 output buffers"):
        jkb.quantize_row_f32_to_q8_32(dev(x), q[:-1], sc, sm)
    with pytest.raises(jkb.TensorBoundsError, match="non-empty"):
        jkb.quantize_row_f32_to_q8_32(torch.empty(0, device="cuda"), q, sc, sm)


def test_scratch_quantizers_match_and_fail_closed(jkb, oracle):
    x0 = oracle.normal(64, 1, 1.0)
    x0[5] = np.nan
    xk = oracle.normal(256, 3, 1.0)
    xk[7] = -np.inf
    e0, ek = oracle.quantize_row_q8_0(x0), oracle.quantize_row_q8_k(xk)
    ws = jkb.ScratchWorkspace(2048)
    with ws.scope() as scope:
        s0 = jkb.quantize_row_q8_0_in_scope(dev(x0), scope)
        sk = jkb.quantize_row_q8_k_in_scope(dev(xk), scope)
        assert np.array_equal(host(s0), e0.view(np.uint8).reshape(-1))
        assert np.array_equal(host(sk), ek.view(np.uint8).reshape(-1))
        assert s0.data_ptr() % 128 == 0 and sk.data_ptr() % 128 == 0
        assert ws.used_bytes() == 128 + 292
    assert ws.used_bytes() == 0  # the scope rewound
    ws.reset()
    a = jkb.quantize_row_q8_0_in_scratch(dev(x0), ws)
    assert np.array_equal(host(a), e0.view(np.uint8).reshape(-1))
    ws.reset()
    b = jkb.quantize_row_q8_k_in_scratch(dev(xk), ws)
    assert np.array_equal(host(b), ek.view(np.uint8).reshape(-1))
    ws.reset()
    for fn, bad in ((jkb.quantize_row_q8_0_in_scratch, torch.empty(0, device="cuda")),
                    (jkb.quantize_row_q8_0_in_scratch, torch.ones(31, device="cuda")),
                    (jkb.quantize_row_q8_k_in_scratch, torch.ones(128, device="cuda"))):
        with pytest.raises(jkb.TensorBoundsError):
            fn(bad, ws)
    assert ws.used_bytes() == 0
    tiny = jkb.ScratchWorkspace(16)
    with pytest.raises(jkb.TensorBoundsError, match="scratch exhausted"):
        jkb.quantize_row_q8_0_in_scratch(dev(x0), tiny)
    assert tiny.used_bytes() == 0
    # an arena over caller-owned memory allocates nothing on the device
    region = torch.empty(4096, dtype=torch.uint8, device="cuda")
    wrapped = jkb.ScratchWorkspace(wrap=region)
    c = jkb.quantize_row_q8_0_in_scratch(dev(x0), wrapped)
    assert c.data_ptr() == region.data_ptr()
    assert np.array_equal(host(region[:72]), e0.view(np.uint8).reshape(-1))
    for w in (ws, tiny, wrapped):
        w.destroy()


@pytest.mark.parametrize("quant,rows,cols", [(8, 300, 4096), (12, 200, 2048), (14, 96, 1024),
                                             (2, 70, 4100 // 32 * 32), (35, 64, 2560)])
def test_view_in_scratch_and_gemv_view(jkb, oracle, quant, rows, cols):
    raw = weights(oracle, quant, rows, cols, 5)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], raw), rows, cols)
    x = oracle.normal(cols, 6, 1.0)
    x[1] = np.nan
    need = jkb.QuantizedActQ8View.scratch_bytes_for_row(cols)
    ws = jkb.ScratchWorkspace(need)
    view = jkb.QuantizedActQ8View.quantize_row_in_scratch(dev(x), ws)
    assert (view.m, view.k) == (1, cols) and ws.used_bytes() <= need
    act = jkb.QuantizedActQ8.quantize(dev(x), 1, cols)
    for pv, pa in zip(view.buffers(), act.buffers()):
        assert np.array_equal(host(pv).view(np.uint8), host(pa).view(np.uint8))
    ref = _oracle_rows(oracle, quant, raw, rows, cols, x, 1)[0]
    out = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    jkb.gemv_repacked_view(out, rw, view)
    assert np.array_equal(bits(host(out)), bits(ref))
    out.fill_(float("nan"))
    rw.gemv_view(out, act.as_view())
    assert np.array_equal(bits(host(out)), bits(ref))
    part = torch.empty(rows - 17, dtype=torch.float32, device="cuda")
    rw.gemv_view_rows(part, view, range(10, rows - 7))
    assert np.array_equal(bits(host(part)), bits(ref[10:rows - 7]))
    with pytest.raises(jkb.TensorBoundsError, match="out of bounds"):
        jkb.gemv_repacked_view_rows(part, rw, view, range(20, rows + 3))
    # the scope form rewinds
    ws.reset()
    with ws.scope() as sc:
        v2 = jkb.QuantizedActQ8View.quantize_row_in_scope(dev(x), sc)
        out.fill_(float("nan"))
        jkb.gemv_repacked_view(out, rw, v2)
        assert np.array_equal(bits(host(out)), bits(ref))
    assert ws.used_bytes() == 0
    # the planes need `need` bytes at worst (an unaligned cursor, the last plane padded);
    # from an aligned start exactly the planes' bytes, one byte fewer fails
    kp = (cols + 31) // 32 * 32
    up = lambda n: (n + 127) // 128 * 128  # noqa: E731
    exact = up(kp) + 2 * up(kp // 32 * 4) + up(kp // 16 * 4) + (cols + 255) // 256 * 4
    small = jkb.ScratchWorkspace(exact - 1)
    with pytest.raises(jkb.TensorBoundsError, match="scratch exhausted"):
        jkb.QuantizedActQ8View.quantize_row_in_scratch(dev(x), small)
    assert small.used_bytes() == 0
    batch = jkb.QuantizedActQ8.quantize(dev(np.concatenate([x, x])), 2, cols)
    with pytest.raises(jkb.TensorBoundsError, match="act.m\\(\\) == 1"):
        jkb.gemv_repacked_view(out, rw, batch.as_view())
    for h in (rw, ws, small, act, batch):
        h.destroy()


@pytest.mark.parametrize("quant", [8, 12, 14])
def test_f32_convenience_entries(jkb, oracle, quant):
    rows, cols, m = 160, 2048, 48
    raw = weights(oracle, quant, rows, cols, 8)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], raw), rows, cols)
    x = oracle.normal(m * cols, 9, 1.0)
    scratch = jkb.QuantizedActQ8(m, cols)
    ref1 = _oracle_rows(oracle, quant, raw, rows, cols, x[:cols], 1)[0]
    out = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    jkb.gemv_repacked_f32(out, rw, dev(x[:cols]), scratch)
    assert np.array_equal(bits(host(out)), bits(ref1))
    part = torch.empty(100, dtype=torch.float32, device="cuda")
    jkb.gemv_repacked_f32_rows(part, rw, dev(x[:cols]), range(33, 133), scratch)
    assert np.array_equal(bits(host(part)), bits(ref1[33:133]))
    with pytest.raises(jkb.TensorBoundsError, match="activation k"):
        jkb.gemv_repacked_f32(out, rw, dev(x[:cols - 32]), scratch)
    r0, r1 = 7, 151
    outm = torch.full((m * (r1 - r0),), float("nan"), dtype=torch.float32, device="cuda")
    with jkb.gemm_exact():
        jkb.gemm_repacked_f32_rows(outm, rw, dev(x), m, range(r0, r1), scratch)
    refm = _oracle_rows(oracle, quant, raw, rows, cols, x, m, r0, r1)
    assert np.array_equal(bits(host(outm).reshape(m, r1 - r0)), bits(refm))
    assert jkb.device_status() == 0
    with pytest.raises(jkb.TensorBoundsError, match="input length"):
        jkb.gemm_repacked_f32_rows(outm, rw, dev(x[:-1]), m, range(r0, r1), scratch)
    rw.destroy()
    scratch.destroy()
