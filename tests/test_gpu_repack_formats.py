"""RepackedWeight for the formats that exist on the reference's hot path only as repacked GEMM
weights -- Q4_1, Q5_1, IQ4_NL (32-element groups, the first two with mins), Q3_K and Q2_K
(16-element groups, Q2_K with mins) -- against the CPU oracle (repack.rs:1814-1911,
quant.rs:118-356):
* the repacked planes (i8 values, scales, mins) bit for bit;
* RepackedWeight::dequantize_row (repack.rs:2529-2598) bit for bit against scale * q - min, and
  within 1e-4 of the block dequantizers as the reference's test asks;
* the GEMM bit for bit in the exact epilogue (dp4a kernel below 32 tokens and for Q2_K,
  tensor cores otherwise) and within the tolerance contract by default;
* the reference's wave-2 contract (tests/test_repack_gemv_gemm.rs:919-997) on its own synthetic
  tensors and activations: cosine > 0.999 and the per-format relative l2 bound."""
import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import assert_gemm_close, bits, dev, gemm_abs_bound, host

pytestmark = pytest.mark.gpu

Q4_1, Q5_1, Q2_K, Q3_K, IQ4_NL = 3, 7, 10, 11, 20
FORMATS = [Q4_1, Q5_1, IQ4_NL, Q3_K, Q2_K]


def _tensor(quant, rows, cols, seed):
    if rows <= 64:
        return R.build_synthetic_quant_tensor(quant, rows, cols, seed)
    # larger matrices: the generator's bytes for a 23-row pool, tiled (values do not matter for
    # parity, and the pool keeps the Python generator fast)
    pool = R.build_synthetic_quant_tensor(quant, 23, cols, seed).reshape(23, -1)
    return np.ascontiguousarray(np.resize(pool, (rows, pool.shape[1]))).reshape(-1)


def _repacked(jkb, quant, raw, rows, cols):
    return jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [cols, rows], raw), rows,
                                          cols)


@pytest.mark.parametrize("quant", FORMATS)
def test_repack_planes_and_dequantize_row(jkb, oracle, quant):
    rows, cols = 37, 512
    raw = _tensor(quant, rows, cols, 5)
    rw = _repacked(jkb, quant, raw, rows, cols)
    q, s, mn = rw.buffers()
    rq, rs, rmn = oracle.repack_block_scaled(quant, raw, rows, cols)
    assert np.array_equal(host(q), rq)
    assert np.array_equal(bits(host(s)), bits(rs))
    assert (mn is None) == (rmn is None)
    if rmn is not None:
        assert np.array_equal(bits(host(mn)), bits(rmn))
    gsz = rq.shape[1] // rs.shape[1]
    expect = (np.repeat(rs, gsz, axis=1) * rq.astype(np.float32)).astype(np.float32)
    if rmn is not None:
        expect = (expect - np.repeat(rmn, gsz, axis=1)).astype(np.float32)
    deq = oracle.dequantize_rows(quant, raw, rows, cols)
    for r in (0, 17, rows - 1):
        got = host(rw.dequantize_row(r))
        assert np.array_equal(bits(got), bits(expect[r, :cols]))
        assert np.all(np.abs(got - deq[r]) < 1e-4)
    with pytest.raises(jkb.TensorBoundsError, match="invalid row"):
        rw.dequantize_row(rows)
    rw.destroy()


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("m,rows,cols", [(5, 40, 512), (33, 300, 4096), (200, 257, 1024)])
@pytest.mark.parametrize("quant", FORMATS)
def test_repacked_gemm(jkb, oracle, quant, m, rows, cols, exact):
    raw = _tensor(quant, rows, cols, 9)
    rw = _repacked(jkb, quant, raw, rows, cols)
    act = oracle.normal(m * cols, 70 + m, 1.0)
    a = jkb.QuantizedActQ8.quantize(dev(act), m, cols)
    out = torch.full((m * rows,), float("nan"), dtype=torch.float32, device="cuda")
    with jkb.gemm_exact(exact):
        rw.gemm(out, a)
    got = host(out).reshape(m, rows)
    assert jkb.device_status() == 0
    q, s, mn = oracle.repack_block_scaled(quant, raw, rows, cols)
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(act, m, cols)
    ref = oracle.gemm_repacked(quant, q, s, mn, rows, cols, xq, xs, xsum, xs16, m, nthreads=8)
    if exact:
        assert np.array_equal(bits(got), bits(ref))
    else:
        assert_gemm_close(got, ref, gemm_abs_bound(oracle, quant, raw, rows, cols, act, m))
    rw.destroy()


WAVE2 = [(Q4_1, 256, 19, 1.5e-2, 0), (Q5_1, 256, 17, 1.5e-2, 2), (Q2_K, 512, 15, 2.0e-2, 3),
         (Q3_K, 512, 19, 1.5e-2, 4), (IQ4_NL, 256, 23, 1.5e-2, 5)]


@pytest.mark.parametrize("quant,cols,rows,max_rel,q_idx", WAVE2)
def test_wave2_contract_on_gpu(jkb, oracle, quant, cols, rows, max_rel, q_idx):
    """tests/test_repack_gemv_gemm.rs:919-997: the test's own tensors (seed q_idx + 17, q_idx
    the format's position in its list) and activations, through the GPU repack and GEMM."""
    raw = R.build_synthetic_quant_tensor(quant, rows, cols, q_idx + 17)
    rw = _repacked(jkb, quant, raw, rows, cols)
    deq = oracle.dequantize_rows(quant, raw, rows, cols)
    for r in (0, rows // 2, rows - 1):
        assert np.all(np.abs(host(rw.dequantize_row(r)) - deq[r]) < 1e-4)
    for m in (1, 5, 8, 17, 64):
        x = R.make_activations(m, cols, 300 + q_idx * 10 + m)
        a = jkb.QuantizedActQ8.quantize(dev(x), m, cols)
        out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
        rw.gemm(out, a)
        want = x.reshape(m, cols).astype(np.float64) @ deq.astype(np.float64).T
        cos, rel = R.cosine_and_rel_l2(host(out).reshape(m, rows), want)
        assert cos > 0.999 and rel < max_rel, (m, cos, rel)
    rw.destroy()


def test_new_formats_have_no_gemv_layout(jkb):
    """The reference has no Q8 block dot for these formats: the GEMV handle refuses them."""
    for quant, (be, bb) in ((Q4_1, (32, 20)), (Q5_1, (32, 24)), (Q2_K, (256, 84)),
                            (Q3_K, (256, 110)), (IQ4_NL, (32, 18))):
        raw = np.zeros(4 * (256 // be) * bb, np.uint8)
        with pytest.raises(jkb.CapabilityMismatch):
            jkb.Weight(jkb.TensorView("w", quant, [256, 4], raw), 4, 256)
