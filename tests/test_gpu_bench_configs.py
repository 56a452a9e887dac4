"""Parity at exactly the configurations bench.py times, through the entry points it times them
with (BASELINE configs[0] to configs[4]).

* configs[1], the Llama-3-8B decode set: one step of bench.DecodeSet -- q/k/v and gate/up as
  grouped f32-input launches (vec_dot_grouped_rvv), o and down as single-item groups, the Q6_K
  lm_head (128256 x 4096) as quantize_row_q8_k + gemv_rows -- over the full-size matrices of the
  bench, two steps (both layer weight copies). Per matrix at least 64 sampled rows (the first
  and last eight, the rest seeded) against the oracle GEMV within the row tolerance, and the
  lm_head's Q8_K input bit for bit.
* configs[4], the Llama-3-70B set at batch 1 (f32-input launches) and batch 16
  (quantize_rows_q8_k + gemv_batch; and on the tensor cores, QuantizedActQ8 + gemm_repacked),
  sampled rows of every token against the oracle; and its
  row sharding over 8 ranks emulated on one GPU: each rank's slice uploaded on its own, the
  stitched outputs equal to the single-GPU call bit for bit (the multi-GPU run is in
  test_gpu_multigpu.py).
* configs[0], the Q4_0 4096 x 4096 GEMV: every block's integer sum and f32 value bit for bit
  and every row within the tolerance, through gemv_q4_0_q8_0 and vec_dot_q4_0_rvv.
* configs[2], the four Q8_0 prefill shapes M in {512, 2048} x (4096 -> 14336, 14336 -> 4096)
  through RepackedWeight.gemm on QuantizedActQ8.quantize, every token of three 32-row ranges
  (first, middle, last weight tiles): the exact epilogue bit for bit, the default within
  |err| <= 1e-5 * sum_k |x~||w~| and l2 relative error < 1e-5.

The reference's tolerance contracts: tests/wave4_quant_gemv_and_argmax.rs:397 (1e-5 on GEMV
rows), tests/wave3_prefill_gqa_and_gemm.rs:123-166 (prefill GEMM)."""
import os
import sys

import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import assert_gemm_close, bits, dev, gemm_abs_bound, host

pytestmark = pytest.mark.gpu
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402

REL = 1e-5


def _sample(rows, seed, n_rand=48):
    r = np.random.default_rng(seed).integers(0, rows, n_rand)
    return np.unique(np.concatenate([np.arange(min(8, rows)), np.arange(max(0, rows - 8), rows),
                                     r]))


def _check_rows(oracle, quant, raw, rows, cols, xq, got, sample, what):
    row_bytes = raw.size // rows
    sub = np.concatenate([raw[r * row_bytes:(r + 1) * row_bytes] for r in sample])
    y_ref = oracle.gemv(quant, sub, len(sample), cols, xq)
    _, _, v_ref = oracle.block_dots(quant, sub, len(sample), cols, xq)
    ok, worst = R.gemv_tolerance_ok(got[sample], y_ref, v_ref, REL)
    assert ok, f"{what}: worst {worst:.3g} of the row bound"
    assert R.l2_rel_err(got[sample], y_ref) < REL, what


def _decode_parity(jkb, oracle, key, batch, steps):
    spec = bench.DECODE_SETS[key]
    ds = bench.DecodeSet(jkb, spec["mats"], spec["acts"], 1, 0, peer=False, batch=batch,
                         layer_copies=spec["copies"], sigma=spec["sigma"])
    xs = {s: ds.xs[s].cpu().numpy().reshape(batch, -1) for s in spec["acts"]}
    for i in range(steps):
        ds.step(i)
        torch.cuda.synchronize()
        for j, (name, quant, rows, cols, s) in enumerate(spec["mats"]):
            c = i % (1 if name == "lm_head" else spec["copies"])
            raw = bench.synth_matrix(quant, rows, cols, 1000 + j + 97 * c, sigma=spec["sigma"])
            got = host(ds.output(name, i)).reshape(batch, rows)
            sample = _sample(rows, 31 * j + i)
            for t in range(batch):
                xq = oracle.quantize_row_q8_k(xs[s][t])
                _check_rows(oracle, quant, raw, rows, cols, xq, got[t], sample,
                            f"{key} {name} step {i} token {t}")
            if batch > 1 or s in ds.prequant:  # the bench's own Q8_K input of this stream
                ref = np.concatenate([oracle.quantize_row_q8_k(xs[s][t]).view(np.uint8)
                                      .reshape(-1) for t in range(batch)])
                assert np.array_equal(host(ds.xq[s]), ref), f"{key} {s} Q8_K input"
    assert jkb.device_status() == 0
    ds.destroy()


def test_decode_8b_step_matches_oracle(jkb, oracle):
    """configs[1] at its full size through the bench's launches, both layer weight copies."""
    _decode_parity(jkb, oracle, "8b", 1, 2)


@pytest.mark.parametrize("batch", [1, 16])
def test_decode_70b_step_matches_oracle(jkb, oracle, batch):
    """configs[4] at its full size on one GPU, batch 1 (f32-input grouped launches) and batch 16
    (gemv_batch)."""
    _decode_parity(jkb, oracle, "70b", batch, 1)


def test_decode_70b_batch16_tensor_cores_match_oracle(jkb, oracle):
    """configs[4] at batch 16 on the tensor cores (the bench's batch16_tc section): i8
    RepackedWeights, the 16 tokens quantized by QuantizedActQ8 and one gemm_repacked per matrix
    on the 32-token tile. Three 32-row ranges per matrix (first, middle, last) for every token
    against oracle.gemm_repacked within the GEMM tolerance (repack.rs:3045-3093 semantics)."""
    spec = bench.DECODE_SETS["70b"]
    batch = 16
    ds = bench.DecodeSet(jkb, spec["mats"], spec["acts"], 1, 0, peer=False, batch=batch,
                         layer_copies=spec["copies"], sigma=spec["sigma"], tc=True)
    xs = {s: ds.xs[s].cpu().numpy() for s in spec["acts"]}
    ds.step(0)
    torch.cuda.synchronize()
    assert jkb.device_status() == 0
    for j, (name, quant, rows, cols, s) in enumerate(spec["mats"]):
        raw = bench.synth_matrix(quant, rows, cols, 1000 + j, sigma=spec["sigma"])
        row_bytes = raw.size // rows
        got = host(ds.output(name, 0)).reshape(batch, rows)
        for r0 in (0, rows // 2 - 16, rows - 32):
            sub = raw[r0 * row_bytes:(r0 + 32) * row_bytes]
            q, sc, mn = oracle.repack_block_scaled(quant, sub, 32, cols)
            xq, xsc, xsum, xs16, _ = oracle.act_q8_quantize(xs[s], batch, cols)
            ref = oracle.gemm_repacked(quant, q, sc, mn, 32, cols, xq, xsc, xsum, xs16, batch,
                                       nthreads=os.cpu_count() or 8)
            bound = gemm_abs_bound(oracle, quant, sub, 32, cols, xs[s], batch)
            assert_gemm_close(got[:, r0:r0 + 32], ref, bound)
    ds.destroy()


@pytest.mark.parametrize("name", ["ffn_gate", "ffn_down", "lm_head"])
def test_70b_row_shards_stitch_bit_exact(jkb, oracle, name):
    """configs[4] sharded over 8 ranks, emulated on one GPU: each rank's row slice uploaded as its
    own weight (as bench.DecodeSet does per rank) and run with the same launch; the slices
    stitched in rank order equal the unsharded call bit for bit."""
    from jkb200.shard import shard_rows

    spec = bench.DECODE_SETS["70b"]
    j = [m[0] for m in spec["mats"]].index(name)
    _, quant, rows, cols, s = spec["mats"][j]
    x = torch.randn(cols, generator=torch.Generator().manual_seed(12)).cuda()
    full_raw = bench.synth_matrix(quant, rows, cols, 1000 + j, sigma=spec["sigma"])
    w = jkb.Weight(jkb.TensorView(name, quant, [rows, cols], full_raw), rows, cols)
    full = torch.empty(rows, dtype=torch.float32, device="cuda")
    jkb.vec_dot_grouped_rvv([(full, w)], x)
    stitched = torch.empty(rows, dtype=torch.float32, device="cuda")
    for p in range(8):
        rr = shard_rows(rows, 8, p)
        raw = bench.synth_matrix(quant, rows, cols, 1000 + j, rr.start, rr.stop, spec["sigma"])
        wp = jkb.Weight(jkb.TensorView(name, quant, [len(rr), cols], raw), len(rr), cols)
        jkb.vec_dot_grouped_rvv([(stitched[rr.start:rr.stop], wp)], x)
        torch.cuda.synchronize()
        wp.destroy()
    assert np.array_equal(bits(host(stitched)), bits(host(full)))
    w.destroy()


def test_q4_0_gemv_4096_matches_oracle(jkb, oracle):
    """the bench's Q4_0 4096 x 4096 matrix, pre-quantized and f32-input entry
    points; every row checked."""
    rows = cols = 4096
    raw = bench.synth_matrix(bench.Q4_0, rows, cols, 4240)
    w = jkb.Weight(jkb.TensorView("q4_0", bench.Q4_0, [rows, cols], raw), rows, cols)
    x = torch.randn(cols, generator=torch.Generator().manual_seed(3))
    xq_ref = oracle.quantize_row_q8_0(x.numpy())
    xq = jkb.empty_q8_0_blocks(cols // 32)
    jkb.quantize_row_q8_0(x.cuda(), xq)
    assert np.array_equal(host(xq), xq_ref.view(np.uint8).reshape(-1))
    sumi, _, vals = (host(t) for t in jkb.gemv_block_dots(w, xq))
    s_ref, _, v_ref = oracle.block_dots(bench.Q4_0, raw, rows, cols, xq_ref)
    assert np.array_equal(sumi, s_ref)
    assert np.array_equal(bits(vals), bits(v_ref))
    y_ref = oracle.gemv(bench.Q4_0, raw, rows, cols, xq_ref)
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    for fn, inp in ((jkb.gemv_q4_0_q8_0, xq), (jkb.vec_dot_q4_0_rvv, x.cuda())):
        out.fill_(float("nan"))
        fn(out, w, inp)
        y = host(out)
        ok, worst = R.gemv_tolerance_ok(y, y_ref, v_ref, REL)
        assert ok, (fn.__name__, worst)
        assert R.l2_rel_err(y, y_ref) < REL
    w.destroy()


@pytest.mark.parametrize("m,n,k", bench.PREFILL)
def test_prefill_q8_0_shapes_match_oracle(jkb, oracle, m, n, k):
    """the bench's weights and activations for this shape (rank 0 of 1)."""
    raw = bench.synth_matrix(bench.Q8_0, n, k, 4243 + n)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", bench.Q8_0, [n, k], raw), n, k)
    x = torch.randn(m * k, generator=torch.Generator().manual_seed(2))
    act = jkb.QuantizedActQ8.quantize(x.cuda(), m, k)
    outs = {}
    for exact in (True, False):
        out = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
        with jkb.gemm_exact(exact):
            rw.gemm(out, act)
        assert jkb.device_status() == 0
        outs[exact] = host(out).reshape(m, n)
    rw.destroy()
    xs = x.numpy()
    row_bytes = raw.size // n
    for r0 in (0, n // 2 - 16, n - 32):
        r1 = r0 + 32
        sub = raw[r0 * row_bytes:r1 * row_bytes]
        q, s, mn = oracle.repack_block_scaled(bench.Q8_0, sub, 32, k)
        xq, xsc, xsum, xs16, _ = oracle.act_q8_quantize(xs, m, k)
        ref = oracle.gemm_repacked(bench.Q8_0, q, s, mn, 32, k, xq, xsc, xsum, xs16, m,
                                   nthreads=os.cpu_count() or 8)
        assert np.array_equal(bits(outs[True][:, r0:r1]), bits(ref)), f"rows {r0}..{r1} exact"
        xd = np.abs(xq.astype(np.float64) * np.repeat(xsc.astype(np.float64), 32, axis=1))
        wd = np.abs(q.astype(np.float64) * np.repeat(s.astype(np.float64), 32, axis=1))
        assert_gemm_close(outs[False][:, r0:r1], ref, xd @ wd.T)
