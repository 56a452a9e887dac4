"""Peer groups on one GPU (world size 1): the all-gather entry point and the bounded wait.

* With one rank the all-gather has nothing to copy: it validates its chunks and returns, and
  outputs computed into the group's buffer stay bit-identical to the plain calls.
* A wait for arrivals that nothing delivers (a count no kernel will reach) ends after its bound
  (about 2 s) with bit 1 of the device error word set, and the context stays usable: a GEMV
  launched afterwards still runs and is correct.
* Chunks that are unaligned or outside the group's buffer are rejected before any launch.
The multi-GPU behaviour (every rank's rows copied to every peer over NVLink) is tested under
torchrun by test_gpu_multigpu.py.
"""
import time

import numpy as np
import pytest
import torch

from gpuutil import bits, dev, host, upload

pytestmark = pytest.mark.gpu
Q4_K, Q6_K = 12, 14


def _weights(oracle):
    w1 = oracle.quantize_weights(Q4_K, oracle.normal(300 * 1024, 1, 0.02), 300, 1024)
    w3 = oracle.quantize_weights(Q6_K, oracle.normal(130 * 1024, 3, 0.02), 130, 1024)
    return w1, w3


def test_single_rank_allgather_keeps_outputs_in_place(jkb, oracle):
    from jkb200.shard import PeerOutputs

    w1, w3 = _weights(oracle)
    W1, W3 = upload(jkb, Q4_K, w1, 300, 1024), upload(jkb, Q6_K, w3, 130, 1024)
    x = dev(oracle.normal(1024, 9, 1.0))
    outs = PeerOutputs([("a", 300), ("b", 130)], 1, 0)
    for step in range(3):
        slot = step % 2
        jkb.vec_dot_q4_k_m_rvv(outs.local_slice("a", slot), W1, x)
        jkb.vec_dot_q6_k_rvv(outs.local_slice("b", slot), W3, x)
        outs.gather(slot)
        assert jkb.device_status() == 0
        ra, rb = torch.empty(300, device="cuda"), torch.empty(130, device="cuda")
        jkb.vec_dot_q4_k_m_rvv(ra, W1, x)
        jkb.vec_dot_q6_k_rvv(rb, W3, x)
        assert np.array_equal(bits(host(outs.output("a", slot))), bits(host(ra)))
        assert np.array_equal(bits(host(outs.output("b", slot))), bits(host(rb)))
    outs.destroy()


def test_wait_that_nothing_satisfies_expires_and_reports(jkb, oracle):
    pg = jkb.PeerGroup(1024, world=1, rank=0)
    t0 = time.time()
    pg.wait(1)  # no kernel ever signals this rank
    with pytest.raises(jkb.K3Error) as e:
        jkb.device_status()
    dt = time.time() - t0
    assert e.value.status == 5 and "flags 2" in e.value.reason, e.value  # JKB_E_TIMEOUT, bit 1
    assert 1.0 < dt < 30.0
    assert jkb.device_status() == 0  # the word was cleared
    # the context is still usable
    w1, _ = _weights(oracle)
    W1 = upload(jkb, Q4_K, w1, 300, 1024)
    x = dev(oracle.normal(1024, 9, 1.0))
    r = torch.empty(300, device="cuda")
    jkb.vec_dot_q4_k_m_rvv(r, W1, x)
    assert np.all(np.isfinite(host(r)))
    pg.destroy()


def test_allgather_chunk_validation(jkb):
    pg = jkb.PeerGroup(1024, world=1, rank=0)
    with pytest.raises(jkb.TensorBoundsError):
        pg.allgather([(1000, 64)])  # past the end of the 1024-byte buffer
    with pytest.raises(jkb.TensorBoundsError):
        pg.allgather([(2, 8)])      # not 4-byte aligned
    with pytest.raises(jkb.TensorBoundsError):
        pg.allgather([(0, 4)] * 17)  # more chunks than the launch takes
    pg.allgather([(0, 1024)])
    assert jkb.device_status() == 0
    pg.destroy()


def test_single_rank_push_and_signal(jkb, oracle):
    """Push mode with one rank: the GEMVs into the group's buffer have no peer to store to and
    stay bit-identical to the plain calls (single, grouped and token-batch launches); signal()
    returns without a wait."""
    from jkb200.shard import PeerOutputs

    w1, w3 = _weights(oracle)
    W1, W3 = upload(jkb, Q4_K, w1, 300, 1024), upload(jkb, Q6_K, w3, 130, 1024)
    outs = PeerOutputs([("a", 300), ("b", 130)], 1, 0, push=True)
    xq = jkb.empty_q8_k_blocks(4 * 4)
    for step in range(3):
        slot = step % 2
        x = dev(oracle.normal(1024, 20 + step, 1.0))
        jkb.vec_dot_grouped_rvv([(outs.local_slice("a", slot), W1)], x)
        jkb.quantize_row_q8_k(x, xq[:4 * 292])
        jkb.gemv_rows(outs.local_slice("b", slot), W3, xq[:4 * 292], range(0, 130))
        outs.gather(slot)
        assert jkb.device_status() == 0
        ra, rb = torch.empty(300, device="cuda"), torch.empty(130, device="cuda")
        jkb.vec_dot_grouped_rvv([(ra, W1)], x)
        jkb.gemv_rows(rb, W3, xq[:4 * 292], range(0, 130))
        assert np.array_equal(bits(host(outs.output("a", slot))), bits(host(ra)))
        assert np.array_equal(bits(host(outs.output("b", slot))), bits(host(rb)))
    outs.destroy()
    # token batch: four tokens through gemv_batch into a pushing buffer
    outs = PeerOutputs([("b", 130)], 1, 0, batch=4, push=True)
    xb = dev(oracle.normal(4 * 1024, 31, 1.0))
    jkb.quantize_rows_q8_k(xb, 4, 1024, xq)
    jkb.gemv_batch(outs.local_slice("b", 0), W3, xq, 4)
    outs.gather(0)
    rb = torch.empty(4 * 130, device="cuda")
    jkb.gemv_batch(rb, W3, xq, 4)
    assert np.array_equal(bits(host(outs.output("b", 0))).reshape(-1), bits(host(rb)))
    assert jkb.device_status() == 0
    outs.destroy()


def test_push_boundaries_fail_closed(jkb, oracle):
    """An output range that crosses the edge of a pushing buffer is rejected before any launch;
    the entry points that do not push (the repacked GEMM) refuse outputs inside one; with push
    disabled again both work."""
    w1, _ = _weights(oracle)
    W1 = upload(jkb, Q4_K, w1, 300, 1024)
    x = dev(oracle.normal(1024, 9, 1.0))
    from jkb200 import _lib
    from jkb200.api import _check

    pg = jkb.PeerGroup(4 * 400, world=1, rank=0)
    pg.set_push(True)
    jkb.vec_dot_q4_k_m_rvv(pg.buffer[:300], W1, x)  # inside: fine
    # 300 outputs starting 200 bytes before the buffer (in the group's own 256-byte header, so
    # the range stays inside the allocation): rejected before any launch
    lo = pg.buffer.data_ptr() - 200
    with pytest.raises(jkb.TensorBoundsError, match="crosses the edge"):
        _check(_lib.load().jkb_vec_dot_q4_k_m_rvv(lo, 300, W1.handle, x.data_ptr(), 1024, None))
    raw = oracle.quantize_weights(8, oracle.normal(64 * 256, 4, 0.02), 64, 256)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [64, 256], raw), 64, 256)
    act = jkb.QuantizedActQ8.quantize(dev(oracle.normal(2 * 256, 5, 1.0)), 2, 256)
    with pytest.raises(jkb.CapabilityMismatch, match="does not push"):
        rw.gemm(pg.buffer[:128], act)
    pg.set_push(False)
    rw.gemm(pg.buffer[:128], act)
    assert jkb.device_status() == 0
    rw.destroy()
    pg.destroy()
