"""Host logic of the multi-GPU path (jkb200.shard) with world_size-2 gloo ranks on CPU.

* Row shards + all-gather reassemble the full outputs: each rank computes its rows of every
  matrix (the CPU oracle stands in for its GPU here), the slices are all-gathered, and the
  assembled vectors equal the unsharded oracle GEMV bit for bit (rows are independent; the
  reference stitches row ranges the same way, tests/test_repack_gemv_gemm.rs:805-826). Row
  counts that do not divide by the world size exercise the uneven split.
* A rank that never joins the step: the other rank's all-gather ends with CollectiveError within
  the process-group timeout instead of hanging.
"""
import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
Q4_K, Q6_K, Q8_0, TQ2_0 = 12, 14, 8, 35


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for p in (os.path.join(ROOT, "jero-kernels-rvv_b200"), os.path.join(ROOT, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)


MATS = [("attn_q", Q4_K, 41, 512), ("lm_head", Q6_K, 37, 512), ("ffn_up", Q8_0, 30, 256)]


def _weights(O, quant, rows, cols, seed):
    return O.quantize_weights(quant, O.normal(rows * cols, seed, 0.02), rows, cols)


def _act(O, quant, cols):
    x = O.normal(cols, 7 + cols, 1.0)
    return O.quantize_row_q8_0(x) if quant == Q8_0 else O.quantize_row_q8_k(x)


def _worker(rank, world, port, mode, q):
    try:
        _setup_paths()
        import torch.distributed as dist
        import pyoracle as O
        from jkb200.shard import CollectiveError, ShardedOutputs

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=4))
        outs = ShardedOutputs([(n, r) for n, _, r, _ in MATS], world, rank, device="cpu")
        if mode == "lost_peer" and rank == 1:
            q.put((rank, "left"))  # leaves between steps: never enters the all-gather
            return
        full = {}
        for i, (name, quant, rows, cols) in enumerate(MATS):
            wb = _weights(O, quant, rows, cols, 100 + i)
            xq = _act(O, quant, cols)
            rr = outs.rows_of(name)
            row_bytes = wb.size // rows
            part = wb[rr.start * row_bytes:rr.stop * row_bytes]
            import torch
            outs.local_slice(name).copy_(torch.from_numpy(O.gemv(quant, part, len(rr), cols, xq)))
            full[name] = O.gemv(quant, wb, rows, cols, xq)
        try:
            outs.gather()
        except CollectiveError as e:
            q.put((rank, f"collective_error: {e}"))
            return
        ok = all(np.array_equal(outs.output(n).numpy().view(np.uint32),
                                full[n].view(np.uint32)) for n, _, _, _ in MATS)
        q.put((rank, "ok" if ok else "mismatch"))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 -- reported to the parent
        q.put((rank, "exception: " + traceback.format_exc()))


def _run(mode, world=2, timeout=60):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=timeout)
        res[r] = msg
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return res


def test_shard_rows_partition():
    _setup_paths()
    from jkb200.shard import shard_rows

    for rows in (1, 7, 8, 37, 128256, 28672):
        for world in (1, 2, 3, 4, 8):
            parts = [shard_rows(rows, world, r) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == rows
            assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
    # the benchmark shapes split evenly over 1/2/4/8 GPUs (8-row tile structure kept)
    for rows in (4096, 1024, 14336, 128256, 28672, 8192):
        assert all(len(shard_rows(rows, 8, r)) == rows // 8 for r in range(8))


def test_sharded_gather_reassembles_full_outputs():
    res = _run("parity")
    assert res == {0: "ok", 1: "ok"}, res


def test_lost_peer_ends_the_collective_with_an_error():
    res = _run("lost_peer")
    assert res[1] == "left", res
    assert res[0].startswith("collective_error"), res
