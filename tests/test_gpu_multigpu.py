"""Multi-GPU parity of the row-sharded path (Llama-3-70B shapes): launches
tests/mgpu_worker.py under torchrun on every visible GPU (at most 8) and checks that each rank
reports bit-exact reassembled outputs (Q4_K_M 8192 -> 28672 and 28672 -> 8192, Q6_K
8192 -> 128256 GEMVs and a Q8_0 prefill GEMM, each against the single-GPU call on rank 0),
both with the NCCL all-gather and with the library's one-kernel all-gather over NVLink peer
memory, and with rows pushed to the peers by the GEMV kernels (both checked on every rank).
Needs at least 2 GPUs; with one GPU the sharded host logic is covered by test_shard_gloo.py."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_row_sharded_outputs_match_single_gpu():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs (host logic: test_shard_gloo.py)")
    n = min(n, 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", "29517", os.path.join(ROOT, "tests", "mgpu_worker.py")]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    lines = [json.loads(x) for x in p.stdout.splitlines() if x.startswith("{")]
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-4000:]
    assert len(lines) == n and all(r["ok"] for r in lines), lines
    r0 = next(r for r in lines if r["rank"] == 0)
    for key in ("ffn_gate", "ffn_down", "lm_head", "prefill_gemm"):
        assert r0[key] == "bit-exact", r0
    assert r0["device_status"] == 0
    for r in lines:  # the NVLink all-gather kernel: every rank holds every row
        assert r["peer_allgather"] == "bit-exact" and r["peer_status"] == 0, r
        # rows pushed by the GEMV kernels themselves, one signal kernel a step
        assert r["peer_push"] == "bit-exact" and r["push_status"] == 0, r
