"""bench.py host logic on CPU: its numpy weight quantizers agree byte for byte with the
oracle's (so bench data and test data are the same format), and the reference arm runs."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("quant", [bench.Q4_0, bench.Q4_K, bench.Q6_K, bench.Q8_0])
def test_bench_quantizers_match_oracle(oracle, quant):
    rows, cols = 24, 1024
    w = oracle.normal(rows * cols, 123 + quant, 0.02)
    w[5] = 0.0
    a = bench.QUANTIZERS[quant](w.reshape(rows, cols))
    b = oracle.quantize_weights(quant, w, rows, cols)
    assert np.array_equal(a, b)


def test_algorithmic_bytes_per_call():
    # GGUF weight blocks + Q8 activation blocks + f32 outputs of one call at batch 1:
    # Q4_0 4096x4096 = 9,437,184 + 4,608 + 16,384; Q4_K 4096->4096 = 9,437,184 + 4,672 + 16,384;
    # Q6_K lm_head 4096->128256 = 430,940,160 + 4,672 + 513,024
    assert bench.algorithmic_bytes(bench.Q4_0, 4096, 4096) == 9_458_176
    assert bench.algorithmic_bytes(bench.Q4_K, 4096, 4096) == 9_458_240
    assert bench.algorithmic_bytes(bench.Q4_K, 4096, 14336) == 33_062_880
    assert bench.algorithmic_bytes(bench.Q6_K, 128256, 4096) == 431_457_856
    # 70B down projection at batch 16: the weights once, 16 tokens of activations and outputs
    assert bench.algorithmic_bytes(bench.Q4_K, 8192, 28672, 16) == \
        132_120_576 + 16 * (112 * 292 + 4 * 8192)


def test_decode_sets_shapes():
    s8, s70 = bench.DECODE_SETS["8b"], bench.DECODE_SETS["70b"]
    assert sum(bench.algorithmic_bytes(q, r, c) for _, q, r, c, _ in s8["mats"]) == 554_357_664
    assert [(r, c) for _, _, r, c, _ in s70["mats"]] == [(28672, 8192), (28672, 8192),
                                                        (8192, 28672), (128256, 8192)]
    for s in (s8, s70):
        assert all(c == s["acts"][st] for _, _, _, c, st in s["mats"])


def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3"], capture_output=True, text=True,
                         timeout=600, check=True).stdout.strip().splitlines()
    assert len(out) == 1
    d = json.loads(out[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["cpu_model"]
    # the same config dict the GPU arm prints at N=1
    assert d["config"] == bench.decode_config(bench.DECODE_SETS["8b"], 1, "peer")


def test_decode_config_names_the_collective():
    """N > 1: the config line says how the output shards are collected (the driver's scaling
    runs use the default, the one-kernel all-gather)."""
    sp = bench.DECODE_SETS["8b"]
    par = {c: bench.decode_config(sp, 2, c)["parallelism"] for c in ("peer", "push", "nccl")}
    assert par["peer"] == "row-shard x2 + one-kernel all-gather over NVLink peer memory"
    assert "pushed to the peers by the GEMVs" in par["push"]
    assert par["nccl"].endswith("NCCL all-gather")
    assert bench.decode_config(sp, 1, "push")["parallelism"] == "row-shard x1"
