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


@pytest.mark.parametrize("quant", [bench.Q4_K, bench.Q6_K, bench.Q8_0])
def test_bench_quantizers_match_oracle(oracle, quant):
    rows, cols = 24, 1024
    w = oracle.normal(rows * cols, 123 + quant, 0.02)
    w[5] = 0.0
    a = bench.QUANTIZERS[quant](w.reshape(rows, cols))
    b = oracle.quantize_weights(quant, w, rows, cols)
    assert np.array_equal(a, b)


def test_algorithmic_bytes_match_baseline_table():
    # Q4_K 4096->4096 = 9,458,240 B; Q6_K lm_head = 431,457,856 B
    assert bench.algorithmic_bytes(bench.Q4_K, 4096, 4096) == 9_458_240
    assert bench.algorithmic_bytes(bench.Q4_K, 4096, 14336) == 33_062_880
    assert bench.algorithmic_bytes(bench.Q6_K, 128256, 4096) == 431_457_856


def test_reference_arm_prints_one_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3"], capture_output=True, text=True,
                         timeout=600, check=True).stdout.strip().splitlines()
    assert len(out) == 1
    d = json.loads(out[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0
