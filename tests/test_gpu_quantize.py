"""GPU activation quantizers vs the CPU oracle: BlockQ8_0 / BlockQ8K rows
(quant_q8.rs:203-219, :447-475), QuantizedActQ8 (repack.rs:175-204, :542-650) and the SubLN
absmax quantizer (lib.rs:1042-1101). All of these are byte-exact contracts."""
import json
import os

import numpy as np
import pytest
import torch

import refgen as R
from gpuutil import bits, dev, host
from test_oracle_cpu import _subln_input, subln_case_check

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def edge_rows(oracle, k):
    rng = np.random.default_rng(k)
    rows = [oracle.normal(k, 0xAC70000 + k, 1.0), R.test_f32_row(k, 3), np.zeros(k, np.float32)]
    x = R.gen_activation(k, 99)
    x[5] = np.nan
    x[min(k - 1, 40)] = np.inf
    x[min(k - 1, 300)] = -np.inf
    rows.append(x)
    rows.append(np.full(k, 1e-40, np.float32))  # subnormal absmax
    rows.append((rng.standard_normal(k) * 1e30).astype(np.float32))
    # exact .5 ties after scaling: values j * amax / 254 round away from zero
    t = (np.arange(k) % 255 - 127).astype(np.float32) * np.float32(0.5)
    rows.append(t)
    return rows


@pytest.mark.parametrize("k", [32, 256, 4096, 14336])
def test_quantize_row_q8_0_bit_exact(jkb, oracle, k):
    for x in edge_rows(oracle, k):
        ref = oracle.quantize_row_q8_0(x)
        out = jkb.empty_q8_0_blocks(k // 32)
        xd = dev(x)
        jkb.quantize_row_q8_0(xd, out)
        assert np.array_equal(host(out), ref.view(np.uint8).reshape(-1))
        # misaligned input pointer takes the scalar load path
        if k >= 64:
            xd2 = dev(np.concatenate([np.zeros(1, np.float32), x]))[1:]
            out2 = jkb.empty_q8_0_blocks(k // 32)
            jkb.quantize_row_q8_0(xd2, out2)
            assert np.array_equal(host(out2), ref.view(np.uint8).reshape(-1))


@pytest.mark.parametrize("k", [256, 4096, 28672])
def test_quantize_row_q8_k_bit_exact(jkb, oracle, k):
    for x in edge_rows(oracle, k):
        ref = oracle.quantize_row_q8_k(x)
        out = jkb.empty_q8_k_blocks(k // 256)
        jkb.quantize_row_q8_k(dev(x), out)
        assert np.array_equal(host(out), ref.view(np.uint8).reshape(-1))


def test_quantize_rows_batched(jkb, oracle):
    m, k = 7, 1024
    x = oracle.normal(m * k, 5, 1.0)
    out0 = jkb.empty_q8_0_blocks(m * k // 32)
    jkb.quantize_rows_q8_0(dev(x), m, k, out0)
    ref0 = np.concatenate([oracle.quantize_row_q8_0(x[i * k:(i + 1) * k]) for i in range(m)])
    assert np.array_equal(host(out0), ref0.view(np.uint8).reshape(-1))
    outk = jkb.empty_q8_k_blocks(m * k // 256)
    jkb.quantize_rows_q8_k(dev(x), m, k, outk)
    refk = np.concatenate([oracle.quantize_row_q8_k(x[i * k:(i + 1) * k]) for i in range(m)])
    assert np.array_equal(host(outk), refk.view(np.uint8).reshape(-1))


def test_quantizer_sanitization_gpu(jkb, oracle):
    """src/quant_q8.rs:3414-3482 inputs on the GPU, compared byte for byte."""
    x96 = R.test_f32_row(96, 1)
    x96[3] = np.nan
    x96[11] = -np.nan
    x96[39] = np.inf
    x96[51] = -np.inf
    x96[64:96] = np.nan
    x96[64] = np.inf
    x96[95] = 0.0
    out = jkb.empty_q8_0_blocks(3)
    jkb.quantize_row_q8_0(dev(x96), out)
    assert np.array_equal(host(out), oracle.quantize_row_q8_0(x96).view(np.uint8).reshape(-1))
    with pytest.raises(jkb.TensorBoundsError):
        jkb.quantize_row_q8_0(dev(np.zeros(31, np.float32)), jkb.empty_q8_0_blocks(1))


@pytest.mark.parametrize("m,k", [(1, 4096), (5, 1000), (3, 14336), (64, 256)])
def test_act_q8_quantize_bit_exact(jkb, oracle, m, k):
    x = oracle.normal(m * k, 77 + k, 1.0)
    x[7] = np.nan
    x[k // 2] = np.inf
    if m > 1:
        x[k:k + 32] = 1e-35  # absmax < 1e-30 -> zero block, scale 0
    q_ref, xs_ref, xsum_ref, xs16_ref, sup_ref = oracle.act_q8_quantize(x, m, k)
    act = jkb.QuantizedActQ8(m, k)
    act.quantize_into(dev(x), m, k)
    q, xs, xsum, xs16, sup = (host(t) for t in act.buffers())
    assert np.array_equal(q, q_ref)
    assert np.array_equal(bits(xs), bits(xs_ref))
    assert np.array_equal(bits(xsum), bits(xsum_ref))
    assert np.array_equal(bits(xs16), bits(xs16_ref))
    assert np.array_equal(bits(sup), bits(sup_ref))
    act.destroy()


def test_act_q8_errors(jkb):
    act = jkb.QuantizedActQ8(4, 256)
    with pytest.raises(jkb.TensorBoundsError):
        act.quantize_into(dev(np.zeros(300, np.float32)), 1, 256)
    with pytest.raises(jkb.TensorBoundsError):
        act.quantize_into(dev(np.zeros(5 * 256, np.float32)), 5, 256)


def _subln_gpu(jkb, x, w, eps):
    out = torch.empty(x.size, dtype=torch.int8, device="cuda")
    sc = torch.empty(1, dtype=torch.float32, device="cuda")
    jkb.subln_quantize_absmax_i8(out, dev(x), dev(w), eps, sc)
    return host(out), np.float32(host(sc)[0])


def test_subln_kats_gpu(jkb, oracle):
    with open(os.path.join(GOLDEN, "kats.json")) as f:
        s = json.load(f)["subln"]
    for c in s["cases"]:
        x = _subln_input(c["input"], s["len"])
        w = _subln_input(c["weight"], s["len"])
        q, scale = _subln_gpu(jkb, x, w, s["eps"])
        subln_case_check(c, q, scale)
        qr, sr = oracle.subln_quantize_absmax_i8(x, w, s["eps"])
        assert np.array_equal(q, qr) and bits(scale) == bits(np.float32(sr)), c["name"]


@pytest.mark.parametrize("k", [256, 2560, 6912])
def test_subln_random_bit_exact(jkb, oracle, k):
    for it in range(4):
        x = oracle.normal(k, 1000 * it + k, 1.0)
        w = (oracle.normal(k, 7 * it + 1, 0.3) + 1.0).astype(np.float32)
        q, scale = _subln_gpu(jkb, x, w, 1e-5)
        qr, sr = oracle.subln_quantize_absmax_i8(x, w, 1e-5)
        assert np.array_equal(q, qr)
        assert bits(scale) == bits(np.float32(sr))
    m = 6
    xs = oracle.normal(m * k, 31, 1.0)
    ws = np.ones(k, np.float32)
    out = torch.empty(m * k, dtype=torch.int8, device="cuda")
    sc = torch.empty(m, dtype=torch.float32, device="cuda")
    jkb.subln_quantize_absmax_i8_rows(out, dev(xs), dev(ws), m, k, 1e-5, sc)
    o, s_ = host(out), host(sc)
    for i in range(m):
        qr, sr = oracle.subln_quantize_absmax_i8(xs[i * k:(i + 1) * k], ws, 1e-5)
        assert np.array_equal(o[i * k:(i + 1) * k], qr) and bits(s_[i]) == bits(np.float32(sr))
