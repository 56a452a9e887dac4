"""The allocation-free GEMM entry point, jkb_gemm_repacked_f32_noalloc.

Some callers cannot allocate device memory. One example is an engine that reserved all
remaining HBM for its KV cache at start-up. Another is a host whose per-token loop forbids
cudaMalloc, because it can synchronize the device. Neither can create the jkb_act_q8 scratch
handle that jkb_gemm_repacked_f32 needs. The no-alloc variant quantizes into a scratch array
built into the library instead.

This file checks, through the C ABI, that two calls in a row match the allocating entry point,
and that batches beyond the scratch limit are rejected. pytest collects this file last, so a run
stopped at the first failure has run every other test first. It also passes on its own in a
fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from gpuutil import bits, dev, host

pytestmark = pytest.mark.gpu

LIMIT = 1 << 21  # m * round_up(cols, 32) elements the built-in scratch holds


def _noalloc(lib, out, rw, x, m):
    return lib.jkb_gemm_repacked_f32_noalloc(out.data_ptr(), out.numel(), rw._h, x.data_ptr(),
                                             x.numel(), m,
                                             torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("quant", [8, 12, 14])
def test_noalloc_matches_allocating_entry_point_twice(jkb, oracle, quant):
    from jkb200 import _lib

    lib = _lib.load()
    rows, cols, m = 384, 2048, 64
    wb = oracle.quantize_weights(quant, oracle.normal(rows * cols, 40 + quant, 0.02), rows, cols)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], wb), rows, cols)
    scratch = jkb.QuantizedActQ8(m, cols)
    for call in range(2):  # the second call reuses the scratch the first call left behind
        mm = m if call == 0 else m - 7
        x = dev(oracle.normal(mm * cols, 1000 * call + quant, 1.0))
        ref = torch.empty(mm * rows, dtype=torch.float32, device="cuda")
        jkb.gemm_repacked_f32(ref, rw, x, mm, scratch)
        out = torch.full((mm * rows,), float("nan"), dtype=torch.float32, device="cuda")
        assert _noalloc(lib, out, rw, x, mm) == 0, lib.jkb_last_error()
        got, want = host(out), host(ref)
        # both entry points run the same quantizer and GEMM, so the outputs agree bit for bit
        # (stricter than the 1e-5 relative tolerance used for f32 outputs elsewhere)
        assert np.array_equal(bits(got), bits(want))
        assert np.all(np.abs(got - want) <= 1e-5 * np.abs(want) + 1e-30)


def test_noalloc_rejects_batches_beyond_the_scratch_limit(jkb, oracle):
    from jkb200 import _lib

    lib = _lib.load()
    rows, cols = 64, 4096
    wb = oracle.quantize_weights(8, oracle.normal(rows * cols, 3, 0.02), rows, cols)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [rows, cols], wb), rows, cols)
    m = LIMIT // cols + 1
    x = torch.zeros(m * cols, dtype=torch.float32, device="cuda")
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    assert _noalloc(lib, out, rw, x, m) == 1
    assert b"limit" in lib.jkb_last_error()
    m_ok = LIMIT // cols
    x = dev(oracle.normal(m_ok * cols, 5, 1.0))
    out = torch.empty(m_ok * rows, dtype=torch.float32, device="cuda")
    assert _noalloc(lib, out, rw, x, m_ok) == 0
    ref = torch.empty(m_ok * rows, dtype=torch.float32, device="cuda")
    jkb.gemm_repacked_f32(ref, rw, x, m_ok, jkb.QuantizedActQ8(m_ok, cols))
    assert np.array_equal(bits(host(out)), bits(host(ref)))
