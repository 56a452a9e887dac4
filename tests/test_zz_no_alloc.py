"""The allocation-free GEMM entry point, jkb_gemm_repacked_f32_noalloc.

Some callers cannot allocate device memory. One example is an engine that reserved all
remaining HBM for its KV cache at start-up. Another is a host whose per-token loop forbids
cudaMalloc, because it can synchronize the device. Neither can create the jkb_act_q8 scratch
handle that jkb_gemm_repacked_f32 needs. The no-alloc variant quantizes into a scratch array
built into the library instead.

This file checks, through the C ABI, that two calls in a row match the allocating entry point
(tensor-core batches, small batches on the dp4a kernel, a K too long for the transposed scale
planes, and Q2_K weights, which take the dp4a kernel here), that batches beyond the scratch
limit are rejected, and that once a device is set up a call changes neither the device's free
memory nor torch's allocation count. pytest collects this file last, so a run
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


def _weights(oracle, quant, rows, cols, seed):
    if quant == 10:  # Q2_K: seeded random bytes (the oracle has no Q2_K weight quantizer)
        return np.random.default_rng(seed).integers(0, 256, rows * (cols // 256) * 84,
                                                    dtype=np.uint8)
    return oracle.quantize_weights(quant, oracle.normal(rows * cols, seed, 0.02), rows, cols)


@pytest.mark.parametrize("quant,rows,cols,m", [
    (8, 384, 2048, 64),     # tensor cores
    (12, 384, 2048, 64),    # tensor cores, min terms
    (14, 384, 2048, 64),    # tensor cores, 16-element groups
    (10, 384, 2048, 64),    # Q2_K: the dp4a kernel on this entry point
    (8, 96, 2048, 9),       # a small batch: the dp4a kernel
    (12, 384, 2048, 16),    # 16 tokens: the tensor cores' 32-token tile
    (8, 40, 163840, 4),     # K too long for the transposed planes (they are not written)
])
def test_noalloc_matches_allocating_entry_point_twice(jkb, oracle, quant, rows, cols, m):
    from jkb200 import _lib

    lib = _lib.load()
    wb = _weights(oracle, quant, rows, cols, 40 + quant)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [rows, cols], wb), rows, cols)
    scratch = jkb.QuantizedActQ8(m, cols)
    for call in range(2):  # the second call reuses the scratch the first call left behind
        mm = m if call == 0 else max(1, m - 7)
        x = dev(oracle.normal(mm * cols, 1000 * call + quant, 1.0))
        ref = torch.empty(mm * rows, dtype=torch.float32, device="cuda")
        out = torch.full((mm * rows,), float("nan"), dtype=torch.float32, device="cuda")
        # Q2_K runs the tensor cores through the allocating entry point and the dp4a kernel
        # through this one; with the exact epilogue both equal the reference bit for bit
        with jkb.gemm_exact(quant == 10 or jkb.gemm_get_exact()):
            jkb.gemm_repacked_f32(ref, rw, x, mm, scratch)
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


def test_noalloc_call_allocates_nothing_once_set_up(jkb, oracle):
    """After one call has set the device up (module loaded, scratch address looked up), further
    calls leave the device's free memory and torch's allocation count unchanged."""
    from jkb200 import _lib

    lib = _lib.load()
    rows, cols, m = 256, 4096, 48
    wb = oracle.quantize_weights(8, oracle.normal(rows * cols, 9, 0.02), rows, cols)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", 8, [rows, cols], wb), rows, cols)
    x = dev(oracle.normal(m * cols, 10, 1.0))
    out = torch.empty(m * rows, dtype=torch.float32, device="cuda")
    assert _noalloc(lib, out, rw, x, m) == 0, lib.jkb_last_error()  # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        assert _noalloc(lib, out, rw, x, m) == 0, lib.jkb_last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == alloc0
