"""C-ABI checks that need no GPU: the in-tree library loads, exports every entry point that
include/jkb200.h declares, the Python binding table matches the header, and argument
validation fails closed (status + TensorBoundsError fields, nothing launched) exactly where the
reference validators do. No call here reaches a kernel."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "jkb200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(jkb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from jkb200 import _lib

    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from jkb200 import _lib

    names = declared()
    assert len(names) >= 50
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert hasattr(lib, n)
    extra = sorted(s for s in exported if s.startswith("jkb_") and s not in names)
    assert not extra, f"exported but undeclared: {extra}"


def test_python_binding_table_matches_header():
    from jkb200 import _lib

    assert sorted(_lib.declared_symbols()) == declared()


def test_abi_version(lib):
    assert lib.jkb_abi_version() == 1


def _err(lib):
    from jkb200 import _lib

    info = _lib.jkb_error_info()
    lib.jkb_last_error_info(C.byref(info))
    return info


def test_quantize_row_validation_fails_closed(lib):
    """validate_activation_quant_slice (quant_q8.rs:111-149); reference test :3415-3424."""
    buf = (C.c_float * 64)()
    rc = lib.jkb_quantize_row_q8_0(C.addressof(buf), 31, C.addressof(buf), 1, None)
    assert rc == 1
    e = _err(lib)
    assert e.status == 1 and b"positive multiple of 32" in e.reason
    assert e.byte_len == 31 * 4
    rc = lib.jkb_quantize_row_q8_0(C.addressof(buf), 0, C.addressof(buf), 0, None)
    assert rc == 1
    rc = lib.jkb_quantize_row_q8_k(C.addressof(buf), 256, C.addressof(buf), 0, None)
    assert rc == 1 and b"output block count 0 != expected 1" in _err(lib).reason
    assert b"TensorBoundsError" in lib.jkb_last_error()
    lib.jkb_clear_error()
    assert lib.jkb_last_error() == b""


def test_misaligned_pointers_rejected_before_launch(lib):
    """Block activations and f32 buffers must be 4-byte aligned (align_of BlockQ8_0); a
    misaligned pointer is a TensorBoundsError, never a device access."""
    buf = (C.c_uint8 * 4096)()
    base = C.addressof(buf)
    rc = lib.jkb_quantize_row_q8_0(base + 1, 32, base + 64, 1, None)
    assert rc == 1 and b"not 4-byte aligned" in _err(lib).reason
    rc = lib.jkb_quantize_row_q8_k(base, 256, base + 2, 1, None)
    assert rc == 1 and b"not 4-byte aligned" in _err(lib).reason
    rc = lib.jkb_vec_dot_q8_0_q8_0(base, 34, base + 3, 1, base + 128, None)
    assert rc == 1 and b"x_blocks" in _err(lib).reason


def test_subln_dimension_mismatch(lib):
    """tests/empirical_challenge_m3_bitnet.rs:271-297."""
    buf = (C.c_float * 256)()
    rc = lib.jkb_subln_quantize_absmax_i8(C.addressof(buf), 127, C.addressof(buf), 128,
                                          C.addressof(buf), 128, 1e-5, C.addressof(buf), None)
    assert rc == 1 and b"dimension mismatch" in _err(lib).reason
    rc = lib.jkb_subln_quantize_absmax_i8(C.addressof(buf), 0, C.addressof(buf), 0,
                                          C.addressof(buf), 0, 1e-5, C.addressof(buf), None)
    assert rc == 1


def _view(quant, shape, data, name=b"w"):
    from jkb200 import _lib

    v = _lib.jkb_tensor_view()
    v.name = name
    v.quant = quant
    v.ndim = len(shape)
    for i, s in enumerate(shape):
        v.shape[i] = s
    v.offset = 0
    v.data = data.ctypes.data
    v.byte_len = data.nbytes
    v.data_on_device = 0
    return v


def test_weight_upload_validation(lib):
    """validate_matrix_view (repack.rs:1208-1284) and the capability check (repack.rs:2341)."""
    h = C.c_void_p()
    raw = np.zeros(18 * 4, np.uint8)
    v = _view(0, [32, 4], raw)  # F32 is dense storage: not built on the GPU
    assert lib.jkb_weight_upload(C.byref(v), 4, 32, None, C.byref(h)) == 2
    v = _view(2, [32, 4], raw)
    assert lib.jkb_weight_upload(C.byref(v), 4, 33, None, C.byref(h)) == 1
    assert b"multiple of Q4_0 block size" in _err(lib).reason
    assert lib.jkb_weight_upload(C.byref(v), 5, 32, None, C.byref(h)) == 1
    assert b"does not match requested rows=5" in _err(lib).reason
    short = np.zeros(18 * 3, np.uint8)
    v = _view(2, [32, 4], short)
    assert lib.jkb_weight_upload(C.byref(v), 4, 32, None, C.byref(h)) == 1
    assert b"backing bytes 54 < required 72" in _err(lib).reason
    v = _view(2, [2, 2, 32], raw)
    assert lib.jkb_weight_upload(C.byref(v), 4, 32, None, C.byref(h)) == 1
    assert b"expected 1D or 2D" in _err(lib).reason
    v = _view(2, [32], raw)
    assert lib.jkb_weight_upload_infer(C.byref(v), None, C.byref(h)) == 1
    assert b"requires a 2D tensor" in _err(lib).reason
    i2s = np.zeros(32 * 2, np.uint8)  # payload without its 32-byte trailer
    v = _view(36, [128, 2], i2s)
    assert lib.jkb_weight_upload(C.byref(v), 2, 128, None, C.byref(h)) == 1


def test_null_and_destroyed_handles(lib):
    buf = (C.c_float * 8)()
    assert lib.jkb_gemv_q4_k_q8_k(C.addressof(buf), 8, None, C.addressof(buf), 1, None) == 6
    assert lib.jkb_weight_destroy(None) == 6
    assert lib.jkb_act_q8_destroy(None) == 6
    assert lib.jkb_gemm_repacked(C.addressof(buf), 8, None, None, None) == 6
    assert lib.jkb_bitlinear_i8(C.addressof(buf), 8, None, C.addressof(buf), 8, 1.0, None) == 6


def test_act_q8_create_validation(lib):
    h = C.c_void_p()
    assert lib.jkb_act_q8_create(0, 128, C.byref(h)) == 1
    assert lib.jkb_act_q8_create(4, 0, C.byref(h)) == 1


def test_vec_dot_row_byte_validation(lib):
    """validate_q8_block_row_bytes (quant_q8.rs:648-667)."""
    buf = (C.c_uint8 * 1024)()
    rc = lib.jkb_vec_dot_q4_k_q8_k(C.addressof(buf), 143, C.addressof(buf), 1,
                                   C.addressof(buf), None)
    assert rc == 1 and b"expected 144 weight bytes for 1 blocks, got 143" in _err(lib).reason
    rc = lib.jkb_vec_dot_q4_0_q8_0(C.addressof(buf), 0, C.addressof(buf), 0,
                                   C.addressof(buf), None)
    assert rc == 1


def test_python_api_surface_imports():
    import jkb200

    for name in jkb200.__all__:
        assert hasattr(jkb200, name), name
    assert jkb200.QuantType.Q4_K_M == 12 and jkb200.QuantType.I2_S == 36
    assert jkb200.BLOCK[jkb200.QuantType.Q6_K] == (256, 210)


# ---------------------------------------------------------------- PackedNibbleMatrix (host side)

@pytest.mark.parametrize("quant", [2, 3, 20, 12])
def test_repack_nibble_into_tile_range_matches_oracle(oracle, quant):
    """The library's host tile packer (repack_nibble_into_tile_range, repack.rs:4414-4645)
    writes the reference's tile layout byte for byte, for the whole matrix and for a sub-range
    of tiles (ragged last tile: 203 rows)."""
    import jkb200 as jkb
    import refgen as R

    rows, cols = 203, 512
    raw = R.fill_pseudo_quant_tensor(quant, rows, cols)
    view = jkb.TensorView("nib", quant, [cols, rows], raw)
    ref = oracle.nibble_pack_tiles(quant, raw, rows, cols)
    got = jkb.repack_nibble_into_tile_range(view, rows, cols, range(0, 26))
    for a, b in zip(got, ref):
        assert (a is None) == (b is None)
        if a is not None:
            assert np.array_equal(a, b)
    kb = cols // 32
    part = jkb.repack_nibble_into_tile_range(view, rows, cols, range(5, 26))
    assert np.array_equal(part[0], ref[0][5 * kb * 128:])
    if quant == 12:
        assert np.array_equal(part[3], ref[3][5 * (cols // 256) * 8 * 16:])
    else:
        assert np.array_equal(part[1], ref[1][5 * kb * 8:])


def test_repack_nibble_into_tile_range_validation():
    import jkb200 as jkb
    import refgen as R

    rows, cols = 16, 64
    raw = R.fill_pseudo_quant_tensor(2, rows, cols)
    view = jkb.TensorView("nib", 2, [cols, rows], raw)
    with pytest.raises(jkb.TensorBoundsError) as e:
        jkb.repack_nibble_into_tile_range(view, rows, cols, range(0, 3))
    assert "exceeds n_tiles (2)" in e.value.reason
    L = jkb._lib.load()
    v = view._c()
    tiles = np.zeros(4 * 128, np.uint8)
    sc = np.zeros(3, np.uint16)
    rc = L.jkb_repack_nibble_into_tile_range(C.byref(v), rows, cols, 0, 2, tiles.ctypes.data, 4,
                                             sc.ctypes.data, 3, None, 0, None, 0)
    assert rc == 1 and b"out_scales_f16 slice length mismatch" in L.jkb_last_error()
    rc = L.jkb_repack_nibble_into_tile_range(C.byref(v), rows, cols, 0, 2, tiles.ctypes.data, 3,
                                             None, 0, None, 0, None, 0)
    assert rc == 1 and b"nibble out_tiles length 3 != 4" in L.jkb_last_error()
    q8 = jkb.TensorView("q8", 8, [cols, rows], np.zeros(rows * 2 * 34, np.uint8))
    with pytest.raises(jkb.CapabilityMismatch):
        jkb.repack_nibble_into_tile_range(q8, rows, cols, range(0, 2))
    raw1 = R.fill_pseudo_quant_tensor(3, rows, cols)
    v1 = jkb.TensorView("q41", 3, [cols, rows], raw1)._c()
    sc = np.zeros(32, np.uint16)
    rc = L.jkb_repack_nibble_into_tile_range(C.byref(v1), rows, cols, 0, 2, tiles.ctypes.data, 4,
                                             sc.ctypes.data, 32, None, 0, None, 0)
    assert rc == 1 and b"Q4_1 requires out_mins_f16 slice" in L.jkb_last_error()


def test_nibble_constructor_validation_fails_closed():
    """Validation order of PackedNibbleMatrix::{from_tensor, from_scale_f16_buffers,
    from_q4_k_buffers} (repack.rs:4686-4788): every error is reported before any device work."""
    import jkb200 as jkb

    with pytest.raises(jkb.CapabilityMismatch):
        jkb.PackedNibbleMatrix.from_tensor(
            jkb.TensorView("q8", 8, [64, 4], np.zeros(4 * 2 * 34, np.uint8)), 4, 64, stream=0)
    with pytest.raises(jkb.TensorBoundsError) as e:
        jkb.PackedNibbleMatrix.from_tensor(
            jkb.TensorView("q4", 2, [64, 4], np.zeros(4 * 2 * 18, np.uint8)), 4, 48, stream=0)
    assert "multiple of Q4_0 block size" in e.value.reason
    with pytest.raises(jkb.TensorBoundsError):
        jkb.PackedNibbleMatrix.repack(jkb.TensorView("q4", 2, [256], np.zeros(144, np.uint8)), stream=0)
    with pytest.raises(jkb.CapabilityMismatch):
        jkb.PackedNibbleMatrix.from_scale_f16_buffers(jkb.QuantType.Q4_K_M, 8, 256,
                                                      np.zeros(8 * 128, np.uint8),
                                                      np.zeros(64, np.uint16), stream=0)
    with pytest.raises(jkb.TensorBoundsError) as e:
        jkb.PackedNibbleMatrix.from_scale_f16_buffers(jkb.QuantType.Q4_0, 8, 64,
                                                      np.zeros(2 * 128, np.uint8),
                                                      np.zeros(15, np.uint16), stream=0)
    assert e.value.reason == "nibble buffer lengths do not match geometry"
    with pytest.raises(jkb.TensorBoundsError) as e:
        jkb.PackedNibbleMatrix.from_q4_k_buffers(8, 96, np.zeros(3 * 128, np.uint8),
                                                 np.zeros(8 * 16, np.uint8), stream=0)
    assert e.value.reason == "invalid rows/cols for Q4_K_M"
