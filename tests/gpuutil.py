"""Helpers shared by the GPU parity tests (device copies, weight upload)."""
import numpy as np
import torch


def dev(a: np.ndarray) -> torch.Tensor:
    """Copy a numpy array (any dtype, viewed as raw bytes when structured) to the GPU."""
    a = np.ascontiguousarray(a)
    if a.dtype.fields is not None:
        a = a.view(np.uint8).reshape(-1)
    return torch.from_numpy(a.copy()).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def upload(jkb, quant, w: np.ndarray, rows: int, cols: int, shape=None, on_device=False,
           name="w"):
    shape = shape or [rows, cols]
    data = dev(w) if on_device else w
    return jkb.Weight(jkb.TensorView(name, quant, shape, data), rows, cols)


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def gemm_abs_bound(oracle, quant, wb, rows, cols, act, m):
    """Per output (m, n) of the repacked GEMM: sum over k of |x~[m,k]| * |w~[n,k]| (plus the
    Q4_K_M min terms), the dequantized operands' absolute dot products in f64. It bounds the
    sum of |block values| the reference adds up, so 1e-5 of it is the per-output tolerance."""
    q, s, mn = oracle.repack_block_scaled(quant, wb, rows, cols)
    xq, xs, xsum, xs16, _ = oracle.act_q8_quantize(act, m, cols)
    kp = q.shape[1]
    gsz = kp // s.shape[1]
    xd = np.abs(xq.astype(np.float64) * np.repeat(xs.astype(np.float64), 32, axis=1))
    wd = np.abs(q.astype(np.float64) * np.repeat(s.astype(np.float64), gsz, axis=1))
    bound = xd @ wd.T
    if mn is not None:
        xsm = xsum if gsz == 32 else xs16
        bound += np.abs(xsm.astype(np.float64)) @ np.abs(mn.astype(np.float64)).T
    return bound


def assert_gemm_close(got, ref, bound):
    """The f32 tolerance contract of the GEMM outputs: |got - ref| <= 1e-5 * bound per output,
    and an l2 relative error below 1e-5 over the whole output."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    assert np.all(err <= 1e-5 * bound + 1e-30), float((err / (bound + 1e-30)).max())
    den = np.linalg.norm(ref)
    if den > 0:
        assert np.linalg.norm(got - ref) / den < 1e-5
