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
