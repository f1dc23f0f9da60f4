"""Helpers for the GPU parity tests: device buffers through torch (plumbing
only) and the error metrics the parity bar is stated in."""
from __future__ import annotations

import numpy as np

# North-star tolerance for fp16/fp32 outputs: max relative error 2e-3 against
# an fp64 reference, measured normwise per output tensor: max|y - r| / max|r|.
REL_TOL = 2e-3


def torch():
    import torch as _t
    return _t


def dev(a: np.ndarray):
    """Copy a numpy array to the GPU as a flat uint8 tensor (keeps the bytes)."""
    t = torch()
    a = np.ascontiguousarray(a)
    return t.from_numpy(a.view(np.uint8).reshape(-1).copy()).cuda()


def empty(nbytes: int, fill: int = 0xFF):
    t = torch()
    return t.full((nbytes,), fill, dtype=t.uint8, device="cuda")


def host(tensor, dtype, shape=None) -> np.ndarray:
    torch().cuda.synchronize()
    a = tensor.cpu().numpy().view(dtype)
    return a.reshape(shape) if shape is not None else a


def normwise_err(y: np.ndarray, ref: np.ndarray) -> float:
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))
