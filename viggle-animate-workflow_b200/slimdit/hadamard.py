"""Regular Hadamard rotation for convrot (same API as the reference's slimdit/hadamard.py).

``build_hadamard`` constructs the matrix on the host (it is a 256x256 constant): Kronecker
powers of the 4x4 seed H4 (entry -1 exactly where row + column index == 3), divided by
sqrt(size), so size must be a power of 4. ``rotate`` runs on the GPU
(libslimdit_b200.so) in the reference's own fp32 summation order, so its output equals the
reference's bit for bit (slimdit/hadamard.py:45-58).
"""

from __future__ import annotations

import math

import numpy as np

H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)

_CACHE: dict[tuple[int, str], np.ndarray] = {}


def _is_power_of_4(n: int) -> bool:
    return n >= 4 and (n & (n - 1)) == 0 and (n.bit_length() - 1) % 2 == 0


def build_hadamard(size: int = 256, dtype=np.float32) -> np.ndarray:
    """Normalised regular Hadamard matrix of ``size`` (a power of 4), cached per (size, dtype)."""
    key = (size, np.dtype(dtype).str)
    hit = _CACHE.get(key)
    if hit is not None:
        return hit
    if not isinstance(size, (int, np.integer)) or not _is_power_of_4(int(size)):
        raise ValueError(f"regular Hadamard size must be a power of 4, got {size}")
    mat = H4
    while mat.shape[0] < size:
        mat = np.kron(mat, H4)
    out = (mat / math.sqrt(size)).astype(dtype)
    _CACHE[key] = out
    return out


def _check_regular(h: np.ndarray, group_size: int) -> None:
    ref = build_hadamard(group_size, np.float64)
    if h.shape != ref.shape or not np.array_equal(np.asarray(h, np.float64), ref):
        raise ValueError("the device rotation implements the regular Hadamard of build_hadamard() only")


def rotate(weight, h, group_size: int = 256):
    """Group-wise rotation ``W @ H^T`` over blocks of ``group_size`` input features.

    ``weight``: float32 numpy [N, K] (returns float32 numpy) or a CUDA tensor (returns an
    fp32 CUDA tensor). Applying it twice is the identity up to rounding (H is symmetric and
    orthogonal). Only ``group_size`` 256 is implemented on the device.
    """
    import torch

    is_tensor = isinstance(weight, torch.Tensor)
    if weight.ndim != 2:
        raise ValueError(f"expected a 2D weight, got shape {tuple(weight.shape)}")
    out_features, in_features = weight.shape
    if in_features % group_size != 0:
        raise ValueError(f"in_features {in_features} not divisible by group_size {group_size}")
    _check_regular(np.asarray(h.cpu() if isinstance(h, torch.Tensor) else h), group_size)
    from . import ops

    if is_tensor:
        return ops.rotate(weight, group_size)
    if weight.dtype != np.float32:
        raise TypeError(f"device rotate() computes in float32; got {weight.dtype} (cast first)")
    if out_features == 0:
        return np.empty((0, in_features), np.float32)
    src = torch.from_numpy(np.ascontiguousarray(weight)).cuda()
    return ops.rotate(src, group_size).cpu().numpy()
