"""INT8 convrot weight format (same API as the reference's slimdit/int8.py).

ComfyUI stores a convrot linear as three tensors: ``<name>.weight`` int8 [N, K] (already
rotated, W @ H^T), ``<name>.weight_scale`` float32 [N, 1] (per-row absmax / 127) and
``<name>.comfy_quant`` uint8 [72] (the JSON descriptor below, NUL padded). The runtime
computes ``x_rot @ (q * scale)^T`` with the activation rotated by the same H.

Quantisation and dequantisation run on the GPU (libslimdit_b200.so) in the reference's
summation order: codes and scales equal the reference's bit for bit.
"""

from __future__ import annotations

import json

import numpy as np

from .hadamard import build_hadamard

#: Length of the ``comfy_quant`` descriptor tensor.
BLOB_LEN = 72
#: The descriptor text ComfyUI parses with ``json.loads`` (field order and spacing matter).
BLOB = '{"format": "int8_tensorwise", "convrot": true, "convrot_groupsize": 256}'


def comfy_quant_blob(group_size: int = 256) -> np.ndarray:
    """uint8 [72] descriptor, NUL padded. Only group size 256 is written."""
    if group_size != 256:
        raise ValueError("this project only writes convrot_groupsize 256")
    raw = BLOB.encode("ascii")
    if len(raw) > BLOB_LEN:
        raise AssertionError(f"descriptor longer than {BLOB_LEN} bytes: {len(raw)}")
    return np.frombuffer(raw.ljust(BLOB_LEN, b"\x00"), dtype=np.uint8).copy()


def descriptor_fields(blob: np.ndarray) -> dict:
    """Parse a ``comfy_quant`` blob back into its JSON fields."""
    return json.loads(bytes(np.asarray(blob, dtype=np.uint8)).rstrip(b"\x00").decode("ascii"))


def quantize_convrot_weight(weight, group_size: int = 256):
    """Rotate then row-wise symmetric INT8 quantise: ``(int8 [N, K], float32 [N, 1])``.

    numpy input (any float/int dtype; cast to float32 like the reference) gives numpy
    outputs; a CUDA tensor (float32/bfloat16/float16) gives CUDA tensors and skips the host.
    """
    import torch

    from . import ops

    if weight.ndim != 2:
        raise ValueError(f"expected a 2D weight, got shape {tuple(weight.shape)}")
    build_hadamard(group_size, np.float32)  # same ValueError as the reference for bad sizes
    if weight.shape[1] % group_size != 0:
        raise ValueError(f"in_features {weight.shape[1]} not divisible by group_size {group_size}")
    if isinstance(weight, torch.Tensor):
        return ops.rotate_quant(weight, group_size, order="reference")
    src = np.ascontiguousarray(weight.astype(np.float32, copy=False))
    if src.shape[0] == 0:
        return np.empty(src.shape, np.int8), np.empty((0, 1), np.float32)
    q, scale = ops.rotate_quant(torch.from_numpy(src).cuda(), group_size, order="reference")
    return q.cpu().numpy(), scale.cpu().numpy()


def dequantize_convrot_weight(q, scale, group_size: int = 256):
    """Inverse of :func:`quantize_convrot_weight`: ``(q * scale) @ H^T`` (fp32)."""
    import torch

    from . import ops

    if q.ndim != 2:
        raise ValueError(f"expected a 2D weight, got shape {tuple(q.shape)}")
    build_hadamard(group_size, np.float32)
    if q.shape[1] % group_size != 0:
        raise ValueError(f"in_features {q.shape[1]} not divisible by group_size {group_size}")
    if isinstance(q, torch.Tensor):
        return ops.dequantize(q, scale, group_size)
    if q.shape[0] == 0:
        return np.empty(q.shape, np.float32)
    qd = torch.from_numpy(np.ascontiguousarray(q, dtype=np.int8)).cuda()
    sd = torch.from_numpy(np.ascontiguousarray(np.asarray(scale, dtype=np.float32).reshape(-1))).cuda()
    return ops.dequantize(qd, sd, group_size).cpu().numpy()
