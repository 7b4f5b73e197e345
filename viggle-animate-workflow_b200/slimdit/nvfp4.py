"""NVFP4 weight format (same API as the reference's slimdit/nvfp4.py).

An NVFP4 linear is stored as (slimdit/nvfp4.py:3-8 of the reference)

    <base>.weight          uint8   [N, K//2]   two E2M1 values per byte
    <base>.weight_scale    uint8   [N, K//16]  E4M3 block scales in the cuBLAS 128x4 tiled layout
    <base>.weight_scale_2  float32 scalar      per-tensor scale amax / (448 * 6)
    <base>.comfy_quant     uint8   [19]        {"format": "nvfp4"}

The reference refuses to quantise without ``comfy_kitchen`` (its NVFP4 arithmetic lives
there). Here the arithmetic runs in libslimdit_b200.so on the GPU: per-tensor amax, block
scales ``e4m3(min(fl(fl(block_amax / 6) / s2), 448))`` and E2M1 codes rounded half to even
from ``fl(x / fl(s2 * block_scale))``, two per byte with element 2i in the high nibble (the
documented layout above). :class:`ComfyKitchenMissing` is kept for API compatibility
and is raised when no sm_100 device or built library is available.
"""

from __future__ import annotations

import json

import numpy as np

from .int8 import BLOB_LEN

#: Block size of the NVFP4 grid and of the cuBLAS tiled scale layout.
NVFP4_BLOCK = 16
TILE_ROWS = 128
TILE_COLS = 4

NVFP4_DESCRIPTOR = '{"format": "nvfp4"}'


class ComfyKitchenMissing(RuntimeError):
    """Raised when NVFP4 is requested but the quantiser cannot run (no library or device)."""


def _ops():
    from . import _native, ops

    try:
        _native.require_cuda()
    except _native.NativeUnavailable as err:
        raise ComfyKitchenMissing(
            f"NVFP4 conversion needs the sm_100a library and a CUDA device: {err}. "
            "Use --quant int8_convrot, or run on a B200.") from err
    return ops


def nvfp4_available() -> bool:
    try:
        _ops()
    except ComfyKitchenMissing:
        return False
    return True


def comfy_quant_blob() -> np.ndarray:
    """``comfy_quant`` descriptor tensor for an NVFP4 layer."""
    raw = NVFP4_DESCRIPTOR.encode("ascii")
    return np.frombuffer(raw, dtype=np.uint8).copy()


def quantized_shapes(rows: int, cols: int) -> tuple[tuple[int, int], ...]:
    """Shapes of ``(weight, weight_scale)`` for an ``[rows, cols]`` NVFP4 linear."""
    if rows % TILE_ROWS or (cols // NVFP4_BLOCK) % TILE_COLS:
        raise ValueError(f"NVFP4 tiling expects rows%128==0 and (cols/16)%4==0, got {rows}x{cols}")
    return (rows, cols // 2), (rows, cols // NVFP4_BLOCK)


def _pack_host(weight: np.ndarray, with_error: bool):
    import torch

    if weight.ndim != 2:
        raise ValueError(f"expected a 2D weight, got shape {weight.shape}")
    quantized_shapes(*weight.shape)
    ops = _ops()
    src = torch.from_numpy(np.ascontiguousarray(weight, dtype=np.float32)).cuda()
    q, sf, ts = ops.nvfp4_pack(src)
    err = ops.nvfp4_error(q, sf, ts, src) if with_error else None
    out = (q.cpu().numpy(), np.ascontiguousarray(sf.cpu().numpy()), np.asarray(ts.cpu().numpy()[0], dtype=np.float32))
    return out if err is None else (*out, err)


def quantize_nvfp4_weight(weight: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Quantize ``[N, K]`` float32 weights into ``(qdata uint8, block_scale uint8, scale f32)``."""
    return _pack_host(weight, with_error=False)


def quantize_nvfp4_with_error(weight: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray, float]:
    """As :func:`quantize_nvfp4_weight`, plus the round-trip error ``||deq - w|| / ||w||``."""
    return _pack_host(weight, with_error=True)


def descriptor_fields(blob: np.ndarray) -> dict:
    text = bytes(np.asarray(blob, dtype=np.uint8)).rstrip(b"\x00").decode("ascii")
    return json.loads(text)


class GpuPacker:
    """Converter hook: packs one linear on this process's GPU (H2D of the bf16 sources,
    concatenated and half-swapped on the device, NVFP4 pack, D2H) and computes the error
    report on the device. Same call shape as the INT8 quantiser of slimdit.convert."""

    def __init__(self, device):
        import torch

        self.ops = _ops()
        self.device = device
        self.stream = torch.cuda.Stream(device)

    def __call__(self, parts, swap: bool, with_error: bool):
        import torch

        rows = sum(p.shape[0] for p in parts)
        cols = parts[0].shape[1]
        quantized_shapes(rows, cols)
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            dev = torch.empty((rows, cols), dtype=parts[0].dtype, device=self.device)
            r0 = 0
            for p in parts:
                dev[r0:r0 + p.shape[0]].copy_(p)
                r0 += p.shape[0]
            if swap:
                half = rows // 2
                if half * 2 != rows:
                    raise ValueError(f"cannot swap halves of {rows} rows")
                dev = torch.cat([dev[half:], dev[:half]], dim=0)
            if dev.dtype not in (torch.bfloat16, torch.float16, torch.float32):
                dev = dev.float()
            q, sf, ts = self.ops.nvfp4_pack(dev)
            err = self.ops.nvfp4_error(q, sf, ts, dev) if with_error else None
            out = (q.cpu().numpy(), sf.cpu().numpy(), float(ts.cpu()[0]))
        self.stream.synchronize()
        return (*out, err)


__all__ = [
    "BLOB_LEN",
    "ComfyKitchenMissing",
    "NVFP4_BLOCK",
    "comfy_quant_blob",
    "descriptor_fields",
    "nvfp4_available",
    "quantize_nvfp4_weight",
    "quantized_shapes",
]
