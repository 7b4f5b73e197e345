"""ORACLE — test infrastructure, not product code.

CPU restatement (numpy) of the NVFP4 weight format that the reference's slimdit/nvfp4.py
writes, used only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU leg as
the checker.

Parity status: UNPINNED. The reference delegates the arithmetic to ``comfy_kitchen``
(``TensorCoreNVFP4Layout.quantize``, slimdit/nvfp4.py:44-51,72-87), which is neither in the
reference tree nor installed, and whose version the reference does not pin
(pyproject.toml lists no comfy_kitchen). No reference test holds NVFP4 bytes. What is
restated here is the published two-level NVFP4 recipe that the reference's own text
describes (slimdit/nvfp4.py:3-15, docs/DEV_NOTES.md:59-71):

* per-tensor scale ``s2 = fl32(amax / (448 * 6))`` (slimdit/nvfp4.py:8);
* per 16-element block along K: ``bs = fl32(fl32(block_amax / 6) / s2)``, clamped to at most
  448, rounded to FP8 E4M3 (round-half-even, subnormals kept) — "fp8-rounded block scales";
* each element ``v = fl32(x / fl32(s2 * e4m3(bs)))`` (0 where that product is 0), clamped to
  [-6, 6] and rounded half-to-even onto the E2M1 grid {0, .5, 1, 1.5, 2, 3, 4, 6}; the sign
  bit is kept, so negative values that round to 0 give the code 0b1000 — "fp4
  round-to-nearest-even";
* block scales stored in the cuBLAS 128x4 tiled layout ("cuBLAS swizzle"):
  within the 512-byte tile of rows [128i, 128i+128) and scale columns [4j, 4j+4), entry
  (r, c) sits at byte (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4; tiles are ordered
  row-tile-major.

Cross-check (tests/test_gpu_nvfp4.py): flashinfer's fp4_quantize, NVIDIA's NVFP4 quantiser,
gives the same block-scale bytes in the same tiled layout and the same codes except where its
reciprocal-multiply rounding and this recipe's division straddle a grid midpoint (one step).

Nibble order: "two E2M1 values per byte, high nibble first" (slimdit/nvfp4.py:5,
docs/DEV_NOTES.md:64): element 2i of a row goes to the HIGH nibble of byte i, element 2i+1 to
the low nibble.

An all-zero tensor (s2 = 0) quantises to zero codes and zero scales here; the recipe as
written would divide 0 by 0.

The activation side (the runtime op's NVFP4 input quantisation) uses the same recipe with
one global scale per token row instead of per tensor, optionally after the group-256
Hadamard rotation in the butterfly order.
"""

from __future__ import annotations

import numpy as np

F4_MAX = np.float32(6.0)
F8_MAX = np.float32(448.0)
BLOCK = 16
TILE_ROWS = 128
TILE_COLS = 4

# E2M1 magnitudes by code (bit 3 is the sign)
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Round non-negative fp32 (<= 448) to FP8 E4M3 (fn variant) bits, half-to-even.

    NaN maps to 0x7F. Subnormals (below 2^-6) are multiples of 2^-9."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape, dtype=np.uint8)
    nan = np.isnan(x)
    sub = (x < np.float32(2.0 ** -6)) & ~nan
    # subnormal range: code = rint(x * 2^9) (exact scaling, numpy rint is half-to-even)
    out[sub] = np.rint(x[sub].astype(np.float64) * 512.0).astype(np.uint8)
    nrm = ~sub & ~nan
    u = x[nrm].view(np.uint32).astype(np.uint64)
    # keep 3 mantissa bits with round-half-even on the 20 dropped bits
    r = (u + 0x7FFFF + ((u >> 20) & 1)) >> 20          # (biased f32 exponent << 3) | mantissa
    exp = (r >> 3).astype(np.int64) - 127 + 7
    man = (r & 7).astype(np.int64)
    out[nrm] = ((exp << 3) | man).astype(np.uint8)
    out[nan] = 0x7F
    return out


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """FP8 E4M3 (fn) bits -> fp32 (exact)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    exp = (b >> 3) & 0xF
    man = b & 7
    mag = np.where(exp == 0, man * 2.0 ** -9, (8 + man) * np.exp2(exp - 10.0))
    mag = np.where((exp == 15) & (man == 7), np.nan, mag)
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def e2m1_encode(v: np.ndarray) -> np.ndarray:
    """fp32 values already clamped to [-6, 6] -> 4-bit codes (sign in bit 3), half-to-even."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    a = np.abs(v)
    code = ((a > 0.25).astype(np.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5) + (a >= 3.5)
            + (a > 5.0)).astype(np.uint8)
    sign = (v.view(np.uint32) >> 31).astype(np.uint8)
    return code | (sign << 3)


def e2m1_decode(c: np.ndarray) -> np.ndarray:
    c = np.asarray(c, dtype=np.uint8)
    mag = E2M1_VALUES[c & 7]
    return np.where(c & 8, -mag, mag).astype(np.float32)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """[R, K] 4-bit codes -> [R, K/2] bytes, high nibble first (element 2i in the high nibble)."""
    codes = np.asarray(codes, dtype=np.uint8)
    return ((codes[:, 0::2] << 4) | codes[:, 1::2]).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = packed >> 4
    out[:, 1::2] = packed & 0xF
    return out


def to_blocked(sf: np.ndarray) -> np.ndarray:
    """Row-major [R, C] block scales (R % 128 == 0, C % 4 == 0) -> the 128x4 tiled layout,
    returned with the same [R, C] shape (slimdit/nvfp4.py:6, quantized_shapes)."""
    r, c = sf.shape
    if r % TILE_ROWS or c % TILE_COLS:
        raise ValueError(f"blocked layout needs rows % 128 == 0 and cols % 4 == 0, got {sf.shape}")
    t = np.asarray(sf, dtype=np.uint8).reshape(r // 128, 4, 32, c // 4, 4)
    return np.ascontiguousarray(t.transpose(0, 3, 2, 1, 4)).reshape(r, c)


def from_blocked(blk: np.ndarray, rows: int, cols: int) -> np.ndarray:
    t = np.asarray(blk, dtype=np.uint8).reshape(rows // 128, cols // 4, 32, 4, 4)
    return np.ascontiguousarray(t.transpose(0, 3, 2, 1, 4)).reshape(rows, cols)


def global_scale(amax) -> np.float32:
    """fl32(amax / (448 * 6))."""
    return np.float32(np.float32(amax) / np.float32(2688.0))


def _quant_rows(x: np.ndarray, gs: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x fp32 [R, K]; gs fp32 [R] (one global scale per row) -> codes [R, K], scale bytes [R, K/16]."""
    r, k = x.shape
    blocks = x.reshape(r, k // BLOCK, BLOCK)
    bamax = np.abs(blocks).max(axis=2)
    g = gs.reshape(r, 1).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        s = (bamax / F4_MAX).astype(np.float32)
        s2 = np.where(g > 0, (s / np.where(g > 0, g, np.float32(1))).astype(np.float32), np.float32(0))
    s2 = np.minimum(s2, F8_MAX).astype(np.float32)
    sf = e4m3_encode(s2)
    total = (g * e4m3_decode(sf)).astype(np.float32)
    safe = np.where(total == 0, np.float32(1), total).astype(np.float32)
    v = (blocks / safe[:, :, None]).astype(np.float32)
    v = np.where((total == 0)[:, :, None], np.float32(0), v)
    v = np.clip(v, -F4_MAX, F4_MAX).astype(np.float32)
    return e2m1_encode(v.reshape(r, k)), sf


def quantize_nvfp4_weight(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.float32]:
    """Per-tensor NVFP4 of fp32 [N, K] -> (packed uint8 [N, K/2], blocked scales uint8
    [N, K/16], fp32 per-tensor scale). Restates the recipe in the module docstring
    (slimdit/nvfp4.py:72-87 delegates it to comfy_kitchen)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if n % TILE_ROWS or (k // BLOCK) % TILE_COLS or k % BLOCK:
        raise ValueError(f"NVFP4 tiling expects rows%128==0 and (cols/16)%4==0, got {n}x{k}")
    gs = global_scale(np.abs(w).max(initial=np.float32(0)))
    codes, sf = _quant_rows(w, np.full(n, gs, dtype=np.float32))
    return pack_nibbles(codes), to_blocked(sf), gs


def quantize_nvfp4_rows(x: np.ndarray, rotate: bool = False) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-token NVFP4 of activations [M, K] (optionally rotated in the butterfly order first)
    -> (packed [M, K/2], blocked scales [ceil(M/128)*128, K/16] with zero padding rows,
    fp32 row scales [M])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if rotate:
        from . import rotate_butterfly

        x = rotate_butterfly(x)
    m, k = x.shape
    gs = (np.abs(x).max(axis=1, initial=np.float32(0)) / np.float32(2688.0)).astype(np.float32)
    codes, sf = _quant_rows(x, gs)
    mp = -(-m // TILE_ROWS) * TILE_ROWS
    sfp = np.zeros((mp, k // BLOCK), dtype=np.uint8)
    sfp[:m] = sf
    return pack_nibbles(codes), to_blocked(sfp), gs


def dequantize(packed: np.ndarray, blocked: np.ndarray, scale, rows: int | None = None) -> np.ndarray:
    """fp64 values code * e4m3(block scale) * scale (scale per tensor or per row) of
    [rows, K] NVFP4 data. Exact: every factor is a short binary fraction."""
    codes = unpack_nibbles(packed)
    r, k = codes.shape
    rp = blocked.shape[0]
    sf = from_blocked(blocked, rp, k // BLOCK)[:r]
    bs = np.repeat(e4m3_decode(sf).astype(np.float64), BLOCK, axis=1)
    sc = np.asarray(scale, dtype=np.float64).reshape(-1, 1) if np.ndim(scale) else np.float64(scale)
    return e2m1_decode(codes).astype(np.float64) * bs * sc


def gemm_reference_f64(a_packed, a_blocked, a_scale, b_packed, b_blocked, b_scale, bias=None):
    """fp64 reference of the block-scaled FP4 GEMM: dequant(A) @ dequant(B)^T + bias, and the
    sum of |products| per output (for the fp32-accumulation tolerance)."""
    a = dequantize(a_packed, a_blocked, a_scale)
    b = dequantize(b_packed, b_blocked, b_scale)
    y = a @ b.T
    t = np.abs(a) @ np.abs(b).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64).reshape(1, -1)
    return y, t


__all__ = [
    "dequantize", "e2m1_decode", "e2m1_encode", "e4m3_decode", "e4m3_encode", "from_blocked", "gemm_reference_f64",
    "global_scale", "pack_nibbles", "quantize_nvfp4_rows", "quantize_nvfp4_weight", "to_blocked", "unpack_nibbles",
]
