"""ORACLE — test infrastructure, not product code.

CPU restatement (numpy) of the reference's in-place INT8/FP8 flash attention
(comfyui/ComfyUI-SlimDiT/attention_triton.py), used only by ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU leg as the checker.

Parity status: PARTLY PINNED. The reference pins no attention outputs, its kernels are Triton
and need a GPU, and the reference does not travel to the GPU machine. Under Triton's CPU
interpreter (tests/golden/make_attention_golden.py) the unrotated ``quant_int8_rows`` and
``tensor_amax`` run faithfully, and their outputs are committed golden vectors that this
restatement (and the GPU kernels) match bit for bit. The rest is unpinned: on this image's
interpreter ``tl.dot`` of bf16 operands returns meaningless values and the float8e4nv cast
mis-rounds on exponent carries, so the rotated quantiser, ``quant_fp8_global`` and
``flash_int8`` could not be run. What is restated is the algorithm as the reference's source
states it:

* quant_int8_rows (attention_triton.py:79-102): per (token, head) row of D values, optionally
  rotated by the unnormalised +-1 Sylvester Hadamard (``_hadamard``, :47-63), then
  ``scale = max(amax, 1e-8) / 127`` and ``q = clip(floor(x / scale + 0.5), -127, 127)``.
  The rotation here is the exact sum rounded once to fp32 (the reference's ``tl.dot`` sums the
  exact +-x products in the tensor core's own order);
* tensor_amax + quant_fp8_global (:104-129, :283-287): one global ``v_scale =
  max(amax / 448, 1e-8)`` and ``v = e4m3(v / v_scale)`` (round to nearest even, saturating);
* flash_int8 (:131-174): online softmax over 128-key tiles on the int32 scores times the
  outer product of the scales, ``p`` rounded to FP8 before both the PV product and the row
  sum ``l``, ``out = bf16(acc * v_scale / l)``; ``attn_scale = D^-0.5 / D`` with the rotation
  (:297-298).

Arithmetic definition shared with the CUDA kernel (fp32 unless stated): the base-2 logit of
key c in row r is ``y * ra`` with ``y = float(s) * ks[c]`` and ``ra = (qs[r] * attn_scale) *
log2(e)``; per tile ``m' = max(m, max_c(y) * ra)``, ``alpha = 2^(m - m')``, ``p = 2^(y * ra -
m')`` (one fused multiply-add). This is the reference's ``exp2((qk - m) * log2e)`` with
``qk = s * (qs * ks) * attn_scale``, regrouped; the roundings differ from the Triton kernel's.
Exponentials here are exact (fp64, rounded to fp32); the GPU uses the hardware ``ex2`` (a few
fp32 ulps), so an FP8-rounded ``p`` can occasionally land one FP8 step apart — the parity
tests bound that.
"""

from __future__ import annotations

import numpy as np

from .nvfp4 import e4m3_decode, e4m3_encode

LOG2E = np.float32(1.4426950408889634)
Q_MAX = np.float32(127.0)
V_MAX = np.float32(448.0)
TILE_KEYS = 128


def sylvester(dim: int) -> np.ndarray:
    """+-1 Sylvester Hadamard: H[i, j] = (-1)^popcount(i & j) (attention_triton.py:47-63)."""
    if dim <= 0 or dim & (dim - 1):
        raise ValueError(f"dim must be a power of two, got {dim}")
    idx = np.arange(dim, dtype=np.int64)
    bits = idx[:, None] & idx[None, :]
    parity = np.zeros_like(bits)
    for b in range(dim.bit_length()):
        parity += (bits >> b) & 1
    return np.where(parity % 2 == 0, 1.0, -1.0)


def split_packed(qkv: np.ndarray, heads: int, dim: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """[S, 3*H*D] packed rows -> q, k, v as fp32 [S, H, D] (attention_triton.py:185-212 layout)."""
    s = qkv.shape[0]
    x = np.asarray(qkv, dtype=np.float32).reshape(s, 3, heads, dim)
    return x[:, 0], x[:, 1], x[:, 2]


def quant_qk(x: np.ndarray, rotate: bool) -> tuple[np.ndarray, np.ndarray]:
    """[S, H, D] fp32 -> (int8 codes [S, H, D], fp32 scales [S, H])."""
    x = np.asarray(x, dtype=np.float32)
    if rotate:
        y = (x.astype(np.float64) @ sylvester(x.shape[-1])).astype(np.float32)
    else:
        y = x
    amax = np.abs(y).max(axis=-1)
    scale = np.maximum(amax, np.float32(1e-8)).astype(np.float32) / Q_MAX
    t = (y / scale[..., None]).astype(np.float32) + np.float32(0.5)
    q = np.clip(np.floor(t), -127, 127).astype(np.int8)
    return q, scale.astype(np.float32)


def v_scale_of(amax: np.float32) -> np.float32:
    return np.float32(max(np.float32(amax) / V_MAX, np.float32(1e-8)))


def quant_v(v: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """[S, H, D] fp32 -> (e4m3 bits [S, H, D], amax). The scale is ``v_scale_of(amax)``."""
    v = np.asarray(v, dtype=np.float32)
    amax = np.float32(np.abs(v).max()) if v.size else np.float32(0)
    t = (v / v_scale_of(amax)).astype(np.float32)
    sign = (t.view(np.uint32) >> 31).astype(np.uint8) << 7
    mag = np.minimum(np.abs(t), V_MAX)
    return (e4m3_encode(mag) | sign).astype(np.uint8), amax


def transpose_v(codes: np.ndarray, seq_pad: int) -> np.ndarray:
    """[S, H, D] codes -> [H, D, seq_pad] (zero padded), the layout the GPU kernel reads."""
    s, h, d = codes.shape
    out = np.zeros((h, d, seq_pad), dtype=np.uint8)
    out[:, :, :s] = codes.transpose(1, 2, 0)
    return out


def attn_scale(dim: int, rotate: bool) -> np.float32:
    return np.float32(dim ** -0.5 / (dim if rotate else 1.0))


def flash(q8: np.ndarray, qs: np.ndarray, k8: np.ndarray, ks: np.ndarray, v8: np.ndarray, amax: np.float32,
          scale: np.float32) -> np.ndarray:
    """Online-softmax attention over 128-key tiles. q8 int8 [Sq, H, D] with qs [Sq, H]; k8 int8
    [S, H, D] with ks [S, H]; v8 e4m3 bits [S, H, D] (Sq may be a leading subset of the S query
    rows). Returns fp32 values of the bf16 output [Sq, H, D]."""
    s_len, heads, dim = q8.shape
    n_keys = k8.shape[0]
    vs = v_scale_of(amax)
    vv = e4m3_decode(v8).astype(np.float64)
    out = np.empty((s_len, heads, dim), dtype=np.float32)
    for h in range(heads):
        qi = q8[:, h].astype(np.float64)
        ra = ((qs[:, h].astype(np.float32) * np.float32(scale)).astype(np.float32) * LOG2E).astype(np.float32)
        m = np.full(s_len, -np.inf, dtype=np.float32)
        acc = np.zeros((s_len, dim), dtype=np.float32)
        l = np.zeros(s_len, dtype=np.float32)
        for k0 in range(0, n_keys, TILE_KEYS):
            k1 = min(k0 + TILE_KEYS, n_keys)
            # integer dot products of int8 codes: |s| < 2^22, exact in fp64 and in fp32
            sc = (qi @ k8[k0:k1, h].astype(np.float64).T).astype(np.float32)
            y = (sc * ks[k0:k1, h].astype(np.float32)[None, :]).astype(np.float32)
            mx = (y.max(axis=1) * ra).astype(np.float32)
            m_new = np.maximum(m, mx)
            with np.errstate(invalid="ignore"):
                alpha = np.exp2((m - m_new).astype(np.float64)).astype(np.float32)
            arg = (y.astype(np.float64) * ra[:, None].astype(np.float64) - m_new[:, None]).astype(np.float32)
            p = np.exp2(arg.astype(np.float64)).astype(np.float32)
            pq = e4m3_decode(e4m3_encode(p)).astype(np.float64)
            o = pq @ vv[k0:k1, h]
            acc = (acc.astype(np.float64) * alpha[:, None] + o).astype(np.float32)
            l = (l.astype(np.float64) * alpha + pq.sum(axis=1)).astype(np.float32)
            m = m_new
        res = ((acc * vs).astype(np.float32) / l[:, None]).astype(np.float32)
        out[:, h] = _bf16(res)
    return out


def attention_packed(qkv: np.ndarray, heads: int, dim: int, rotate: bool = True) -> np.ndarray:
    """The whole override (attention_triton.py:265-299) on a [S, 3*H*D] packed buffer ->
    fp32 values of the bf16 output [S, H*D]."""
    q, k, v = split_packed(qkv, heads, dim)
    q8, qs = quant_qk(q, rotate)
    k8, ks = quant_qk(k, rotate)
    v8, amax = quant_v(v)
    out = flash(q8, qs, k8, ks, v8, amax, attn_scale(dim, rotate))
    return out.reshape(qkv.shape[0], heads * dim)


def dense_attention_f64(qkv: np.ndarray, heads: int, dim: int) -> np.ndarray:
    """Unquantised softmax(q k^T / sqrt(D)) v in fp64, [S, H*D]."""
    q, k, v = (t.astype(np.float64) for t in split_packed(qkv, heads, dim))
    out = np.empty((qkv.shape[0], heads, dim))
    for h in range(heads):
        lg = q[:, h] @ k[:, h].T * dim ** -0.5
        lg -= lg.max(axis=1, keepdims=True)
        w = np.exp(lg)
        out[:, h] = (w @ v[:, h]) / w.sum(axis=1, keepdims=True)
    return out.reshape(qkv.shape[0], heads * dim)


def _bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


__all__ = [
    "attention_packed", "attn_scale", "dense_attention_f64", "flash", "quant_qk", "quant_v", "split_packed",
    "sylvester", "transpose_v", "v_scale_of",
]
