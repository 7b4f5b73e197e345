"""Rank-r curve replacement of the adaLN modulation linears (host numpy).

Every block's adaLN linear consumes the same time-embedding curve c(t) =
silu(time_embedder(t)). On a dense grid t = linspace(0, 1, grid) that curve is close to
rank r, so the checkpoint stores ``table = c @ P`` [grid, r] once and ``A = W @ P`` [out, r]
per block, with P the top-r right singular vectors of c. ComfyUI detects the format from
the tensor shapes and consumes the table linearly.

This is host code on purpose: the converter must write the same bytes as the reference
(slimdit/curve.py:35-88), which depend on numpy's float32 arithmetic and LAPACK's SVD, and
the work is tiny next to the INT8 quantisation. Same math, same numpy calls and dtypes.
"""

from __future__ import annotations

import math

import numpy as np

FREQ_DIM = 256
TIME_EMBED_DIM = 2688


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def time_embeddings(t: np.ndarray, proj_in_w: np.ndarray, proj_in_b: np.ndarray, proj_out_w: np.ndarray,
                    proj_out_b: np.ndarray) -> np.ndarray:
    """Sinusoidal frequency embedding of fp32 timesteps in [0, 1] through the two-layer embedder."""
    half = FREQ_DIM // 2
    freqs = np.exp(-math.log(10000.0) * np.arange(half, dtype=np.float32) / half)
    phase = t.astype(np.float32)[:, None] * freqs[None, :]
    emb = np.concatenate([np.cos(phase), np.sin(phase)], axis=-1).astype(np.float32)
    hidden = silu(emb @ proj_in_w.T + proj_in_b)
    return hidden @ proj_out_w.T + proj_out_b


def build_curve_basis(proj_in_w: np.ndarray, proj_in_b: np.ndarray, proj_out_w: np.ndarray, proj_out_b: np.ndarray,
                      rank: int = 8, grid: int = 1025) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``(table [grid, rank], basis [D, rank], curve [grid, D])`` for t = linspace(0, 1, grid)."""
    t = np.linspace(0.0, 1.0, grid, dtype=np.float32)
    curve = silu(time_embeddings(t, proj_in_w, proj_in_b, proj_out_w, proj_out_b))
    _, _, vt = np.linalg.svd(curve, full_matrices=False)
    basis = np.ascontiguousarray(vt[:rank].T.astype(np.float32))
    table = (curve @ basis).astype(np.float32)
    return table, basis, curve


def project_weight(weight: np.ndarray, basis: np.ndarray) -> np.ndarray:
    """``A = W @ P``: the per-block linear stored next to the shared table."""
    return weight.astype(np.float32, copy=False) @ basis


def modulation_family(weight: np.ndarray, curve: np.ndarray) -> np.ndarray:
    """Exact modulation ``W @ c(t)^T`` for every grid timestep -> [out, grid]."""
    return weight.astype(np.float32, copy=False) @ curve.T


def curve_residual(weight: np.ndarray, curve: np.ndarray, table: np.ndarray, projected: np.ndarray) -> float:
    """Relative Frobenius error of ``A @ table^T`` against the exact modulation family."""
    exact = modulation_family(weight, curve)
    return float(np.linalg.norm(exact - projected @ table.T) / np.linalg.norm(exact))
