"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

No real MiniMax-H3 weights or activations exist in this environment; these generators stand
in for them (N(0, 0.02) weights with a few outlier input channels scaled x50; Student-t(4)
x 0.5 activations with 16 outlier channels x 30). Values are rounded to bf16 because the
sources are bf16 tensors. Shared by the golden-fixture script, the tests and bench.py.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np


def bf16_round_f32(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bf16 (ties to even); returns fp32 holding bf16 values."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round_f32(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def weight(rows: int, cols: int, seed: int = 0, std: float = 0.02, outlier_frac: float = 0.001,
           outlier_scale: float = 50.0) -> np.ndarray:
    """N(0, std) weight [rows, cols] with round(outlier_frac * cols) (>= 1) input channels x50."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)
    n_out = max(1, int(round(outlier_frac * cols)))
    chans = rng.choice(cols, size=n_out, replace=False)
    w[:, chans] *= np.float32(outlier_scale)
    return bf16_round_f32(w)


def activations(rows: int, cols: int, seed: int = 1, nu: float = 4.0, scale: float = 0.5,
                n_outlier: int = 16, outlier_scale: float = 30.0) -> np.ndarray:
    """Student-t(nu) * scale activations [rows, cols] with n_outlier fixed channels x30."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_t(nu, size=(rows, cols)) * scale).astype(np.float32)
    chans = np.random.default_rng(12345).choice(cols, size=min(n_outlier, cols), replace=False)
    x[:, chans] *= np.float32(outlier_scale)
    return bf16_round_f32(x)


def ffn_hidden(rows: int, cols: int, seed: int = 3) -> np.ndarray:
    """A GELU-shaped FFN hidden [rows, cols] in bf16: h = u * s(1.702 u), s(z) = (1 + z / (1 + |z|)) / 2,
    u = 2 * activations(rows, cols, seed). Rational arithmetic only (every operation correctly rounded),
    so the values are the same on any host; like GELU it keeps large positive inputs and squeezes
    negative ones towards zero, which gives each 256-group a wide spread of magnitudes."""
    u = activations(rows, cols, seed=seed) * np.float32(2.0)
    z = u * np.float32(1.702)
    s = (np.float32(1.0) + z / (np.float32(1.0) + np.abs(z))) * np.float32(0.5)
    return bf16_round_f32((u * s).astype(np.float32))


# --------------------------------------------------------------------------- checkpoints
# Official key layout of one MiniMax-H3 transformer (the key template of the reference's
# tests/test_mapping.py:6-59), with shapes scaled by `hidden` / `ffn` / `time_hidden`.

def official_shapes(n_blocks: int, hidden: int, ffn: int, time_hidden: int, n_refiner: int = 2,
                    patch_in: int = 64, audio_in: int = 32, cond_in: int = 128) -> dict[str, tuple[int, ...]]:
    s: dict[str, tuple[int, ...]] = {}
    for i in range(n_blocks):
        p = f"transformer_blocks.{i}"
        s[f"{p}.adaln_proj.linear.weight"] = (6 * hidden, hidden)
        s[f"{p}.adaln_proj.linear.bias"] = (6 * hidden,)
        s[f"{p}.attn.norm_k.weight"] = (128,)
        s[f"{p}.attn.norm_q.weight"] = (128,)
        for n in ("to_q", "to_k", "to_v"):
            s[f"{p}.attn.{n}.weight"] = (hidden, hidden)
        s[f"{p}.attn.to_out.0.weight"] = (hidden, hidden)
        s[f"{p}.ff.net.0.proj.weight"] = (ffn, hidden)
        s[f"{p}.ff.net.2.weight"] = (hidden, ffn)
        s[f"{p}.norm1.weight"] = (hidden,)
        s[f"{p}.norm2.weight"] = (hidden,)
    for i in range(n_refiner):
        p = f"token_refiner.refiner_blocks.{i}"
        s[f"{p}.attn.norm_k.weight"] = (128,)
        s[f"{p}.attn.norm_q.weight"] = (128,)
        for n in ("to_q", "to_k", "to_v"):
            s[f"{p}.attn.{n}.weight"] = (hidden, hidden)
        s[f"{p}.attn.to_out.0.weight"] = (hidden, hidden)
        s[f"{p}.ff.net.0.proj.weight"] = (ffn, hidden)
        s[f"{p}.ff.net.2.weight"] = (hidden, ffn)
        s[f"{p}.norm1.weight"] = (hidden,)
        s[f"{p}.norm2.weight"] = (hidden,)
    s.update({
        "audio_proj_in.bias": (hidden,), "audio_proj_in.weight": (hidden, audio_in),
        "audio_proj_out.bias": (audio_in,), "audio_proj_out.weight": (audio_in, hidden),
        "context_embedder.bias": (hidden,), "context_embedder.weight": (hidden, cond_in),
        "norm_out.linear.bias": (2 * hidden,), "norm_out.linear.weight": (2 * hidden, hidden),
        "norm_out.norm.weight": (hidden,),
        "proj_in.bias": (hidden,), "proj_in.weight": (hidden, patch_in),
        "proj_out.bias": (patch_in,), "proj_out.weight": (patch_in, hidden),
        "time_embedder.linear_1.bias": (time_hidden,), "time_embedder.linear_1.weight": (time_hidden, 256),
        "time_embedder.linear_2.bias": (hidden,), "time_embedder.linear_2.weight": (hidden, time_hidden),
        "rope.inv_freq": (16,),
        "token_refiner.final_norm.weight": (hidden,),
    })
    return s


def _write_safetensors(path: Path, tensors: dict[str, np.ndarray]) -> None:
    """Minimal bf16/f32 safetensors writer (keys sorted, as the official shards are)."""
    header: dict = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        arr = tensors[name]
        if arr.dtype == np.uint16:
            dt = "BF16"
        elif arr.dtype == np.float32:
            dt = "F32"
        else:
            raise TypeError(arr.dtype)
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        blobs.append(raw)
    hb = json.dumps(header, separators=(",", ":")).encode()
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(hb)))
        fh.write(hb)
        for b in blobs:
            fh.write(b)


def official_checkpoint(directory: str | Path, n_blocks: int = 2, hidden: int = 512, ffn: int = 1024,
                        time_hidden: int = 64, seed: int = 7, n_shards: int = 2) -> Path:
    """Write a seeded synthetic official-layout checkpoint as bf16 safetensors shards.

    Linear weights ~ N(0, 0.02) with outlier input channels x50; norms ~ 1 + N(0, 0.02);
    biases ~ N(0, 0.02); rope.inv_freq as f32.
    """
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    shapes = official_shapes(n_blocks, hidden, ffn, time_hidden)
    rng = np.random.default_rng(seed)
    tensors: dict[str, np.ndarray] = {}
    for i, name in enumerate(sorted(shapes)):
        shape = shapes[name]
        if name == "rope.inv_freq":
            tensors[name] = (1.0 / (10000.0 ** (np.arange(16, dtype=np.float32) / 16))).astype(np.float32)
            continue
        if len(shape) == 2:
            vals = weight(shape[0], shape[1], seed=seed * 1000 + i)
        elif name.endswith("norm.weight") or ".norm" in name:
            vals = bf16_round_f32(1.0 + rng.standard_normal(shape).astype(np.float32) * np.float32(0.02))
        else:
            vals = bf16_round_f32(rng.standard_normal(shape).astype(np.float32) * np.float32(0.02))
        tensors[name] = f32_to_bf16_bits(vals)
    names = sorted(tensors)
    per = (len(names) + n_shards - 1) // n_shards
    for s in range(n_shards):
        part = {n: tensors[n] for n in names[s * per:(s + 1) * per]}
        _write_safetensors(directory / f"diffusion_pytorch_model-{s + 1:05d}-of-{n_shards:05d}.safetensors", part)
    return directory
