"""Verify a converted checkpoint's contents on the GPU (same modes, arguments and report as
the reference's tools/verify_checkpoint.py).

``--reference`` compares every tensor against another slim checkpoint: INT8 linears in the
rotated basis (codes times row scales, verify_checkpoint.py:71-75), NVFP4 linears dequantised,
other tensors as stored; a relative L2 error above the tolerance is a finding
(verify_checkpoint.py:81-118). ``--official`` measures the conversion error of selected INT8 /
NVFP4 linears against the released bf16 weights and the adaLN curve residual of block 0
(verify_checkpoint.py:121-152).

The distances are reduced on the device (slim_rel_l2_int8 / slim_rel_l2, fp64 sums); the INT8
dequantisation for the official mode is the reference-order kernel (bit-identical to
slimdit.int8.dequantize_convrot_weight); the curve residual stays on the host with the
reference's numpy code path.

    python -m slimdit.verify --checkpoint ours.safetensors --reference reference.safetensors
    python -m slimdit.verify --checkpoint ours.safetensors --official /models/viggle-official
"""

from __future__ import annotations

import argparse
import re
import sys
from pathlib import Path

import numpy as np
import torch

from . import curve as curve_mod
from .int8 import descriptor_fields
from .safetensors_io import ShardSet

OFFICIAL_FOR = {
    "attn.qkv_proj.weight": ("attn.to_q.weight", "attn.to_k.weight", "attn.to_v.weight"),
    "attn.out_proj.weight": ("attn.to_out.0.weight",),
    "mlp.fc1.weight": ("ff.net.0.proj.weight",),
    "mlp.fc2.weight": ("ff.net.2.weight",),
}

#: Curve tensors are derived analytically and differ between releases: excluded from the
#: reference comparison, covered by the official-weight mode (verify_checkpoint.py:45-47).
CURVE_KEYS = re.compile(r"adaln_t_table|adaln_proj")


def _device() -> torch.device:
    from . import _native

    _native.require_cuda()
    return torch.device("cuda", torch.cuda.current_device())


class _Dist:
    """fp64 [sum (a-b)^2, sum b^2] accumulators on the device."""

    def __init__(self, dev):
        from . import _native

        self.nat = _native
        self.lib = _native.load()
        self.dev = dev
        self.acc = torch.zeros((2,), dtype=torch.float64, device=dev)

    def rel(self) -> float:
        e2, b2 = self.acc.cpu().tolist()
        self.acc.zero_()
        return float(np.sqrt(e2 / b2)) if b2 else 0.0

    def int8(self, qa, sa, qb, sb) -> float:
        rows, k = qa.shape
        st = torch.cuda.current_stream(self.dev).cuda_stream
        self.nat.check(self.lib.slim_rel_l2_int8(qa.data_ptr(), sa.data_ptr(), qb.data_ptr(), sb.data_ptr(), rows, k,
                                                 self.acc.data_ptr(), st))
        return self.rel()

    def dense(self, a: torch.Tensor, b: torch.Tensor) -> float:
        from .ops import _DT

        a, b = a.contiguous(), b.contiguous()
        for t in (a, b):
            if t.dtype not in _DT:
                raise TypeError(f"cannot compare dtype {t.dtype}")
        st = torch.cuda.current_stream(self.dev).cuda_stream
        self.nat.check(self.lib.slim_rel_l2(a.data_ptr(), _DT[a.dtype], b.data_ptr(), _DT[b.dtype], a.numel(),
                                            self.acc.data_ptr(), st))
        return self.rel()


def _format(src: ShardSet, key: str) -> str | None:
    if not key.endswith(".weight"):
        return None
    desc = key[: -len(".weight")] + ".comfy_quant"
    if desc not in src.manifest:
        return None
    return descriptor_fields(src.get(desc).numpy()).get("format")


def _device_value(src: ShardSet, key: str, dev, rotated: bool):
    """("int8", codes, row scales) in the rotated basis, or ("dense", fp32/bf16/f16 tensor)."""
    from . import ops

    tensor = src.get(key)
    fmt = _format(src, key)
    if fmt == "nvfp4":
        base = key[: -len(".weight")]
        q = tensor.to(dev)
        bs = src.get(f"{base}.weight_scale").view(torch.uint8).to(dev)
        s2 = src.get(f"{base}.weight_scale_2").float().reshape(1).to(dev)
        return ("dense", ops.nvfp4_dequantize(q, bs, s2))
    scale_key = key[: -len(".weight")] + ".weight_scale" if key.endswith(".weight") else None
    if scale_key is not None and scale_key in src.manifest and tensor.dtype == torch.int8:
        q = tensor.to(dev)
        s = src.get(scale_key).float().reshape(-1).to(dev)
        if rotated:
            return ("int8", q, s)
        return ("dense", ops.dequantize(q, s))
    if tensor.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        tensor = tensor.float()
    return ("dense", tensor.to(dev))


def compare_reference(ours: ShardSet, ref: ShardSet, tolerance: float, limit: int) -> int:
    dev = _device()
    dist = _Dist(dev)
    shared = sorted(k for k in set(ours.manifest) & set(ref.manifest) if not CURVE_KEYS.search(k))
    mismatched_layout = sorted(set(ours.manifest) ^ set(ref.manifest))
    worst: list[tuple[float, str]] = []
    failures = 0
    skipped_format = 0
    for key in shared:
        if key.endswith(".comfy_quant"):
            if bytes(ours.get(key).numpy().tobytes()) != bytes(ref.get(key).numpy().tobytes()):
                print(f"  DESCRIPTOR MISMATCH {key}")
                failures += 1
            continue
        if _format(ours, key) != _format(ref, key):
            skipped_format += 1
            continue
        a, b = _device_value(ours, key, dev, rotated=True), _device_value(ref, key, dev, rotated=True)
        shape_a = tuple(a[1].shape)
        shape_b = tuple(b[1].shape)
        if shape_a != shape_b or a[0] != b[0]:
            print(f"  SHAPE MISMATCH {key}: {shape_a} vs {shape_b}")
            failures += 1
            continue
        rel = dist.int8(a[1], a[2], b[1], b[2]) if a[0] == "int8" else dist.dense(a[1], b[1])
        worst.append((rel, key))
    worst.sort(reverse=True)
    print(f"compared {len(shared)} tensors (curve keys excluded); {len(mismatched_layout)} keys unique to one side")
    if skipped_format:
        print(f"  {skipped_format} tensors skipped: different quantization format than the reference")
    if mismatched_layout:
        print(f"  one-sided keys (first 5): {mismatched_layout[:5]}")
    print(f"worst {limit} deviations from the reference:")
    for rel, key in worst[:limit]:
        flag = "FAIL" if rel > tolerance else "ok  "
        print(f"  [{flag}] {rel * 100:9.4f}%  {key}")
    failures += sum(1 for rel, _ in worst if rel > tolerance)
    print(f">>> {failures} findings (tolerance {tolerance * 100:.2f}%)")
    return failures


def official_quant_errors(slim: ShardSet, official: ShardSet, layers: list[str]) -> dict[str, float]:
    """Relative conversion error of each named linear against the official bf16 weights."""
    dev = _device()
    dist = _Dist(dev)
    out = {}
    for key in layers:
        block = key.split(".")[1]
        suffix = key.split(".", 2)[2]
        parts = [official.get(f"transformer_blocks.{block}.{n}").to(dev) for n in OFFICIAL_FOR[suffix]]
        ref = parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)
        if suffix == "mlp.fc1.weight":
            # the runtime's swiglu takes [up; gate]; the released checkpoint stores [gate; up]
            half = ref.shape[0] // 2
            ref = torch.cat([ref[half:], ref[:half]], dim=0)
        restored = _device_value(slim, key, dev, rotated=False)[1]
        out[key] = dist.dense(restored, ref)
    return out


def compare_official(slim: ShardSet, official: ShardSet, layers: list[str], rank: int, grid: int) -> int:
    failures = 0
    for key, rel in official_quant_errors(slim, official, layers).items():
        print(f"  {key}: quant error {rel * 100:.4f}%")
        failures += rel > 0.15
    emb = (
        official.get("time_embedder.linear_1.weight").float().numpy(),
        official.get("time_embedder.linear_1.bias").float().numpy(),
        official.get("time_embedder.linear_2.weight").float().numpy(),
        official.get("time_embedder.linear_2.bias").float().numpy(),
    )
    table = slim.get("adaln_t_table").float().numpy()
    curve = curve_mod.silu(curve_mod.time_embeddings(np.linspace(0, 1, grid, dtype=np.float32), *emb))
    weight = official.get("transformer_blocks.0.adaln_proj.linear.weight").float().numpy()
    projected = slim.get("blocks.0.adaln_proj.linear.weight").float().numpy()
    residual = curve_mod.curve_residual(weight, curve, table, projected)
    print(f"  blocks.0 curve: modulation error {residual * 100:.5f}% (rank {rank}, grid {grid})")
    failures += residual > 5e-4
    return failures


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--checkpoint", required=True)
    ap.add_argument("--reference", default=None, help="another slim checkpoint to compare against")
    ap.add_argument("--official", default=None, help="directory of official shards")
    ap.add_argument("--tolerance", type=float, default=0.02)
    ap.add_argument("--layers", default="blocks.0.attn.qkv_proj.weight,blocks.0.mlp.fc1.weight,blocks.17.mlp.fc2.weight")
    ap.add_argument("--rank", type=int, default=8)
    ap.add_argument("--grid", type=int, default=1025)
    args = ap.parse_args(argv)

    slim = ShardSet(Path(args.checkpoint))
    print(f"checkpoint: {args.checkpoint} ({len(slim.manifest)} tensors)")
    failures = 0
    if args.reference:
        failures += compare_reference(slim, ShardSet(Path(args.reference)), args.tolerance, 10)
    if args.official:
        failures += compare_official(slim, ShardSet(args.official), [k.strip() for k in args.layers.split(",") if k.strip()],
                                     args.rank, args.grid)
    print("CONTENTS OK" if not failures else f"CONTENTS SUSPECT ({failures} findings)")
    return 0 if not failures else 1


if __name__ == "__main__":
    sys.exit(main())
