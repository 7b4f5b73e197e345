"""Verify a converted checkpoint's contents on the GPU (same modes, arguments and report as
the reference's tools/verify_checkpoint.py).

``--reference`` compares every tensor against another slim checkpoint: INT8 linears in the
rotated basis (codes times row scales, verify_checkpoint.py:71-75), NVFP4 linears dequantised,
other tensors as stored; a relative L2 error above the tolerance is a finding
(verify_checkpoint.py:81-118). ``--official`` measures the conversion error of selected INT8 /
NVFP4 linears against the released bf16 weights and the adaLN curve residual of block 0
(verify_checkpoint.py:121-152).

How it is organised here: a comparison is planned on the host first (which tensors, in which
form, which ones cannot be compared), then every distance of the plan is reduced on the device
into one fp64 array (slim_rel_l2_int8 / slim_rel_l2) that is read back once. The INT8
dequantisation of the official mode is the reference-order kernel (bit-identical to
slimdit.int8.dequantize_convrot_weight); the curve residual stays on the host with the
reference's numpy code path. Which official tensors make up each quantised linear comes from
the converter's own key plan (slimdit/mapping.py).

    python -m slimdit.verify --checkpoint ours.safetensors --reference reference.safetensors
    python -m slimdit.verify --checkpoint ours.safetensors --official /models/viggle-official
"""

from __future__ import annotations

import argparse
import dataclasses
import sys
from pathlib import Path

import numpy as np
import torch

from . import curve as curve_mod
from . import mapping
from .int8 import descriptor_fields
from .safetensors_io import ShardSet

#: quantised linear (suffix inside a block) -> the official tensors it is made of, in order
OFFICIAL_FOR = {out: srcs for out, srcs, _ in mapping.QUANT_BLOCK_LAYERS}
#: quantised linears whose two halves the converter exchanges ([gate; up] -> [up; gate])
SWAPPED = {out for out, _, swap in mapping.QUANT_BLOCK_LAYERS if swap}


def is_curve_key(key: str) -> bool:
    """Curve tensors (the shared table and each block's projected adaLN weight) are derived
    analytically and differ between releases: the reference mode leaves them out, the
    official mode checks them (verify_checkpoint.py:45-47)."""
    return key == "adaln_t_table" or ".adaln_proj." in key


def _device() -> torch.device:
    from . import _native

    _native.require_cuda()
    return torch.device("cuda", torch.cuda.current_device())


class _Distances:
    """Relative L2 distances of n tensor pairs, reduced on the device: slot i accumulates
    [sum (a - b)^2, sum b^2] in fp64; ``values()`` reads all slots back at once."""

    def __init__(self, dev: torch.device, n: int):
        from . import _native

        self.nat, self.lib, self.dev = _native, _native.load(), dev
        self.acc = torch.zeros((max(n, 1), 2), dtype=torch.float64, device=dev)

    def _slot(self, i: int) -> int:
        return self.acc[i].data_ptr()

    def int8(self, i: int, qa, sa, qb, sb) -> None:
        """Slot i: INT8 rows in the rotated basis, fl32(q * row scale) on both sides."""
        rows, k = qa.shape
        st = torch.cuda.current_stream(self.dev).cuda_stream
        self.nat.check(self.lib.slim_rel_l2_int8(qa.data_ptr(), sa.data_ptr(), qb.data_ptr(), sb.data_ptr(), rows, k,
                                                 self._slot(i), st))

    def dense(self, i: int, a: torch.Tensor, b: torch.Tensor) -> None:
        """Slot i: two tensors of float dtypes, compared as fp32 values."""
        from .ops import _DT

        a, b = a.contiguous(), b.contiguous()
        for t in (a, b):
            if t.dtype not in _DT:
                raise TypeError(f"cannot compare dtype {t.dtype}")
        st = torch.cuda.current_stream(self.dev).cuda_stream
        self.nat.check(self.lib.slim_rel_l2(a.data_ptr(), _DT[a.dtype], b.data_ptr(), _DT[b.dtype], a.numel(),
                                            self._slot(i), st))

    def values(self) -> np.ndarray:
        e2, b2 = self.acc.cpu().numpy().T
        with np.errstate(invalid="ignore", divide="ignore"):
            return np.where(b2 > 0, np.sqrt(e2 / np.where(b2 > 0, b2, 1.0)), 0.0)


def _quant_format(src: ShardSet, key: str) -> str | None:
    """The comfy_quant format of a ``*.weight`` (None for tensors stored as they are)."""
    if not key.endswith(".weight"):
        return None
    desc = key[: -len(".weight")] + ".comfy_quant"
    return descriptor_fields(src.get(desc).numpy()).get("format") if desc in src.manifest else None


def _on_device(src: ShardSet, key: str, dev, rotated: bool):
    """A tensor in the form it is compared in: ("int8", codes, row scales) in the rotated basis
    (rotated=True), else ("dense", float tensor) - INT8 linears rotated back to the original
    basis, NVFP4 linears dequantised, everything else as stored (widened to fp32 if needed)."""
    from . import ops

    tensor = src.get(key)
    base = key[: -len(".weight")] if key.endswith(".weight") else None
    if _quant_format(src, key) == "nvfp4":
        block_scale = src.get(f"{base}.weight_scale").view(torch.uint8).to(dev)
        tensor_scale = src.get(f"{base}.weight_scale_2").float().reshape(1).to(dev)
        return "dense", ops.nvfp4_dequantize(tensor.to(dev), block_scale, tensor_scale)
    if base is not None and tensor.dtype == torch.int8 and f"{base}.weight_scale" in src.manifest:
        codes = tensor.to(dev)
        scales = src.get(f"{base}.weight_scale").float().reshape(-1).to(dev)
        return ("int8", codes, scales) if rotated else ("dense", ops.dequantize(codes, scales))
    if tensor.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        tensor = tensor.float()
    return "dense", tensor.to(dev)


@dataclasses.dataclass
class _Plan:
    """What a reference comparison does, decided before any device work."""

    compared: list[str]          # every shared, non-curve key
    one_sided: list[str]         # keys present in only one of the two checkpoints
    descriptors: list[str]       # comfy_quant tensors: compared byte for byte
    distances: list[str]         # tensors whose distance is measured on the device
    format_skipped: int          # stored in a different quantisation format on the two sides


def _plan(ours: ShardSet, ref: ShardSet) -> _Plan:
    shared = sorted(k for k in ours.manifest.keys() & ref.manifest.keys() if not is_curve_key(k))
    descriptors = [k for k in shared if k.endswith(".comfy_quant")]
    rest = [k for k in shared if not k.endswith(".comfy_quant")]
    same_format = [k for k in rest if _quant_format(ours, k) == _quant_format(ref, k)]
    return _Plan(compared=shared, one_sided=sorted(ours.manifest.keys() ^ ref.manifest.keys()),
                 descriptors=descriptors, distances=same_format, format_skipped=len(rest) - len(same_format))


def compare_reference(ours: ShardSet, ref: ShardSet, tolerance: float, limit: int) -> int:
    """The reference mode: prints the report, returns the number of findings."""
    dev = _device()
    plan = _plan(ours, ref)
    findings = 0
    for key in plan.descriptors:
        if ours.get(key).numpy().tobytes() != ref.get(key).numpy().tobytes():
            print(f"  DESCRIPTOR MISMATCH {key}")
            findings += 1
    dist = _Distances(dev, len(plan.distances))
    measured: list[str] = []
    for key in plan.distances:
        a, b = _on_device(ours, key, dev, rotated=True), _on_device(ref, key, dev, rotated=True)
        if a[0] != b[0] or a[1].shape != b[1].shape:
            print(f"  SHAPE MISMATCH {key}: {tuple(a[1].shape)} vs {tuple(b[1].shape)}")
            findings += 1
            continue
        slot = len(measured)
        if a[0] == "int8":
            dist.int8(slot, a[1], a[2], b[1], b[2])
        else:
            dist.dense(slot, a[1], b[1])
        measured.append(key)
    rel = dist.values()[: len(measured)]
    order = np.argsort(-rel, kind="stable")
    print(f"compared {len(plan.compared)} tensors (curve keys excluded); {len(plan.one_sided)} keys unique to one side")
    if plan.format_skipped:
        print(f"  {plan.format_skipped} tensors skipped: different quantization format than the reference")
    if plan.one_sided:
        print(f"  one-sided keys (first 5): {plan.one_sided[:5]}")
    print(f"worst {limit} deviations from the reference:")
    for i in order[:limit]:
        print(f"  [{'FAIL' if rel[i] > tolerance else 'ok  '}] {rel[i] * 100:9.4f}%  {measured[i]}")
    findings += int((rel > tolerance).sum())
    print(f">>> {findings} findings (tolerance {tolerance * 100:.2f}%)")
    return findings


def _official_weight(official: ShardSet, key: str, dev) -> torch.Tensor:
    """The released bf16 weight that quantised linear ``key`` (blocks.<i>.<suffix>) was made
    from, assembled the way the converter assembles it (slimdit/mapping.py)."""
    _, block, suffix = key.split(".", 2)
    parts = [official.get(f"transformer_blocks.{block}.{name}").to(dev) for name in OFFICIAL_FOR[suffix]]
    weight = torch.cat(parts, dim=0) if len(parts) > 1 else parts[0]
    if suffix in SWAPPED:  # the runtime's swiglu takes [up; gate]; the release stores [gate; up]
        weight = torch.cat(weight.chunk(2, dim=0)[::-1], dim=0)
    return weight


def official_quant_errors(slim: ShardSet, official: ShardSet, layers: list[str]) -> dict[str, float]:
    """Relative conversion error of each named linear against the official bf16 weights."""
    dev = _device()
    dist = _Distances(dev, len(layers))
    for slot, key in enumerate(layers):
        dist.dense(slot, _on_device(slim, key, dev, rotated=False)[1], _official_weight(official, key, dev))
    return dict(zip(layers, (float(v) for v in dist.values())))


def compare_official(slim: ShardSet, official: ShardSet, layers: list[str], rank: int, grid: int) -> int:
    """The official-weight mode: prints the report, returns the number of findings."""
    errors = official_quant_errors(slim, official, layers)
    for key, rel in errors.items():
        print(f"  {key}: quant error {rel * 100:.4f}%")
    findings = sum(rel > 0.15 for rel in errors.values())
    embedder = [official.get(f"time_embedder.{name}").float().numpy()
                for name in ("linear_1.weight", "linear_1.bias", "linear_2.weight", "linear_2.bias")]
    t = np.linspace(0, 1, grid, dtype=np.float32)
    curve = curve_mod.silu(curve_mod.time_embeddings(t, *embedder))
    residual = curve_mod.curve_residual(official.get("transformer_blocks.0.adaln_proj.linear.weight").float().numpy(),
                                        curve, slim.get("adaln_t_table").float().numpy(),
                                        slim.get("blocks.0.adaln_proj.linear.weight").float().numpy())
    print(f"  blocks.0 curve: modulation error {residual * 100:.5f}% (rank {rank}, grid {grid})")
    return findings + int(residual > 5e-4)


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

    checkpoint = ShardSet(Path(args.checkpoint))
    print(f"checkpoint: {args.checkpoint} ({len(checkpoint.manifest)} tensors)")
    modes = []
    if args.reference:
        modes.append(lambda: compare_reference(checkpoint, ShardSet(Path(args.reference)), args.tolerance, 10))
    if args.official:
        layers = [name.strip() for name in args.layers.split(",") if name.strip()]
        modes.append(lambda: compare_official(checkpoint, ShardSet(args.official), layers, args.rank, args.grid))
    findings = sum(mode() for mode in modes)
    print("CONTENTS OK" if not findings else f"CONTENTS SUSPECT ({findings} findings)")
    return 1 if findings else 0


if __name__ == "__main__":
    sys.exit(main())
