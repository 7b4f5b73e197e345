"""Convert the official Viggle-Animate checkpoint into the curve + INT8 convrot checkpoint.

    python -m slimdit.convert --src <official transformer dir> --out <file.safetensors>
    torchrun --nproc-per-node 8 -m slimdit.convert --src ... --out ...   # one process per GPU

Drop-in for the reference's slimdit/convert.py (same function signature, flags, output
bytes). The difference is where the time goes: every quantised linear is rotated and
quantised on the GPU (csrc/rotate_quant.cu, in the reference's own summation order, so
the file is byte-identical), straight from the bf16 source bytes; the curve, copy and
derived tensors are small host work done with the same numpy/torch calls as the reference.

Work split: the output layout (names, dtypes, shapes, offsets) is known before any tensor
is produced, so the file is created once with its header and full size, and each tensor is
written at its own offset. With several processes (torchrun; one GPU each) the ops are
partitioned per tensor (greedy by output bytes); every process writes only its tensors; a
barrier orders "file created" before the writes and "all written" before the end. There
is no collective on the data path.
"""

from __future__ import annotations

import argparse
import os
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import curve as curve_mod
from . import mapping
from .int8 import comfy_quant_blob
from .safetensors_io import OffsetWriter, ShardSet, numel, to_bytes

try:
    from tqdm import tqdm
except ImportError:  # pragma: no cover
    def tqdm(it, **_):
        return it


@dataclass
class Report:
    curve_errors: list[float]
    quant_errors: list[float]

    def summary(self) -> str:
        lines = []
        if self.curve_errors:
            worst = max(self.curve_errors)
            lines.append(f"curve fit: {len(self.curve_errors)} blocks checked, worst modulation error {worst * 100:.5f}%")
        if self.quant_errors:
            arr = np.array(self.quant_errors)
            lines.append(f"int8 quant: {len(arr)} layers, per-row error mean {arr.mean() * 100:.4f}% / "
                         f"p95 {np.percentile(arr, 95) * 100:.4f}%")
        return "\n".join(lines) if lines else "(no verification requested)"


def _skipped(name: str, block_limit: int | None) -> bool:
    return block_limit is not None and name.startswith("blocks.") and int(name.split(".")[1]) >= block_limit


def output_manifest(ops: list[mapping.Op], src: ShardSet, rank: int, grid: int, block_limit: int | None,
                    quant: str = "int8_convrot") -> list[tuple[str, str, tuple[int, ...]]]:
    """Ordered (name, dtype, shape) of every tensor the converter writes."""
    out: list[tuple[str, str, tuple[int, ...]]] = [("adaln_t_table", "F32", (grid, rank))]
    for op in ops:
        if _skipped(op.out[0], block_limit):
            continue
        if op.kind == "quant":
            rows = sum(src.manifest[s][1][0] for s in op.src)
            cols = src.manifest[op.src[0]][1][1]
            base = op.out[0][: -len(".weight")]
            if quant == "int8_convrot":
                out += [(f"{base}.weight", "I8", (rows, cols)), (f"{base}.weight_scale", "F32", (rows, 1)),
                        (f"{base}.comfy_quant", "U8", (72,))]
            elif quant == "nvfp4":
                from . import nvfp4
                wshape, sshape = nvfp4.quantized_shapes(rows, cols)
                out += [(f"{base}.weight", "U8", wshape), (f"{base}.weight_scale", "U8", sshape),
                        (f"{base}.weight_scale_2", "F32", ()),
                        (f"{base}.comfy_quant", "U8", (len(nvfp4.NVFP4_DESCRIPTOR),))]
            else:
                raise ValueError(f"unknown quantization format {quant!r}")
        elif op.kind == "copy":
            out.append((op.out[0], op.dtype.upper(), src.manifest[op.src[0]][1]))
        elif op.kind == "concat":
            rows = sum(src.manifest[s][1][0] for s in op.src)
            out.append((op.out[0], op.dtype.upper(), (rows, src.manifest[op.src[0]][1][1])))
        elif op.kind == "curve":
            out.append((op.out[0], op.dtype.upper(), (src.manifest[op.src[0]][1][0], rank)))
        elif op.kind == "derived":
            from .rope import INV_FREQ_LEN
            out.append((op.out[0], op.dtype.upper(), (INV_FREQ_LEN,)))
        else:
            raise ValueError(f"unhandled op kind {op.kind!r}")
    return out


def _prepare(tensor: torch.Tensor, op: mapping.Op) -> torch.Tensor:
    """The op's layout fix-up before storing: swap the row halves ([gate; up] -> [up; gate])."""
    if op.swap_halves:
        half = tensor.shape[0] // 2
        if half * 2 != tensor.shape[0]:
            raise ValueError(f"{op.out[0]}: cannot swap halves of {tuple(tensor.shape)}")
        tensor = torch.cat([tensor[half:], tensor[:half]], dim=0)
    return tensor


def partition(costs: list[int], workers: int) -> list[int]:
    """Greedy longest-first assignment of items to `workers` by cost -> owner per item."""
    owner = [0] * len(costs)
    load = [0] * workers
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        w = min(range(workers), key=lambda w: (load[w], w))
        owner[i] = w
        load[w] += costs[i]
    return owner


def _op_cost(op: mapping.Op, src: ShardSet) -> int:
    cost = sum(src.nbytes(s) for s in op.src)
    if op.kind == "quant":
        cost *= 2  # source read + codes written
    return max(cost, 1)


def _dist():
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        return torch.distributed.get_rank(), torch.distributed.get_world_size()
    return 0, 1


def _barrier(workers: int) -> None:
    if workers > 1:
        torch.distributed.barrier()


class _GpuQuantizer:
    """Quantises one linear on this process's GPU: H2D of the bf16 sources (concatenated and
    half-swapped while copying), reference-order rotate + INT8, D2H of codes and scales; the
    error report (dequantise + relative norm) is computed on the device too."""

    def __init__(self, device: torch.device):
        from . import ops

        self.ops = ops
        self.device = device
        self.stream = torch.cuda.Stream(device)

    def __call__(self, parts: list[torch.Tensor], swap: bool, with_error: bool):
        rows = sum(p.shape[0] for p in parts)
        cols = parts[0].shape[1]
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            dev = torch.empty((rows, cols), dtype=parts[0].dtype, device=self.device)
            r0 = 0
            for p in parts:
                dev[r0:r0 + p.shape[0]].copy_(p, non_blocking=False)
                r0 += p.shape[0]
            if swap:
                half = rows // 2
                if half * 2 != rows:
                    raise ValueError(f"cannot swap halves of {rows} rows")
                dev = torch.cat([dev[half:], dev[:half]], dim=0)
            if dev.dtype not in (torch.bfloat16, torch.float16, torch.float32):
                dev = dev.float()
            q, scale = self.ops.rotate_quant(dev, 256, order="reference")
            err = None
            if with_error:
                deq = self.ops.dequantize(q, scale)
                w = dev.float()
                err = float(torch.linalg.vector_norm(deq - w) / torch.linalg.vector_norm(w))
                del deq, w
            q_h = q.cpu()
            s_h = scale.cpu()
        self.stream.synchronize()
        return q_h.numpy(), s_h.numpy(), err


def convert(src_dir: str | Path, out_path: str | Path, rank: int = 8, grid: int = 1025, block_limit: int | None = None,
            verify_blocks: int = 0, curve_dtype: str = "f16", metadata: dict | None = None,
            quant: str = "int8_convrot", quant_report: bool = True) -> Report:
    """Write the converted checkpoint; returns the quantisation/curve report.

    Same arguments as the reference's ``convert``; ``quant_report=False`` skips the
    dequantise-and-compare error report. Under ``torch.distributed`` each process converts
    its share of the tensors on its current CUDA device.
    """
    worker, workers = _dist()
    src = ShardSet(src_dir)
    ops = mapping.build_plan(src.manifest.keys())
    missing = mapping.missing_sources(ops, src.manifest)
    if missing:
        raise SystemExit(f"missing source tensors: {missing[:5]} (+{max(0, len(missing) - 5)} more)")
    manifest = output_manifest(ops, src, rank, grid, block_limit, quant)
    report = Report(curve_errors=[], quant_errors=[])
    todo = [op for op in ops if not _skipped(op.out[0], block_limit)]
    owner = partition([_op_cost(op, src) for op in todo], workers)
    mine = [op for op, w in zip(todo, owner) if w == worker]

    t0 = time.time()
    if worker == 0:
        writer = OffsetWriter(out_path, manifest, metadata or {"format": "pt"}, create=True)
    _barrier(workers)
    if worker != 0:
        writer = OffsetWriter(out_path, manifest, metadata or {"format": "pt"}, create=False)

    table = basis = None
    need_basis = worker == 0 or any(op.kind == "curve" for op in mine) or verify_blocks
    if need_basis:
        table, basis, _curve = curve_mod.build_curve_basis(
            *(src.get(name).float().numpy() for name in mapping.CURVE_SOURCES), rank=rank, grid=grid)
        del _curve
    if worker == 0:
        writer.write("adaln_t_table", to_bytes(torch.from_numpy(table), "F32"))

    quantizer = None
    if any(op.kind == "quant" for op in mine):
        if quant != "int8_convrot":
            from . import nvfp4
            quantizer = nvfp4.GpuPacker(torch.device("cuda", torch.cuda.current_device()))
        else:
            quantizer = _GpuQuantizer(torch.device("cuda", torch.cuda.current_device()))
    blob = comfy_quant_blob().tobytes()

    for op in tqdm(mine, unit="op", desc=f"convert[{worker}/{workers}]", disable=workers > 1 and worker != 0):
        name = op.out[0]
        if op.kind == "quant":
            base = name[: -len(".weight")]
            parts = [src.get(s) for s in op.src]
            if quant == "int8_convrot":
                q, scale, err = quantizer(parts, op.swap_halves, quant_report)
                writer.write(f"{base}.weight", q.tobytes())
                writer.write(f"{base}.weight_scale", np.ascontiguousarray(scale, dtype=np.float32).tobytes())
                writer.write(f"{base}.comfy_quant", blob)
            else:
                from . import nvfp4
                qd, bs, ts, err = quantizer(parts, op.swap_halves, quant_report)
                writer.write(f"{base}.weight", qd.tobytes())
                writer.write(f"{base}.weight_scale", bs.tobytes())
                writer.write(f"{base}.weight_scale_2", np.float32(ts).tobytes())
                writer.write(f"{base}.comfy_quant", nvfp4.comfy_quant_blob().tobytes())
            if err is not None:
                report.quant_errors.append(err)
            del parts
        elif op.kind == "copy":
            writer.write(name, to_bytes(_prepare(src.get(op.src[0]), op), op.dtype.upper()))
        elif op.kind == "concat":
            parts = [src.get(s) for s in op.src]
            merged = parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)
            writer.write(name, to_bytes(_prepare(merged, op), op.dtype.upper()))
        elif op.kind == "curve":
            projected = curve_mod.project_weight(src.get(op.src[0]).float().numpy(), basis)
            writer.write(name, to_bytes(torch.from_numpy(projected), curve_dtype.upper()))
        elif op.kind == "derived":
            from .rope import rope_inv_freq
            writer.write(name, rope_inv_freq().tobytes())
        else:
            raise ValueError(f"unhandled op kind {op.kind!r}")

    expect = {n for op in mine for n in _outputs(op, quant)} | ({"adaln_t_table"} if worker == 0 else set())
    writer.close(expect=expect)
    _barrier(workers)
    if workers > 1:
        gathered: list = [None] * workers
        torch.distributed.all_gather_object(gathered, report.quant_errors)
        report.quant_errors = [e for part in gathered for e in part]

    if verify_blocks:
        report = _verify(src, table, basis, rank, grid, verify_blocks)
    if worker == 0:
        print(f"wrote {out_path} in {time.time() - t0:.1f}s ({len(manifest)} tensors)")
    return report


def _outputs(op: mapping.Op, quant: str) -> list[str]:
    if op.kind != "quant":
        return [op.out[0]]
    base = op.out[0][: -len(".weight")]
    if quant == "int8_convrot":
        return [f"{base}.weight", f"{base}.weight_scale", f"{base}.comfy_quant"]
    return [f"{base}.weight", f"{base}.weight_scale", f"{base}.weight_scale_2", f"{base}.comfy_quant"]


def _verify(src: ShardSet, table: np.ndarray, basis: np.ndarray, rank: int, grid: int, n_blocks: int) -> Report:
    """Recompute the exact modulation family for the first ``n_blocks`` blocks and measure the fit."""
    _, _, crv = curve_mod.build_curve_basis(*(src.get(n).float().numpy() for n in mapping.CURVE_SOURCES),
                                            rank=rank, grid=grid)
    errors: list[float] = []
    for i in range(n_blocks):
        weight = src.get(f"transformer_blocks.{i}.adaln_proj.linear.weight").float().numpy()
        projected = curve_mod.project_weight(weight, basis)
        errors.append(curve_mod.curve_residual(weight, crv, table, projected))
    return Report(curve_errors=errors, quant_errors=[])


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--src", required=True, help="directory holding the official transformer shards")
    ap.add_argument("--out", required=True, help="output .safetensors path")
    ap.add_argument("--rank", type=int, default=8, help="curve rank (time_embed_dim), default 8")
    ap.add_argument("--grid", type=int, default=1025, help="adaln_t_table rows, default 1025")
    ap.add_argument("--block-limit", type=int, default=None, help="only convert the first N blocks (trials)")
    ap.add_argument("--verify-blocks", type=int, default=0, help="measure curve fit on the first N blocks")
    ap.add_argument("--curve-dtype", choices=["f16", "f32"], default="f16")
    ap.add_argument("--quant", choices=["int8_convrot", "nvfp4"], default="int8_convrot",
                    help="weight format for the block linears")
    args = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not torch.distributed.is_initialized():
        import datetime
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    if int(os.environ.get("RANK", "0")) == 0:
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
    report = convert(args.src, args.out, rank=args.rank, grid=args.grid, block_limit=args.block_limit,
                     verify_blocks=args.verify_blocks, curve_dtype=args.curve_dtype, quant=args.quant)
    if int(os.environ.get("RANK", "0")) == 0:
        print(report.summary())
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


__all__ = ["Report", "convert", "main", "output_manifest", "partition", "numel"]

if __name__ == "__main__":
    raise SystemExit(main())
