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


_ST_TORCH = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}


def _raw_bytes(src: ShardSet, op: mapping.Op) -> np.ndarray | None:
    """The output bytes of a copy/concat op assembled from the sources' stored bytes, when the
    op is a pure byte rearrangement (same dtype, optional half swap) or a bf16 -> f32 widening
    (exact); None when it needs a rounding cast (done with torch as in the reference)."""
    dts = {src.manifest[name][0] for name in op.src}
    target = op.dtype.upper()
    if len(dts) != 1:
        return None
    stored = dts.pop()
    if stored != target and not (stored == "BF16" and target == "F32"):
        return None
    total = sum(src.nbytes(name) for name in op.src)
    buf = np.empty((total,), dtype=np.uint8)
    off = 0
    for name in op.src:
        off += src.read_into(name, buf, off)
    if op.swap_halves:
        rows = sum(src.manifest[name][1][0] for name in op.src)
        if rows % 2:
            raise ValueError(f"{op.out[0]}: cannot swap halves of {rows} rows")
        half = total // 2
        buf = np.concatenate([buf[half:], buf[:half]])
    if stored == target:
        return buf
    return (buf.view(np.uint16).astype(np.uint32) << 16).view(np.float32)


class _HostWiden:
    """bf16 -> fp32 of a large source tensor (exact, as the reference's ``.float()``) from its
    stored bytes, into buffers reused per host thread (no per-call allocation)."""

    def __init__(self):
        import threading

        self.local = threading.local()

    @staticmethod
    def accepts(src: ShardSet, name: str) -> bool:
        return src.manifest[name][0] == "BF16" and len(src.manifest[name][1]) == 2

    def __call__(self, src: ShardSet, name: str) -> np.ndarray:
        rows, cols = src.manifest[name][1]
        n = rows * cols
        loc = self.local
        if getattr(loc, "u16", None) is None or loc.u16.size < n:
            loc.u16 = np.empty((n,), dtype=np.uint16)
            loc.u32 = np.empty((n,), dtype=np.uint32)
        u16, u32 = loc.u16[:n], loc.u32[:n]
        src.read_into(name, u16.view(np.uint8), 0)
        np.left_shift(u16, 16, out=u32, dtype=np.uint32)
        return u32.view(np.float32).reshape(rows, cols)


class _Pipeline:
    """The quantised linears of one process as a three-stage pipeline, so that reading the
    sources, the GPU work and writing the results overlap across linears instead of taking
    turns:

    * reader threads (two): the source tensors' stored bytes straight from the shard files into
      pinned staging buffers (positional reads, concatenated in q/k/v order);
    * this thread: one async H2D per linear on a copy stream, then on a compute stream the
      half swap, the reference-order rotate + INT8 kernel, the device error report and the
      D2H of codes and scales into pinned output buffers;
    * writer thread: waits for that linear's D2H event and writes its three tensors at their
      header offsets.

    DEPTH staging buffers of each kind rotate; a buffer is refilled only after the copy that
    read it (CUDA event) or the write that used it (future) has finished. The bytes written
    are those of the sequential path: same kernel, same inputs, positional writes."""

    DEPTH = 3

    def __init__(self, device: torch.device, src: ShardSet, writer, blob: bytes, with_error: bool):
        from concurrent.futures import ThreadPoolExecutor

        from . import ops

        self.ops = ops
        self.dev = device
        self.src = src
        self.writer = writer
        self.blob = blob
        self.with_error = with_error
        self.h2d = torch.cuda.Stream(device)
        self.comp = torch.cuda.Stream(device)
        self.reader = ThreadPoolExecutor(2, thread_name_prefix="convert-read")
        self.wpool = ThreadPoolExecutor(1, thread_name_prefix="convert-write")
        self.stage_in: list = [None] * self.DEPTH
        self.stage_q: list = [None] * self.DEPTH
        self.stage_s: list = [None] * self.DEPTH
        self.in_done: list = [None] * self.DEPTH     # event: the H2D that read stage_in[slot]
        self.out_done: list = [None] * self.DEPTH    # future: the write that used stage_q/s[slot]
        self.errors: list = []

    @staticmethod
    def accepts(op, src: ShardSet) -> bool:
        return all(src.manifest[name][0] in _ST_TORCH for name in op.src) and \
            len({src.manifest[name][0] for name in op.src}) == 1

    def _pinned(self, store: list, slot: int, nbytes: int) -> torch.Tensor:
        buf = store[slot]
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty((nbytes,), dtype=torch.uint8, pin_memory=True)
            store[slot] = buf
        return buf

    def _read(self, op, slot: int):
        if self.in_done[slot] is not None:
            self.in_done[slot].synchronize()
        nbytes = sum(self.src.nbytes(name) for name in op.src)
        buf = self._pinned(self.stage_in, slot, nbytes)
        arr = buf.numpy()
        off = 0
        for name in op.src:
            off += self.src.read_into(name, arr, off)
        rows = sum(self.src.manifest[name][1][0] for name in op.src)
        cols = self.src.manifest[op.src[0]][1][1]
        return buf, nbytes, _ST_TORCH[self.src.manifest[op.src[0]][0]], rows, cols

    def _write(self, base: str, done: torch.cuda.Event, q_buf, s_buf, nq: int, ns: int, keep) -> None:
        done.synchronize()
        del keep
        self.writer.write(f"{base}.weight", memoryview(q_buf.numpy()[:nq]))
        self.writer.write(f"{base}.weight_scale", memoryview(s_buf.numpy()[:ns]))
        self.writer.write(f"{base}.comfy_quant", self.blob)

    def run(self, quant_ops: list) -> list[float]:
        from collections import deque

        reads: deque = deque()
        nxt = 0
        for i, op in enumerate(quant_ops):
            while nxt < len(quant_ops) and len(reads) < self.DEPTH - 1:
                reads.append(self.reader.submit(self._read, quant_ops[nxt], nxt % self.DEPTH))
                nxt += 1
            buf, nbytes, dtype, rows, cols = reads.popleft().result()
            slot = i % self.DEPTH
            with torch.cuda.device(self.dev):
                with torch.cuda.stream(self.h2d):
                    raw = torch.empty((nbytes,), dtype=torch.uint8, device=self.dev)
                    raw.copy_(buf[:nbytes], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.h2d)
                self.in_done[slot] = ev
                if self.out_done[slot] is not None:
                    self.out_done[slot].result()  # the output staging of this slot is written out
                with torch.cuda.stream(self.comp):
                    self.comp.wait_event(ev)
                    raw.record_stream(self.comp)
                    w = raw.view(dtype).view(rows, cols)
                    if op.swap_halves:
                        half = rows // 2
                        if half * 2 != rows:
                            raise ValueError(f"cannot swap halves of {rows} rows")
                        w = torch.cat([w[half:], w[:half]], dim=0)
                    q, scale = self.ops.rotate_quant(w, 256, order="reference")
                    if self.with_error:
                        deq = self.ops.dequantize(q, scale)
                        wf = w.float()
                        self.errors.append(torch.linalg.vector_norm(deq - wf) / torch.linalg.vector_norm(wf))
                        del deq, wf
                    nq, ns = q.numel(), scale.numel() * 4
                    q_buf = self._pinned(self.stage_q, slot, nq)
                    s_buf = self._pinned(self.stage_s, slot, ns)
                    q_buf[:nq].copy_(q.view(-1).view(torch.uint8), non_blocking=True)
                    s_buf[:ns].copy_(scale.view(-1).view(torch.uint8), non_blocking=True)
                    done = torch.cuda.Event()
                    done.record(self.comp)
            base = op.out[0][: -len(".weight")]
            self.out_done[slot] = self.wpool.submit(self._write, base, done, q_buf, s_buf, nq, ns, (raw, w, q, scale))
        for f in self.out_done:
            if f is not None:
                f.result()
        self.reader.shutdown()
        self.wpool.shutdown()
        torch.cuda.synchronize(self.dev)
        return [float(e) for e in self.errors]


def convert(src_dir: str | Path, out_path: str | Path, rank: int = 8, grid: int = 1025, block_limit: int | None = None,
            verify_blocks: int = 0, curve_dtype: str = "f16", metadata: dict | None = None,
            quant: str = "int8_convrot", quant_report: bool = True, pipeline: bool = True) -> Report:
    """Write the converted checkpoint; returns the quantisation/curve report.

    Same arguments as the reference's ``convert``; ``quant_report=False`` skips the
    dequantise-and-compare error report. Under ``torch.distributed`` each process converts
    its share of the tensors on its current CUDA device. ``pipeline=True`` overlaps source
    reads, GPU work and writes across the INT8 linears (``_Pipeline``) and runs the curve
    basis and the curve, copy and derived tensors on four host threads alongside (copies as
    positional byte moves, the adaLN weights widened from their stored bf16 bytes);
    ``pipeline=False`` takes the ops one at a time. Both write the same bytes. If the
    conversion fails on any rank, every rank raises and the partial output file is removed
    (the positional writer sizes the file up front, so a partial one would look complete).
    """

    worker, workers = _dist()
    steps = _convert_steps(src_dir, out_path, rank, grid, block_limit, verify_blocks, curve_dtype, metadata, quant,
                           quant_report, pipeline, worker, workers)
    # Two synchronisation points: after rank 0 has created the output file, and after every
    # rank has written its tensors. At each, every rank reports whether its part succeeded (a
    # MIN all-reduce, reached by failing ranks too); on any failure rank 0 removes the partial
    # output (pre-sized, it would look complete) and every rank raises.
    for _ in range(2):
        failure = None
        try:
            next(steps)
        except BaseException as exc:  # noqa: BLE001 - re-raised below, after the collective
            failure = exc
        if not _all_ok(failure is None, workers):
            steps.close()
            if worker == 0:
                Path(out_path).unlink(missing_ok=True)
            if failure is not None:
                raise failure
            raise RuntimeError("conversion failed on another rank; the partial output was removed")
    try:
        next(steps)
    except StopIteration as done:
        return done.value
    raise AssertionError("conversion steps did not finish")  # pragma: no cover


def _all_ok(ok: bool, workers: int) -> bool:
    """True when this rank and (under torch.distributed) every other rank succeeded. A peer
    that died or never joined makes the collective raise (process-group timeout): not ok."""
    if workers == 1:
        return ok
    try:
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32)
        if torch.distributed.get_backend() == "nccl":
            flag = flag.cuda()
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
        return bool(flag.item())
    except Exception:  # noqa: BLE001 - a failed collective means some rank did not succeed
        return False


def _convert_steps(src_dir, out_path, rank, grid, block_limit, verify_blocks, curve_dtype, metadata, quant,
                   quant_report, pipeline, worker, workers):
    """The body of ``convert``; yields at its two synchronisation points (see there)."""
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
    try:
        yield  # synchronisation point 1: the output file exists
    except GeneratorExit:  # another rank failed: release the files and stop
        if worker == 0:
            writer.close()
        src.close()
        raise
    if worker != 0:
        writer = OffsetWriter(out_path, manifest, metadata or {"format": "pt"}, create=False)

    need_basis = worker == 0 or any(op.kind == "curve" for op in mine) or verify_blocks

    def build_basis():
        table_, basis_, _curve = curve_mod.build_curve_basis(
            *(src.get(name).float().numpy() for name in mapping.CURVE_SOURCES), rank=rank, grid=grid)
        del _curve
        if worker == 0:
            writer.write("adaln_t_table", to_bytes(torch.from_numpy(table_), "F32"))
        return table_, basis_

    quantizer = None
    if any(op.kind == "quant" for op in mine):
        if quant != "int8_convrot":
            from . import nvfp4
            quantizer = nvfp4.GpuPacker(torch.device("cuda", torch.cuda.current_device()))
        else:
            quantizer = _GpuQuantizer(torch.device("cuda", torch.cuda.current_device()))
    blob = comfy_quant_blob().tobytes()

    piped: list = []
    host_jobs = None
    basis_job = None
    if pipeline and quant == "int8_convrot" and quantizer is not None:
        piped = [op for op in mine if op.kind == "quant" and _Pipeline.accepts(op, src)]
    if pipeline:
        from concurrent.futures import ThreadPoolExecutor
        host_jobs = ThreadPoolExecutor(4, thread_name_prefix="convert-host")
        if need_basis:
            basis_job = host_jobs.submit(build_basis)
    elif need_basis:
        table, basis = build_basis()
    host_futs = []
    piped_ids = {id(op) for op in piped}
    widen = _HostWiden() if pipeline else None

    def host_op(op):
        name = op.out[0]
        raw = _raw_bytes(src, op) if op.kind in ("copy", "concat") else None
        if raw is not None:
            writer.write(name, raw)
        elif op.kind == "copy":
            writer.write(name, to_bytes(_prepare(src.get(op.src[0]), op), op.dtype.upper()))
        elif op.kind == "concat":
            parts = [src.get(s) for s in op.src]
            merged = parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)
            writer.write(name, to_bytes(_prepare(merged, op), op.dtype.upper()))
        elif op.kind == "curve":
            # widen first: only the projection needs the basis (still being built on another thread)
            weight = widen(src, op.src[0]) if widen is not None and widen.accepts(src, op.src[0]) else \
                src.get(op.src[0]).float().numpy()
            basis_ = basis_job.result()[1] if basis_job is not None else basis
            projected = curve_mod.project_weight(weight, basis_)
            writer.write(name, to_bytes(torch.from_numpy(projected), curve_dtype.upper()))
        elif op.kind == "derived":
            from .rope import rope_inv_freq
            writer.write(name, rope_inv_freq().tobytes())
        else:
            raise ValueError(f"unhandled op kind {op.kind!r}")

    # the write phase: on any failure, stop the host jobs and close the file before the failure
    # reaches the next synchronisation point (where the ranks agree that the conversion failed)
    try:
        if host_jobs is not None:
            host_futs = [host_jobs.submit(host_op, op) for op in mine if op.kind != "quant"]
        errors_by_op: dict[int, float] = {}
        if piped:
            piped_errors = _Pipeline(quantizer.device, src, writer, blob, quant_report).run(piped)
            errors_by_op.update((id(op), e) for op, e in zip(piped, piped_errors))
        for op in tqdm(mine, unit="op", desc=f"convert[{worker}/{workers}]", disable=workers > 1 and worker != 0):
            name = op.out[0]
            if id(op) in piped_ids or (host_jobs is not None and op.kind != "quant"):
                continue
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
                    errors_by_op[id(op)] = err
                del parts
            else:
                host_op(op)

        for f in host_futs:
            f.result()
        if basis_job is not None:
            table, basis = basis_job.result()
        if host_jobs is not None:
            host_jobs.shutdown()
        report.quant_errors = [errors_by_op[id(op)] for op in mine if id(op) in errors_by_op]
        expect = {n for op in mine for n in _outputs(op, quant)} | ({"adaln_t_table"} if worker == 0 else set())
        writer.close(expect=expect)
    except BaseException:
        if host_jobs is not None:
            host_jobs.shutdown(wait=True, cancel_futures=True)
        writer.close()
        src.close()
        raise
    src.close()
    yield  # synchronisation point 2: every rank's tensors are written
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
