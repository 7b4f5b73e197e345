"""Streaming safetensors writer and memory-mapped shard reader.

The output file is byte-compatible with the reference's slimdit/safetensors_io.py:35-132:
an 8-byte little-endian header length, the compact JSON header (``separators=(",", ":")``,
``__metadata__`` first, then the tensors in manifest order with contiguous
``data_offsets``), then the tensor bytes in that order.

``Writer`` keeps the reference's API (header first, ``append`` in manifest order,
``close`` checks completeness, ``abort`` closes without the check). ``OffsetWriter`` is the
parallel form: since every offset is known from the header, tensors can be written in any
order — by several threads or several processes (one per GPU) into one pre-sized file.
"""

from __future__ import annotations

import json
import os
import struct
from functools import reduce
from operator import mul
from pathlib import Path

import torch
from safetensors import safe_open

DTYPE_SIZE = {"F32": 4, "F16": 2, "BF16": 2, "I8": 1, "U8": 1}
TORCH_TO_ST = {
    torch.float32: "F32",
    torch.float16: "F16",
    torch.bfloat16: "BF16",
    torch.int8: "I8",
    torch.uint8: "U8",
}
_ST_TO_TORCH = {v: k for k, v in TORCH_TO_ST.items()}


def numel(shape) -> int:
    return reduce(mul, shape, 1)


def tensor_nbytes(dtype: str, shape) -> int:
    if dtype not in DTYPE_SIZE:
        raise ValueError(f"unsupported storage dtype {dtype!r}")
    return DTYPE_SIZE[dtype] * numel(shape)


def layout(manifest) -> dict[str, tuple[int, int]]:
    """name -> (start, end) byte offsets inside the data section."""
    out: dict[str, tuple[int, int]] = {}
    pos = 0
    for name, dtype, shape in manifest:
        n = tensor_nbytes(dtype, shape)
        out[name] = (pos, pos + n)
        pos += n
    return out


def build_header(manifest: list[tuple[str, str, tuple[int, ...]]], metadata: dict | None) -> bytes:
    """Serialized header for the ordered manifest: ``<u64 length><compact JSON>``."""
    offsets = {}
    pos = 0
    for name, dtype, shape in manifest:
        if dtype not in DTYPE_SIZE:
            raise ValueError(f"unsupported storage dtype {dtype!r} for {name}")
        n = DTYPE_SIZE[dtype] * numel(shape)
        offsets[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [pos, pos + n]}
        pos += n
    doc: dict = {}
    if metadata:
        doc["__metadata__"] = metadata
    doc.update(offsets)
    raw = json.dumps(doc, separators=(",", ":")).encode("utf-8")
    return struct.pack("<Q", len(raw)) + raw


def to_bytes(tensor: torch.Tensor, dtype: str) -> bytes:
    """Cast ``tensor`` to the storage dtype and return its little-endian bytes."""
    target = _ST_TO_TORCH.get(dtype)
    if target is None:
        raise ValueError(f"unsupported storage dtype {dtype!r}")
    out = tensor.to(target)
    if out.dtype == torch.bfloat16:
        return out.contiguous().view(torch.uint16).numpy().tobytes()
    return out.contiguous().numpy().tobytes()


class Writer:
    """Header first, then tensors in manifest order (the reference's streaming writer)."""

    def __init__(self, path: str | Path, manifest: list[tuple[str, str, tuple[int, ...]]], metadata: dict | None = None):
        self.path = Path(path)
        self.manifest = manifest
        self._expected = [name for name, _, _ in manifest]
        self._written: list[str] = []
        self._fh = self.path.open("wb")
        self._fh.write(build_header(manifest, metadata))

    def append(self, name: str, payload: bytes) -> None:
        expected = self._expected[len(self._written)]
        if name != expected:
            raise RuntimeError(f"out-of-order write: expected {expected!r}, got {name!r}")
        self._fh.write(payload)
        self._written.append(name)

    def close(self) -> None:
        if len(self._written) != len(self._expected):
            missing = self._expected[len(self._written):][:4]
            self._fh.close()
            raise RuntimeError(f"incomplete write: {len(self._written)}/{len(self._expected)} tensors ({missing}...)")
        self._fh.close()

    def abort(self) -> None:
        """Close without the completeness check (error path; the partial file is unusable)."""
        self._fh.close()


class OffsetWriter:
    """Positional writer: any tensor, any order, any number of writers on one file.

    ``create=True`` writes the header and sizes the file (do it once, e.g. on rank 0, before
    the other writers open it with ``create=False``).
    """

    def __init__(self, path: str | Path, manifest, metadata: dict | None = None, create: bool = True):
        self.path = Path(path)
        self.manifest = manifest
        header = build_header(manifest, metadata)
        self.data_start = len(header)
        self.offsets = layout(manifest)
        total = self.data_start + (max((e for _, e in self.offsets.values()), default=0))
        if create:
            with self.path.open("wb") as fh:
                fh.write(header)
                fh.truncate(total)
        self._fd = os.open(self.path, os.O_RDWR)
        self.written: set[str] = set()

    def write(self, name: str, payload) -> None:
        start, end = self.offsets[name]
        view = memoryview(payload).cast("B")
        if len(view) != end - start:
            raise RuntimeError(f"{name}: payload of {len(view)} bytes, layout expects {end - start}")
        done = 0
        while done < len(view):
            done += os.pwrite(self._fd, view[done:], self.data_start + start + done)
        self.written.add(name)

    def close(self, expect: set[str] | None = None) -> None:
        """Close the file (a second call only repeats the completeness check)."""
        if self._fd >= 0:
            os.close(self._fd)
            self._fd = -1
        if expect is not None and not expect <= self.written:
            missing = sorted(expect - self.written)[:4]
            raise RuntimeError(f"incomplete write: missing {missing}...")


def read_header(path: str | Path) -> dict:
    with open(path, "rb") as fh:
        (n,) = struct.unpack("<Q", fh.read(8))
        return json.loads(fh.read(n))


class ShardSet:
    """The official shards, memory-mapped, keyed by tensor name."""

    def __init__(self, directory: str | Path):
        source = Path(directory)
        self.directory = source if source.is_dir() else source.parent
        self._readers: dict[str, object] = {}
        self.manifest: dict[str, tuple[str, tuple[int, ...]]] = {}
        self.index: dict[str, str] = {}
        shards = [source] if source.is_file() else sorted(source.glob("*.safetensors"))
        self._paths: dict[str, Path] = {}
        self._fds: dict[str, int] = {}
        self._raw: dict[str, tuple[int, int]] = {}  # name -> (absolute byte offset in its shard, bytes)
        for shard in shards:
            reader = safe_open(str(shard), framework="pt", device="cpu")
            self._readers[shard.name] = reader
            self._paths[shard.name] = shard
            with shard.open("rb") as fh:
                (hlen,) = struct.unpack("<Q", fh.read(8))
                header = json.loads(fh.read(hlen))
            data_start = 8 + hlen
            for key, meta in header.items():
                if key != "__metadata__":
                    b0, b1 = meta["data_offsets"]
                    self._raw[key] = (data_start + b0, b1 - b0)
            for key in reader.keys():
                sl = reader.get_slice(key)
                raw = sl.get_dtype()
                stored = raw if isinstance(raw, str) else TORCH_TO_ST[raw]
                if stored not in DTYPE_SIZE:
                    raise ValueError(f"unsupported on-disk dtype {stored!r} for {key}")
                self.manifest[key] = (stored, tuple(sl.get_shape()))
                self.index[key] = shard.name

    def get(self, name: str) -> torch.Tensor:
        return self._readers[self.index[name]].get_tensor(name)

    def nbytes(self, name: str) -> int:
        dtype, shape = self.manifest[name]
        return tensor_nbytes(dtype, shape)

    def read_into(self, name: str, out, offset: int = 0) -> int:
        """Copy the tensor's stored bytes into the writable byte buffer ``out`` (e.g. a pinned
        uint8 tensor's numpy view) at ``offset`` with positional reads; returns the byte count.
        Thread-safe: no shared file position."""
        start, n = self._raw[name]
        shard = self.index[name]
        fd = self._fds.get(shard)
        if fd is None:
            fd = self._fds.setdefault(shard, os.open(self._paths[shard], os.O_RDONLY))
        view = memoryview(out).cast("B")[offset:offset + n]
        if len(view) != n:
            raise ValueError(f"{name}: buffer too small ({len(view)} of {n} bytes)")
        done = 0
        while done < n:
            got = os.preadv(fd, [view[done:]], start + done)
            if got <= 0:
                raise OSError(f"{name}: short read at byte {done} of {n}")
            done += got
        return n

    def close(self) -> None:
        for fd in self._fds.values():
            os.close(fd)
        self._fds.clear()


__all__ = ["DTYPE_SIZE", "TORCH_TO_ST", "OffsetWriter", "ShardSet", "Writer", "build_header", "layout", "numel",
           "read_header", "tensor_nbytes", "to_bytes"]

