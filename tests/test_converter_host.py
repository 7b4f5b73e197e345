"""Converter host logic without a GPU: key plan (the reference's tests/test_mapping.py),
safetensors layout (tests/test_io.py), derived tensors (tests/test_rope.py, test_curve.py),
the byte-exact output of every host-side op against the reference's own convert(), and the
multi-process (gloo) per-tensor split."""

import hashlib
import os
import socket
import struct
from pathlib import Path

import numpy as np
import pytest
import torch

import synthetic
from slimdit import curve as curve_mod
from slimdit import mapping
from slimdit.convert import convert, output_manifest, partition
from slimdit.rope import rope_inv_freq
from slimdit.safetensors_io import OffsetWriter, ShardSet, Writer, build_header, read_header, to_bytes


def _official_keys(n_blocks=2):
    return list(synthetic.official_shapes(n_blocks, 512, 1024, 64))


# ------------------------------------------------------------------ mapping
def test_every_source_resolves_and_blocks_are_counted():
    keys = _official_keys(3)
    plan = mapping.build_plan(keys)
    assert mapping.block_count(keys) == 3
    assert mapping.missing_sources(plan, keys) == []


def test_output_names_are_the_ones_the_loader_detects():
    outs = {name for op in mapping.build_plan(_official_keys(1)) for name in op.out}
    for expected in ["blocks.0.attn.qkv_proj.weight", "blocks.0.attn.out_proj.weight", "blocks.0.mlp.fc1.weight",
                     "blocks.0.mlp.fc2.weight", "blocks.0.attn.q_norm.weight", "blocks.0.attn.k_norm.weight",
                     "blocks.0.norm1.weight", "blocks.0.norm2.weight", "blocks.0.adaln_proj.linear.weight",
                     "video_patch_proj.weight", "final_layer.video_out.weight", "final_layer.norm.weight",
                     "final_layer.adaln_proj.linear.weight", "condition_proj.weight",
                     "token_refiner.blocks.0.attn.qkv_proj.weight", "rope.inv_freq"]:
        assert expected in outs, expected


def test_exactly_the_four_block_linears_are_quantised():
    plan = mapping.build_plan(_official_keys(1))
    assert {op.out[0] for op in plan if op.kind == "quant"} == {
        "blocks.0.attn.qkv_proj.weight", "blocks.0.attn.out_proj.weight", "blocks.0.mlp.fc1.weight",
        "blocks.0.mlp.fc2.weight"}
    assert {op.out[0] for op in plan if op.kind == "curve"} == {
        "blocks.0.adaln_proj.linear.weight", "final_layer.adaln_proj.linear.weight"}
    fc1 = next(op for op in plan if op.out[0] == "blocks.0.mlp.fc1.weight")
    assert fc1.swap_halves
    qkv = next(op for op in plan if op.out[0] == "blocks.0.attn.qkv_proj.weight")
    assert qkv.src == ("transformer_blocks.0.attn.to_q.weight", "transformer_blocks.0.attn.to_k.weight",
                       "transformer_blocks.0.attn.to_v.weight")


def test_plan_rejects_non_transformer_keys():
    with pytest.raises(ValueError):
        mapping.build_plan(["foo.weight"])


# ------------------------------------------------------------------ safetensors layout
def test_round_trip_preserves_names_dtypes_and_values(tmp_path):
    manifest = [("adaln_t_table", "F32", (5, 2)), ("blocks.0.attn.qkv_proj.weight", "I8", (4, 8)),
                ("blocks.0.attn.qkv_proj.weight_scale", "F32", (4, 1)), ("blocks.0.attn.qkv_proj.comfy_quant", "U8", (72,)),
                ("blocks.0.norm1.weight", "BF16", (6,)), ("blocks.0.adaln_proj.linear.weight", "F16", (4, 2))]
    payloads = {
        "adaln_t_table": np.arange(10, dtype=np.float32).reshape(5, 2),
        "blocks.0.attn.qkv_proj.weight": np.arange(32, dtype=np.int8).reshape(4, 8),
        "blocks.0.attn.qkv_proj.weight_scale": np.full((4, 1), 0.25, dtype=np.float32),
        "blocks.0.attn.qkv_proj.comfy_quant": np.zeros(72, dtype=np.uint8),
        "blocks.0.norm1.weight": np.linspace(-1, 1, 6, dtype=np.float32),
        "blocks.0.adaln_proj.linear.weight": np.linspace(-0.5, 0.5, 8, dtype=np.float32).reshape(4, 2),
    }
    w = Writer(tmp_path / "a.safetensors", manifest, metadata={"format": "pt"})
    for name, dtype, _ in manifest:
        w.append(name, to_bytes(torch.from_numpy(payloads[name]), dtype))
    w.close()
    # the positional writer, in reverse order, produces the same bytes
    ow = OffsetWriter(tmp_path / "b.safetensors", manifest, metadata={"format": "pt"})
    for name, dtype, _ in reversed(manifest):
        ow.write(name, to_bytes(torch.from_numpy(payloads[name]), dtype))
    ow.close(expect={n for n, _, _ in manifest})
    assert (tmp_path / "a.safetensors").read_bytes() == (tmp_path / "b.safetensors").read_bytes()
    reader = ShardSet(tmp_path / "a.safetensors")
    assert dict(reader.manifest) == {n: (d, s) for n, d, s in manifest}
    assert np.array_equal(reader.get("blocks.0.attn.qkv_proj.weight").numpy(), payloads["blocks.0.attn.qkv_proj.weight"])
    assert reader.get("blocks.0.norm1.weight").dtype == torch.bfloat16


def test_writers_reject_bad_writes(tmp_path):
    manifest = [("a", "F32", (1,)), ("b", "F32", (1,))]
    w = Writer(tmp_path / "x.safetensors", manifest)
    with pytest.raises(RuntimeError):
        w.append("b", b"\x00\x00\x00\x00")
    w.abort()
    ow = OffsetWriter(tmp_path / "y.safetensors", manifest)
    with pytest.raises(RuntimeError):
        ow.write("a", b"\x00\x00")
    ow.write("a", b"\x00" * 4)
    with pytest.raises(RuntimeError):
        ow.close(expect={"a", "b"})
    w2 = Writer(tmp_path / "z.safetensors", manifest)
    w2.append("a", b"\x00" * 4)
    with pytest.raises(RuntimeError):
        w2.close()


def test_header_is_compact_json_with_metadata_first():
    raw = build_header([("x", "F32", (2, 3))], {"format": "pt"})
    (n,) = struct.unpack("<Q", raw[:8])
    assert raw[8:8 + n] == b'{"__metadata__":{"format":"pt"},"x":{"dtype":"F32","shape":[2,3],"data_offsets":[0,24]}}'


# ------------------------------------------------------------------ derived tensors
ROPE_REFERENCE = np.array([1.0, 0.5623413324356079, 0.3162277638912201, 0.17782793939113617, 0.10000000149011612,
                           0.05623412877321243, 0.03162277862429619, 0.017782794311642647, 0.009999999776482582,
                           0.005623413249850273, 0.003162277862429619, 0.0017782794311642647, 0.0010000000474974513,
                           0.000562341301701963, 0.0003162277862429619, 0.00017782794020604342], dtype=np.float32)


def test_rope_matches_the_table_the_runtime_checkpoint_ships():
    values = rope_inv_freq()
    assert values.dtype == np.float32 and np.array_equal(values, ROPE_REFERENCE)


def test_time_embedding_shape_and_curve_basis():
    rng = np.random.default_rng(0)
    w1 = rng.standard_normal((16, 256)).astype(np.float32)
    w2 = rng.standard_normal((8, 16)).astype(np.float32)
    t = np.linspace(0.0, 1.0, 33, dtype=np.float32)
    out = curve_mod.time_embeddings(t, w1, np.zeros(16, np.float32), w2, np.zeros(8, np.float32))
    assert out.shape == (33, 8) and np.isfinite(out).all() and not np.allclose(out[0], out[-1])
    table, basis, crv = curve_mod.build_curve_basis(w1, np.zeros(16, np.float32), w2, np.zeros(8, np.float32),
                                                    rank=4, grid=33)
    assert table.shape == (33, 4) and basis.shape == (8, 4) and crv.shape == (33, 8)


# ------------------------------------------------------------------ partition
def test_partition_is_deterministic_balanced_and_total():
    costs = [100, 90, 80, 10, 10, 10, 5, 1]
    for workers in (1, 2, 3, 8):
        owner = partition(costs, workers)
        assert owner == partition(costs, workers)
        assert len(owner) == len(costs) and set(owner) <= set(range(workers))
        loads = [sum(c for c, o in zip(costs, owner) if o == w) for w in range(workers)]
        assert max(loads) - min(loads) <= max(costs)


# ------------------------------------------------------------------ byte parity vs the reference
@pytest.fixture(scope="module")
def official_dir(tmp_path_factory, golden_meta):
    case = golden_meta["convert"]["case"]
    d = synthetic.official_checkpoint(tmp_path_factory.mktemp("official"), **case)
    for p in sorted(d.glob("*.safetensors")):
        assert hashlib.sha256(p.read_bytes()).hexdigest() == golden_meta["convert"]["src_sha256"][p.name]
    return d


def test_manifest_and_header_equal_the_reference_header(official_dir, golden_meta):
    src = ShardSet(official_dir)
    ops = mapping.build_plan(src.manifest.keys())
    manifest = output_manifest(ops, src, rank=8, grid=65, block_limit=None)
    raw = build_header(manifest, {"format": "pt"})
    assert raw[8:].decode("utf-8") == golden_meta["convert"]["header"]


def test_host_side_tensors_byte_identical_to_reference_convert(official_dir, golden_meta, tmp_path):
    out = tmp_path / "block0.safetensors"
    convert(official_dir, out, rank=8, grid=65, block_limit=0)
    assert hashlib.sha256(out.read_bytes()).hexdigest() == golden_meta["convert_block0"]["sha256_file"]
    assert read_header(out)["__metadata__"] == {"format": "pt"}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, src, out, result_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        convert(src, out, rank=8, grid=65, block_limit=0)
        Path(result_dir, f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_multi_process_split_writes_the_same_bytes(official_dir, golden_meta, tmp_path, world):
    """Per-tensor partition over `world` gloo ranks, each writing its tensors at their offsets."""
    import torch.multiprocessing as mp
    out = tmp_path / "split.safetensors"
    mp.start_processes(_worker, args=(world, _free_port(), str(official_dir), str(out), str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    assert all((tmp_path / f"ok{r}").exists() for r in range(world))
    assert hashlib.sha256(out.read_bytes()).hexdigest() == golden_meta["convert_block0"]["sha256_file"]


def _failing_worker(rank, world, port, src, out, result_dir, mode):
    """Rank 1 fails: "raise" makes its writes raise inside its share of the work; "absent" makes
    it leave right after joining the process group, never entering the conversion."""
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=10))
    outcome = "ok"
    try:
        if rank == 1 and mode == "absent":
            outcome = "absent"
            return
        if rank == 1 and mode == "raise":
            def broken_write(self, name, payload):
                raise RuntimeError("injected write failure")
            OffsetWriter.write = broken_write
        convert(src, out, rank=8, grid=65, block_limit=0)
    except BaseException as exc:  # noqa: BLE001 - the outcome is what the test checks
        outcome = f"{type(exc).__name__}: {exc}"
    finally:
        Path(result_dir, f"rank{rank}.txt").write_text(outcome)
        if not (rank == 1 and mode == "absent"):
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


@pytest.mark.parametrize("mode", ["raise", "absent"])
def test_a_failing_rank_fails_every_rank_and_removes_the_partial_output(official_dir, tmp_path, mode):
    """Failure detection across ranks: every rank that reaches a synchronisation point learns of
    the failure (rank 0 from the all-reduce of the ranks' success flags, or from the collective
    erroring when a rank is gone), raises, and the pre-sized output file is removed."""
    import time

    import torch.multiprocessing as mp
    out = tmp_path / "split.safetensors"
    t0 = time.time()
    mp.start_processes(_failing_worker, args=(2, _free_port(), str(official_dir), str(out), str(tmp_path), mode),
                       nprocs=2, join=True, start_method="spawn")
    assert time.time() - t0 < 120
    r0 = (tmp_path / "rank0.txt").read_text()
    r1 = (tmp_path / "rank1.txt").read_text()
    assert r0 != "ok" and "RuntimeError" in r0, r0
    if mode == "raise":
        assert "another rank" in r0 and "injected write failure" in r1, (r0, r1)
    else:
        assert r1 == "absent"
    assert not out.exists()


def test_byte_level_copies_equal_the_torch_path(tmp_path):
    """Copy/concat ops assembled from the stored bytes (positional reads, half swaps, exact
    bf16 -> f32 widening) give the bytes of the torch cast path the reference uses."""
    import torch

    import synthetic
    from slimdit import mapping
    from slimdit.convert import _prepare, _raw_bytes
    from slimdit.safetensors_io import ShardSet, to_bytes

    src = ShardSet(synthetic.official_checkpoint(tmp_path / "official", n_blocks=2))
    checked = 0
    for op in mapping.build_plan(src.manifest.keys()):
        if op.kind not in ("copy", "concat"):
            continue
        raw = _raw_bytes(src, op)
        if raw is None:
            continue
        parts = [src.get(s) for s in op.src]
        merged = parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)
        assert bytes(memoryview(raw).cast("B")) == to_bytes(_prepare(merged, op), op.dtype.upper()), op.out
        checked += 1
    src.close()
    assert checked >= 20


@pytest.mark.parametrize("pipeline", [True, False])
def test_a_failing_host_job_closes_the_files_and_removes_the_output(official_dir, tmp_path, monkeypatch, pipeline):
    """A host-side op that raises during the write phase (here the curve projection): the
    conversion raises that error, the host threads are stopped, no file descriptor is left open
    and the pre-sized partial output is removed."""
    def fail(*args, **kwargs):
        raise RuntimeError("injected projection failure")

    monkeypatch.setattr(curve_mod, "project_weight", fail)
    out = tmp_path / "failed.safetensors"
    fds_before = len(os.listdir("/proc/self/fd"))
    with pytest.raises(RuntimeError, match="injected projection failure"):
        convert(official_dir, out, rank=8, grid=65, block_limit=0, pipeline=pipeline)
    assert not out.exists()
    assert len(os.listdir("/proc/self/fd")) <= fds_before
