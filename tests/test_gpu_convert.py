"""Whole-checkpoint conversion on the GPU, byte-identical to the reference's convert().

Synthetic 2-block official checkpoint (tests/synthetic.py, hidden 512, FFN 1024, seeded
N(0, 0.02) weights with outlier channels), converted with rank 8 / grid 65: the output file's
SHA-256 must equal the one the reference's slimdit.convert.convert wrote for the same shards
(tests/golden/golden.json). Also split over two processes sharing cuda:0 (the split's
kernels never wait on each other) and through the command-line entry point.
"""

import hashlib
import os
import socket
from pathlib import Path

import pytest

import synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def official_dir(tmp_path_factory, golden_meta):
    case = golden_meta["convert"]["case"]
    d = synthetic.official_checkpoint(tmp_path_factory.mktemp("official_gpu"), **case)
    for p in sorted(d.glob("*.safetensors")):
        assert hashlib.sha256(p.read_bytes()).hexdigest() == golden_meta["convert"]["src_sha256"][p.name]
    return d


def test_full_conversion_byte_identical_to_reference(cuda, official_dir, golden_meta, tmp_path):
    from slimdit import _native
    from slimdit.convert import convert
    out = tmp_path / "converted.safetensors"
    report = convert(official_dir, out, rank=8, grid=65)
    raw = out.read_bytes()
    assert len(raw) == golden_meta["convert"]["size"]
    assert hashlib.sha256(raw).hexdigest() == golden_meta["convert"]["sha256_file"]
    # the error report (computed on the device) tracks the reference's float32 numpy one
    ref_err = golden_meta["convert"]["quant_errors"]
    assert len(report.quant_errors) == len(ref_err)
    for a, b in zip(report.quant_errors, ref_err):
        assert abs(a - b) <= 1e-3 * b
    assert _native.device_error() == 0


def test_sequential_path_byte_identical(cuda, official_dir, golden_meta, tmp_path):
    """pipeline=False (ops one at a time) writes the same file as the pipelined default."""
    from slimdit.convert import convert
    out = tmp_path / "sequential.safetensors"
    report = convert(official_dir, out, rank=8, grid=65, pipeline=False)
    assert hashlib.sha256(out.read_bytes()).hexdigest() == golden_meta["convert"]["sha256_file"]
    assert len(report.quant_errors) == len(golden_meta["convert"]["quant_errors"])


def test_cli_entry_point(cuda, official_dir, golden_meta, tmp_path):
    from slimdit.convert import main
    out = tmp_path / "cli.safetensors"
    assert main(["--src", str(official_dir), "--out", str(out), "--grid", "65"]) == 0
    assert hashlib.sha256(out.read_bytes()).hexdigest() == golden_meta["convert"]["sha256_file"]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, src, out, result_dir):
    import torch
    import torch.distributed as dist
    from slimdit.convert import convert
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        convert(src, out, rank=8, grid=65)
        Path(result_dir, f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


def test_two_process_split_byte_identical(cuda, official_dir, golden_meta, tmp_path):
    import torch.multiprocessing as mp
    out = tmp_path / "split.safetensors"
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.start_processes(_worker, args=(2, _free_port(), str(official_dir), str(out), str(tmp_path)),
                       nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
    assert hashlib.sha256(out.read_bytes()).hexdigest() == golden_meta["convert"]["sha256_file"]
