"""Output-column split (slimdit/colsplit.py): shard bounds, and the two-rank gather over a
gloo process group on CPU. The per-rank linear is the oracle's CPU restatement (codes from
the oracle, exact int32 GEMM, fp32 dequant, bf16), standing in for the CUDA linear, so the
test checks the sharding and the gathered layouts; the 2-GPU test of the CUDA path is in
tests/test_gpu_multi.py."""

import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch

from slimdit import colsplit


def test_shard_bounds():
    assert colsplit.shard_bounds(15360, 8, 0) == (0, 1920)
    assert colsplit.shard_bounds(15360, 8, 7) == (13440, 15360)
    assert colsplit.shard_bounds(512, 1, 0) == (0, 512)
    with pytest.raises(ValueError):
        colsplit.shard_bounds(100, 2, 0)       # shards must be multiples of 8
    with pytest.raises(ValueError):
        colsplit.shard_bounds(512, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_linear(x, qweight, wscales, convrot_groupsize=256, bias=None):
    import oracle
    qx, sx = oracle.quantize_activations(x.float().numpy())
    acc = oracle.int8_gemm_i32(qx, qweight.numpy())
    y = acc.astype(np.float32) * (sx.reshape(-1, 1) * wscales.numpy().reshape(1, -1))
    if bias is not None:
        y = y + bias.float().numpy().reshape(1, -1)
    return torch.from_numpy(y.astype(np.float32)).to(torch.bfloat16)


def _worker(rank, world, port, result_dir):
    import torch.distributed as dist

    import synthetic
    from slimdit import colsplit as cs
    from slimdit import ops
    ops.int8_linear = _cpu_linear   # CPU stand-in for the CUDA linear (this process only)
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        x = torch.from_numpy(synthetic.activations(24, 512, seed=5))
        rng = np.random.default_rng(6)
        qw = torch.from_numpy(rng.integers(-127, 128, size=(64, 512), dtype=np.int8))
        sw = torch.from_numpy((rng.random(64, dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32))
        bias = torch.from_numpy(rng.standard_normal(64).astype(np.float32) * 0.02).to(torch.bfloat16)
        full = _cpu_linear(x, qw, sw, bias=bias)
        q_s, s_s, b_s = cs.shard_weight(qw, sw, bias, rank, world)
        rows = cs.int8_linear_colsplit(x, q_s, s_s, b_s, layout="rows")
        blocks = cs.int8_linear_colsplit(x, q_s, s_s, b_s, layout="blocks")
        assert torch.equal(rows, full)
        assert blocks.shape == (world, 24, 64 // world)
        for g in range(world):
            assert torch.equal(blocks[g], full[:, g * 64 // world:(g + 1) * 64 // world])
        x3 = x.reshape(2, 12, 512)
        assert torch.equal(cs.int8_linear_colsplit(x3, q_s, s_s, b_s).reshape(24, 64), full)
        Path(result_dir, f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_matches_full_linear(tmp_path):
    import torch.multiprocessing as mp
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
