"""Multi-GPU paths on 2 GPUs of one node (skipped when fewer are visible).

* output-column split (slimdit/colsplit.py): each rank computes its column block with the
  CUDA linear and NCCL all-gathers them, or (PeerColumnSplit) its GEMM epilogue stores the
  tiles into every rank's output over NVLink; either way the result must equal, bit for bit,
  the single-GPU linear on the full weight computed on the same rank;
* attention with the heads split over the ranks (slimdit.attention.attention_heads) equals the
  single-GPU attention of those heads (the V amax all-reduced).
"""

import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import datetime

    import torch.distributed as dist

    import synthetic
    from slimdit import _native, colsplit, ops
    from slimdit.int8 import quantize_convrot_weight
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        m, n, k = 1000, 1536, 5120
        x = torch.from_numpy(synthetic.activations(m, k, seed=31)).to(dev).to(torch.bfloat16)
        qw, sw = quantize_convrot_weight(synthetic.weight(n, k, seed=32))
        qw, sw = torch.from_numpy(qw).to(dev), torch.from_numpy(sw).to(dev)
        bias = torch.from_numpy(np.random.default_rng(33).standard_normal(n).astype(np.float32) * 0.02)
        bias = bias.to(dev).to(torch.bfloat16)
        full = ops.int8_linear(x, qw, sw, bias=bias)
        q_s, s_s, b_s = colsplit.shard_weight(qw, sw, bias, rank, world)
        rows = colsplit.int8_linear_colsplit(x, q_s, s_s, b_s, layout="rows")
        blocks = colsplit.int8_linear_colsplit(x, q_s, s_s, b_s, layout="blocks")
        torch.cuda.synchronize(dev)
        assert torch.equal(rows, full)
        for g in range(world):
            assert torch.equal(blocks[g], full[:, g * n // world:(g + 1) * n // world])
        # the all-gather inside the GEMM epilogue (peer stores over NVLink)
        for mode in ("dma", "stores"):
            for layout in ("rows", "blocks"):
                fused = colsplit.PeerColumnSplit(m, n, k, device=dev, mode=mode, chunk_rows=384, layout=layout)
                try:
                    for mm in (m, m, 37):  # the buffer is reused; then a short batch
                        y = fused(x[:mm], q_s, s_s, b_s)
                        torch.cuda.synchronize(dev)
                        if layout == "rows":
                            assert torch.equal(y, full[:mm]), (mode, layout)
                        else:
                            for g in range(world):
                                assert torch.equal(y[g], full[:mm, g * n // world:(g + 1) * n // world]), (mode, layout)
                finally:
                    fused.close()
        # attention with the heads split over the ranks: the V amax is all-reduced, so each rank's
        # heads equal the single-GPU result bit for bit
        from slimdit import attention
        seq, heads = 700, 4
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        qkv = (torch.randn((seq, 3 * heads * 128), generator=g, device=dev) * 0.5).to(torch.bfloat16)
        qkv[:, 2 * heads * 128 + 3] *= 4.0  # the largest |v| sits in head 0: rank 1 needs the all-reduced amax
        dist.broadcast(qkv, src=0)          # every rank attends over the same buffer
        whole = attention.attention_packed(qkv, heads)
        mine = attention.attention_heads(qkv, heads, rank, world)
        torch.cuda.synchronize(dev)
        hl = heads // world
        assert torch.equal(mine, whole[:, rank * hl * 128:(rank + 1) * hl * 128])
        assert _native.device_error() == 0
        Path(result_dir, f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_column_split_two_gpus_bit_identical(tmp_path):
    import torch.multiprocessing as mp
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
