"""Output-column split of the convrot linear over the GPUs of one node.

Each rank holds N/G consecutive rows of the weight (output channels), computes its column
block of y = x @ W^T on its own GPU with the single-GPU linear, and the blocks are
all-gathered over NVLink (NCCL): the only collective of the path. Token rows of x are
replicated. Because rotation and quantisation are per token and every output column depends
only on its own weight row, the gathered result is identical, bit for bit, to the
single-GPU linear on the full weight.

Layouts of the gathered output:
  "blocks"  [G, M, N/G] as NCCL writes it (no extra pass; block g holds columns
            [g*N/G, (g+1)*N/G)),
  "rows"    [M, N] row-major (one extra device copy).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of an N-row weight owned by `rank` (equal shards, multiples of 8)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n % (8 * world):
        raise ValueError(f"out_features {n} must split into {world} shards that are multiples of 8")
    step = n // world
    return rank * step, (rank + 1) * step


def shard_weight(qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None, rank: int, world: int):
    """This rank's rows of (qweight [N, K], wscales [N(,1)], bias [N])."""
    lo, hi = shard_bounds(qweight.shape[0], world, rank)
    ws = wscales.reshape(-1)[lo:hi]
    return qweight[lo:hi].contiguous(), ws.contiguous(), (None if bias is None else bias[lo:hi].contiguous())


def gather_columns(y_local: torch.Tensor, group=None, layout: str = "rows") -> torch.Tensor:
    """All-gather the ranks' [M, N/G] column blocks -> [M, N] ("rows") or [G, M, N/G] ("blocks")."""
    if layout not in ("rows", "blocks"):
        raise ValueError("layout must be 'rows' or 'blocks'")
    world = dist.get_world_size(group)
    m, nl = y_local.shape
    blocks = torch.empty((world * m, nl), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(blocks, y_local.contiguous(), group=group)
    blocks = blocks.view(world, m, nl)
    if layout == "blocks":
        return blocks
    return blocks.permute(1, 0, 2).reshape(m, world * nl)


def int8_linear_colsplit(x: torch.Tensor, qweight_shard: torch.Tensor, wscales_shard: torch.Tensor,
                         bias_shard: torch.Tensor | None = None, group=None, layout: str = "rows",
                         convrot_groupsize: int = 256) -> torch.Tensor:
    """Convrot linear with the output columns split over the process group.

    x: [..., K] (same on every rank); qweight_shard/wscales_shard/bias_shard: this rank's
    rows from :func:`shard_weight`. Returns the full output on every rank.
    """
    from . import ops

    lead = x.shape[:-1]
    y = ops.int8_linear(x.reshape(-1, x.shape[-1]), qweight_shard, wscales_shard,
                        convrot_groupsize=convrot_groupsize, bias=bias_shard)
    full = gather_columns(y, group=group, layout=layout)
    return full.reshape(*lead, -1) if layout == "rows" else full
