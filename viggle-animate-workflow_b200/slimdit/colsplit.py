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


class _DeviceArray:
    """Zero-copy view of library-owned device memory for torch.as_tensor (CUDA array interface)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "strides": None, "version": 3}


class PeerColumnSplit:
    """Column-split linear whose all-gather overlaps the GEMM over NVLink, writing straight
    into every rank's output buffer (mapped into each process with CUDA IPC):

      mode="dma"     the token rows are processed in chunks; each chunk's GEMM writes this
                     rank's column block into the local output, and the copy engines push the
                     finished chunk to every peer (one stream per peer) while the next chunk
                     computes;
      mode="stores"  the GEMM epilogue itself stores every tile into all ranks' outputs.

    layout="rows" gives the [M, N] output (a pushed chunk is a 2-D copy of rows of N/G
    columns); layout="blocks" gives [G, M, N/G] as NCCL's all-gather does (block g holds
    columns [g*N/G, (g+1)*N/G); a pushed chunk is one contiguous copy).

    One instance per process (rank), created collectively; it owns the [m_max, n_full] bf16
    output buffer this rank exposes to its peers (allocated by the library with a CUDA IPC
    handle; plain peer mappings, no multicast object). A call synchronises the ranks twice with a
    one-element NCCL all-reduce on the current stream: before the GEMM (every rank has
    finished with the previous result) and after it (every rank's stores have landed). The
    returned tensor is this rank's full output, valid until the next call.
    """

    def __init__(self, m_max: int, n_full: int, k: int, device=None, group=None, mode: str = "dma",
                 chunk_rows: int = 4096, layout: str = "rows"):
        import ctypes

        from . import _native as nat

        self._ct = ctypes
        self._nat = nat
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (GPUs of one node)")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if mode not in ("dma", "stores"):
            raise ValueError("mode must be 'dma' or 'stores'")
        if layout not in ("rows", "blocks"):
            raise ValueError("layout must be 'rows' or 'blocks'")
        if n_full % (8 * self.world):
            raise ValueError(f"n_full {n_full} must split into {self.world} shards that are multiples of 8")
        self.mode, self.chunk_rows, self.layout = mode, max(1, chunk_rows), layout
        self.m_max, self.n_full, self.k = m_max, n_full, k
        self._copy_streams = [torch.cuda.Stream(device=self.device) for _ in range(max(0, self.world - 1))]
        self.lib = nat.load()
        self._own = None
        self._opened = []
        handle = ctypes.create_string_buffer(64)
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            nat.check(self.lib.slim_peer_buffer_alloc(m_max * n_full * 2, ctypes.byref(own), handle))
        self._own = own.value
        self.buf = torch.as_tensor(_DeviceArray(self._own, (m_max, n_full), "<i2"), device=self.device)
        self.buf = self.buf.view(torch.bfloat16)
        infos = [None] * self.world
        dist.all_gather_object(infos, (self.rank, handle.raw), group=group)
        self.ptrs = [0] * self.world
        with torch.cuda.device(self.device):
            for r, h in infos:
                if r == self.rank:
                    self.ptrs[r] = self._own
                    continue
                p = ctypes.c_void_p()
                nat.check(self.lib.slim_peer_open(h, 0, ctypes.byref(p)))
                self.ptrs[r] = p.value
                self._opened.append((p.value, 0))
        self.xq = torch.empty((m_max, k), dtype=torch.int8, device=self.device)
        self.sx = torch.empty((m_max,), dtype=torch.float32, device=self.device)
        self._flag = torch.zeros((1,), dtype=torch.float32, device=self.device)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it before
        tearing down; tensors returned by earlier calls are invalid afterwards)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p, off in self._opened:
                self._nat.check(self.lib.slim_peer_close(p, off))
            self._opened = []
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)  # every peer has unmapped this rank's buffer
            if self._own is not None:
                self.buf = None
                self._nat.check(self.lib.slim_peer_buffer_free(self._own))
                self._own = None

    def __call__(self, x: torch.Tensor, qweight_shard: torch.Tensor, wscales_shard: torch.Tensor,
                 bias_shard: torch.Tensor | None = None, epilogue: str | None = None) -> torch.Tensor:
        from . import ops

        nat = self._nat
        if x.dim() != 2 or x.shape[0] > self.m_max or x.shape[1] != self.k:
            raise ValueError(f"x must be [<= {self.m_max}, {self.k}], got {tuple(x.shape)}")
        if x.dtype not in ops._DT or not x.is_cuda:
            raise TypeError("x must be a bf16/f16/f32 CUDA tensor")
        m = x.shape[0]
        nl = qweight_shard.shape[0]
        if nl * self.world != self.n_full:
            raise ValueError(f"shard of {nl} rows x {self.world} ranks != {self.n_full} output features")
        x = x.contiguous()
        sw = ops._vec(wscales_shard, nl, torch.float32, self.device, "wscales_shard")
        b = ops._vec(bias_shard, nl, torch.bfloat16, self.device, "bias_shard")
        if self.layout == "rows":
            base, ldo = self.rank * nl * 2, self.n_full  # this rank's columns inside [M, N]
        else:
            base, ldo = self.rank * self.m_max * nl * 2, nl  # this rank's block of [G, M, N/G]
        pitch = ldo * 2
        peers = [r for r in range(self.world) if r != self.rank]
        cur = torch.cuda.current_stream(self.device)
        dist.all_reduce(self._flag, group=self.group)  # every rank is done with the previous result
        with torch.cuda.device(self.device):
            if self.mode == "stores":
                outs = [self.ptrs[self.rank] + base] + [self.ptrs[r] + base for r in peers]
                self._linear(x, qweight_shard, sw, b, outs, ldo, 0, m, nl, epilogue, cur)
            else:
                for r0 in range(0, m, self.chunk_rows):
                    rows = min(self.chunk_rows, m - r0)
                    self._linear(x, qweight_shard, sw, b, [self.ptrs[self.rank] + base], ldo, r0, rows, nl, epilogue,
                                 cur)
                    ev = torch.cuda.Event()
                    ev.record(cur)
                    off = base + r0 * pitch
                    for s, r in zip(self._copy_streams, peers):
                        s.wait_event(ev)
                        if self.layout == "rows":
                            nat.check(self.lib.slim_copy_2d(self.ptrs[r] + off, pitch, self.ptrs[self.rank] + off,
                                                            pitch, nl * 2, rows, s.cuda_stream))
                        else:  # the chunk's rows of this rank's block are contiguous
                            nbytes = rows * pitch
                            nat.check(self.lib.slim_copy_2d(self.ptrs[r] + off, nbytes, self.ptrs[self.rank] + off,
                                                            nbytes, nbytes, 1, s.cuda_stream))
                for s in self._copy_streams:
                    cur.wait_stream(s)
        dist.all_reduce(self._flag, group=self.group)  # every rank's data has landed
        if self.layout == "rows":
            return self.buf[:m]
        return self.buf.view(-1)[: self.world * self.m_max * nl].view(self.world, self.m_max, nl)[:, :m]

    def _linear(self, x, qw, sw, b, outs, ldo, r0, rows, nl, epilogue, stream):
        from . import ops

        arr = (self._ct.c_void_p * len(outs))(*[o + r0 * ldo * 2 for o in outs])
        self._nat.check(self.lib.slim_int8_linear_colsplit(
            x.data_ptr() + r0 * self.k * x.element_size(), ops._DT[x.dtype], qw.data_ptr(), sw.data_ptr(), ops._ptr(b),
            arr, len(outs), ldo, self.xq.data_ptr() + r0 * self.k, self.sx.data_ptr() + r0 * 4, rows, nl,
            self.k, 256, ops._EPI[epilogue], stream.cuda_stream))
