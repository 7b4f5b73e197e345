"""In-place INT8/FP8 flash attention for the Viggle / MiniMax-H3 DiT on sm_100a.

Drop-in for the reference's comfyui/ComfyUI-SlimDiT/attention_triton.py: the same public
names (``packed_geometry``, ``unwrap``, ``TritonAttnConfig``, ``TritonAttnOverride``,
``install_triton_attn``) and the same dispatch rules, with the Triton kernels replaced by the
tcgen05 kernels of libslimdit_b200 (``slim_attn_*``):

    Q, K  int8, one scale per (token, head), after the +-1 Sylvester Hadamard (``rotate``)
    V     E4M3 with one global scale
    QK    tcgen05 kind::i8, int32 in tensor memory; PV tcgen05 kind::f8f6f4, fp32

The packed [S, 3*H*D] bf16 buffer the DiT splits into q/k/v views is read in place
(attention_triton.py:185-222); no contiguous copies are made. Calls the kernel cannot take
(a mask, a layout other than the packed views, a head dim other than 128, a sequence shorter
than ``min_seq``) go back to the model's own attention, as in the reference
(attention_triton.py:253-263, 301-305). There is no CPU path: ``attention_packed`` raises
``NativeUnavailable`` without the library and an sm_100 GPU.
"""

from __future__ import annotations

import ctypes
import dataclasses
import time

DEFAULT_MIN_SEQ = 12000  # below this the dense path wins outright (attention_triton.py:34)
HEAD_DIM = 128  # the one head dim the kernel supports (MiniMax-H3: 56 heads x 128)


def unwrap(value):
    """The tensor inside an attention argument (the contract of attention_triton.py:177-187).

    A tensor is returned as it is. ComfyUI may instead pass a single-owner container whose
    ``take()`` hands over (and gives up) the tensor: that tensor is returned. Anything else is
    returned unchanged for the caller to reject."""
    import torch

    if torch.is_tensor(value):
        return value
    take = getattr(value, "take", None)
    return value if take is None else take()


def packed_geometry(q, k, v, heads):
    """Geometry of the DiT's packed attention input, or None when q, k, v are anything else.

    The kernel reads the projection output in place: one bf16 buffer of rows
    [q heads | k heads | v heads] (3 * heads * dim elements each), of which q, k and v are
    (1, heads, seq, dim) views, k starting heads * dim elements after q and v twice that
    (attention_triton.py:190-222 accepts the same layout). Returned keys: seq, heads, dim,
    row_stride (elements between tokens), head_stride (elements between heads) and row_bytes
    (bytes from one view to the next)."""
    import torch

    views = (q, k, v)
    if any(getattr(t, "ndim", None) != 4 for t in views):
        return None
    batch, n_heads, seq, dim = q.shape
    if batch != 1 or n_heads != heads or seq < 1 or dim < 1 or dim & (dim - 1):
        return None
    row = 3 * heads * dim
    step = heads * dim * q.element_size()
    for i, t in enumerate(views):
        if t.dtype != torch.bfloat16 or tuple(t.shape) != (1, heads, seq, dim):
            return None
        if tuple(t.stride())[1:] != (dim, row, 1) or t.data_ptr() != q.data_ptr() + i * step:
            return None
    return {"seq": seq, "heads": heads, "dim": dim, "row_stride": row, "head_stride": dim, "row_bytes": step}


def attn_scale(dim: int, rotate: bool) -> float:
    """The unnormalised Hadamard makes (qH).(kH)^T = dim * q.k^T, so the scale carries 1/dim
    (attention_triton.py:296-298)."""
    return dim ** -0.5 / (dim if rotate else 1.0)


def workspace_bytes(seq: int, heads: int, dim: int = HEAD_DIM) -> int:
    from . import _native as nat

    out = ctypes.c_uint64(0)
    nat.check(nat.load().slim_attn_workspace_bytes(int(seq), int(heads), int(dim), ctypes.byref(out)))
    return int(out.value)


def attention_packed(qkv, heads: int, rotate: bool = True, out=None, workspace=None):
    """Attention over a packed [seq, 3*heads*128] bf16 CUDA buffer (rows may be longer: the row
    pitch is taken from the tensor's stride) -> bf16 [seq, heads*128].

    The device entry point behind ``TritonAttnOverride``: quantise q/k (int8 per token and
    head, rotated) and v (E4M3, global scale), then the tcgen05 flash kernel."""
    from . import _native as nat

    torch = nat.require_cuda()
    if qkv.dim() != 2 or qkv.dtype != torch.bfloat16 or not qkv.is_cuda or qkv.stride(1) != 1:
        raise ValueError("qkv must be a CUDA bf16 [seq, 3*heads*dim] tensor with unit column stride")
    seq, width = qkv.shape
    hd = heads * HEAD_DIM
    if width != 3 * hd:
        raise ValueError(f"qkv has {width} columns; {heads} heads of dim {HEAD_DIM} need {3 * hd}")
    lib = nat.load()
    dev = qkv.device
    if out is None:
        out = torch.empty((seq, hd), dtype=torch.bfloat16, device=dev)
    if seq == 0:
        return out
    if out.shape != (seq, hd) or out.dtype != torch.bfloat16 or out.stride(1) != 1:
        raise ValueError("out must be bf16 [seq, heads*dim] with unit column stride")
    need = workspace_bytes(seq, heads)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty((need,), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    row_stride = qkv.stride(0)
    if row_stride == 3 * hd and out.stride(0) == hd:
        nat.check(lib.slim_attn_packed(qkv.data_ptr(), seq, heads, HEAD_DIM, int(bool(rotate)), out.data_ptr(),
                                       workspace.data_ptr(), need, st))
        return out
    # general row pitches: the three stages with the packed entry's workspace layout
    parts = _workspace_views(workspace, seq, heads)
    nat.check(lib.slim_attn_quant_qk(qkv.data_ptr(), seq, heads, HEAD_DIM, row_stride, 0, hd, int(bool(rotate)),
                                     parts["q"], parts["qs"], parts["k"], parts["ks"], parts["seq_pad"], st))
    nat.check(lib.slim_attn_quant_v(qkv.data_ptr(), seq, heads, HEAD_DIM, row_stride, 2 * hd, parts["v"],
                                    parts["seq_pad"], parts["amax"], st))
    nat.check(lib.slim_attn_int8(parts["q"], parts["qs"], parts["k"], parts["ks"], parts["v"], parts["amax"],
                                 attn_scale(HEAD_DIM, rotate), seq, heads, HEAD_DIM, parts["seq_pad"],
                                 out.data_ptr(), out.stride(0), st))
    return out


def _workspace_views(workspace, seq: int, heads: int) -> dict:
    """Byte offsets of the quantised operands inside a slim_attn_packed workspace."""
    def up(v, a=256):
        return (v + a - 1) // a * a

    hd = heads * HEAD_DIM
    seq_pad = up(seq, 128)
    base = workspace.data_ptr()
    off = {}
    o = 0
    for name, size in (("q", seq * hd), ("k", seq * hd), ("v", hd * seq_pad), ("qs", heads * seq_pad * 4),
                       ("ks", heads * seq_pad * 4), ("amax", 4)):
        off[name] = base + o
        o = up(o + size)
    off["seq_pad"] = seq_pad
    return off


def quantized_operands(qkv, heads: int, rotate: bool = True) -> dict:
    """The quantiser stage alone (test and inspection hook): int8 q/k [seq, heads*128], their
    scales [heads, seq_pad], v as E4M3 bits [heads, 128, seq_pad] and max|v|."""
    from . import _native as nat

    torch = nat.require_cuda()
    seq = qkv.shape[0]
    hd = heads * HEAD_DIM
    seq_pad = (seq + 127) // 128 * 128
    dev = qkv.device
    q = torch.empty((seq, hd), dtype=torch.int8, device=dev)
    k = torch.empty((seq, hd), dtype=torch.int8, device=dev)
    qs = torch.empty((heads, seq_pad), dtype=torch.float32, device=dev)
    ks = torch.empty((heads, seq_pad), dtype=torch.float32, device=dev)
    v = torch.empty((heads, HEAD_DIM, seq_pad), dtype=torch.uint8, device=dev)
    amax = torch.empty((1,), dtype=torch.float32, device=dev)
    lib = nat.load()
    st = torch.cuda.current_stream(dev).cuda_stream
    nat.check(lib.slim_attn_quant_qk(qkv.data_ptr(), seq, heads, HEAD_DIM, qkv.stride(0), 0, hd, int(bool(rotate)),
                                     q.data_ptr(), qs.data_ptr(), k.data_ptr(), ks.data_ptr(), seq_pad, st))
    nat.check(lib.slim_attn_quant_v(qkv.data_ptr(), seq, heads, HEAD_DIM, qkv.stride(0), 2 * hd, v.data_ptr(), seq_pad,
                                    amax.data_ptr(), st))
    return {"q": q, "q_scale": qs, "k": k, "k_scale": ks, "v": v, "v_amax": amax, "seq_pad": seq_pad}


def attention_quantized(ops: dict, seq: int, heads: int, scale: float, out=None):
    """The flash kernel alone on ``quantized_operands`` output -> bf16 [seq, heads*128]."""
    from . import _native as nat

    torch = nat.require_cuda()
    dev = ops["q"].device
    hd = heads * HEAD_DIM
    if out is None:
        out = torch.empty((seq, hd), dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    nat.check(nat.load().slim_attn_int8(ops["q"].data_ptr(), ops["q_scale"].data_ptr(), ops["k"].data_ptr(),
                                        ops["k_scale"].data_ptr(), ops["v"].data_ptr(), ops["v_amax"].data_ptr(),
                                        float(scale), seq, heads, HEAD_DIM, ops["seq_pad"], out.data_ptr(),
                                        out.stride(0), st))
    return out


def attention_heads(qkv, heads: int, rank: int, world: int, rotate: bool = True, group=None, out=None):
    """Heads [rank*H/world, (rank+1)*H/world) of the packed [seq, 3*H*128] buffer on this GPU ->
    bf16 [seq, H/world*128].

    The V scale is one number for the whole tensor (attention_triton.py:283-286): every rank
    computes max|v| over its own heads, the maxima are all-reduced (MAX, one float), and every
    rank quantises with the global value, so the result equals the single-GPU one bit for bit.
    Q/K quantisation and the attention itself are per head; no other data crosses GPUs."""
    from . import _native as nat
    import torch.distributed as dist

    torch = nat.require_cuda()
    if heads % world:
        raise ValueError(f"{heads} heads do not split over {world} ranks")
    hl = heads // world
    h0 = rank * hl
    hd = heads * HEAD_DIM
    seq = qkv.shape[0]
    if qkv.shape[1] != 3 * hd or qkv.stride(1) != 1 or qkv.dtype != torch.bfloat16:
        raise ValueError("qkv must be a bf16 [seq, 3*heads*128] tensor with unit column stride")
    seq_pad = (seq + 127) // 128 * 128
    dev = qkv.device
    lib = nat.load()
    st = torch.cuda.current_stream(dev).cuda_stream
    q = torch.empty((seq, hl * HEAD_DIM), dtype=torch.int8, device=dev)
    k = torch.empty_like(q)
    qs = torch.empty((hl, seq_pad), dtype=torch.float32, device=dev)
    ks = torch.empty_like(qs)
    v = torch.empty((hl, HEAD_DIM, seq_pad), dtype=torch.uint8, device=dev)
    amax = torch.empty((1,), dtype=torch.float32, device=dev)
    if out is None:
        out = torch.empty((seq, hl * HEAD_DIM), dtype=torch.bfloat16, device=dev)
    row = qkv.stride(0)
    nat.check(lib.slim_attn_quant_qk(qkv.data_ptr(), seq, hl, HEAD_DIM, row, h0 * HEAD_DIM, hd + h0 * HEAD_DIM,
                                     int(bool(rotate)), q.data_ptr(), qs.data_ptr(), k.data_ptr(), ks.data_ptr(),
                                     seq_pad, st))
    nat.check(lib.slim_attn_v_amax(qkv.data_ptr(), seq, hl, HEAD_DIM, row, 2 * hd + h0 * HEAD_DIM, amax.data_ptr(), st))
    if world > 1:
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    nat.check(lib.slim_attn_quant_v_scaled(qkv.data_ptr(), seq, hl, HEAD_DIM, row, 2 * hd + h0 * HEAD_DIM,
                                           v.data_ptr(), seq_pad, amax.data_ptr(), st))
    nat.check(lib.slim_attn_int8(q.data_ptr(), qs.data_ptr(), k.data_ptr(), ks.data_ptr(), v.data_ptr(),
                                 amax.data_ptr(), attn_scale(HEAD_DIM, rotate), seq, hl, HEAD_DIM, seq_pad,
                                 out.data_ptr(), out.stride(0), st))
    return out


@dataclasses.dataclass
class TritonAttnConfig:
    """Settings of the attention override (the reference's name, attention_triton.py:225-245).

    enabled      the override may be installed (install_triton_attn returns None otherwise)
    min_seq      shorter sequences stay on the model's own attention
    fail_closed  raise at install when the kernel cannot run here (default: keep the model's
                 attention and say so)
    rotate       Hadamard-rotate q and k before their int8 quantisation
    """

    enabled: bool = False
    min_seq: int = DEFAULT_MIN_SEQ
    fail_closed: bool = False
    rotate: bool = True

    def describe(self) -> dict:
        return {"kernel": "tcgen05 int8 QK / fp8 PV flash attention, head dim 128", "min_seq": self.min_seq,
                "rotate": self.rotate}


class TritonAttnOverride:
    """A stand-in for ``comfy.ldm.minimax.model.optimized_attention`` (the reference's override,
    attention_triton.py:248-305): same call signature; the packed DiT layout runs on the sm_100a
    kernel, every other call goes to the model's own attention (``dense``).

    ``install()`` puts it in the model module and keeps the function it replaces; used without
    installing (an attention router holding it), ``dense`` is the module's function at the time
    of the first call it cannot take. ``stats`` counts ``calls``, ``kernel_calls`` and
    ``fallback_calls`` and adds up ``kernel_seconds`` (host time to dispatch the kernels)."""

    MODEL_MODULE = "comfy.ldm.minimax.model"

    def __init__(self, config: TritonAttnConfig, stats: dict | None = None):
        if not config.enabled:
            raise ValueError("TritonAttnOverride needs a config with enabled=True")
        self.config = config
        self.stats = {} if stats is None else stats
        for key, zero in (("calls", 0), ("kernel_calls", 0), ("fallback_calls", 0), ("kernel_seconds", 0.0)):
            self.stats.setdefault(key, zero)
        self.dense = None          # the model's own attention
        self._installed_in = None  # the module this instance was put into
        self._workspace = {}       # device -> uint8 workspace of the kernels

    # ------------------------------------------------------------------ installation
    def install(self):
        import importlib

        module = importlib.import_module(self.MODEL_MODULE)
        self.dense = module.optimized_attention
        problem = _kernel_problem()
        if problem is not None:
            if self.config.fail_closed:
                raise RuntimeError(f"sm_100a attention unavailable: {problem}")
            print(f"[slim-attn] disabled, the model keeps its attention: {problem}", flush=True)
            return self
        module.optimized_attention = self
        self._installed_in = module
        return self

    def uninstall(self):
        module, self._installed_in = self._installed_in, None
        if module is not None and module.optimized_attention is self:
            module.optimized_attention = self.dense

    # ------------------------------------------------------------------ calls
    def __call__(self, q, k, v, heads, mask=None, skip_reshape=False, skip_output_reshape=False, **kwargs):
        self.stats["calls"] += 1
        q, k, v = unwrap(q), unwrap(k), unwrap(v)  # containers give their tensor up once
        geometry = self._takes(q, k, v, heads, mask, skip_reshape)
        if geometry is None:
            self.stats["fallback_calls"] += 1
            return self._dense()(q, k, v, heads, mask=mask, skip_reshape=skip_reshape,
                                 skip_output_reshape=skip_output_reshape, **kwargs)
        started = time.perf_counter()
        out = self._attend(q, geometry)
        self.stats["kernel_seconds"] += time.perf_counter() - started
        self.stats["kernel_calls"] += 1
        seq, dim = geometry["seq"], geometry["dim"]
        if skip_output_reshape:  # (1, heads, seq, dim), as the model's own attention returns it
            return out.view(1, seq, heads, dim).transpose(1, 2)
        return out.view(1, seq, heads * dim)

    def _takes(self, q, k, v, heads, mask, skip_reshape):
        """The geometry when the kernel takes this call: no mask, the packed layout of pre-shaped
        views, head dim 128 and at least min_seq tokens; else None."""
        if mask is not None or not skip_reshape:
            return None
        geometry = packed_geometry(q, k, v, heads)
        if geometry is None or geometry["dim"] != HEAD_DIM or geometry["seq"] < self.config.min_seq:
            return None
        return geometry

    def _attend(self, q, geometry):
        import torch

        seq, heads, dim = geometry["seq"], geometry["heads"], geometry["dim"]
        # q is the first column block of the packed rows: the whole [seq, 3*heads*dim] buffer as a 2-D view
        packed = torch.as_strided(q, (seq, 3 * heads * dim), (geometry["row_stride"], 1), q.storage_offset())
        need = workspace_bytes(seq, heads, dim)
        ws = self._workspace.get(q.device)
        if ws is None or ws.numel() < need:
            ws = self._workspace[q.device] = torch.empty((need,), dtype=torch.uint8, device=q.device)
        return attention_packed(packed, heads, rotate=self.config.rotate, workspace=ws)

    def _dense(self):
        if self.dense is None:
            import importlib

            self.dense = importlib.import_module(self.MODEL_MODULE).optimized_attention
        return self.dense


def _kernel_problem() -> str | None:
    """Why the sm_100a attention cannot run in this process (no library, no sm_100 device), or None."""
    try:
        from . import _native

        _native.load()
        _native.require_cuda()
    except Exception as exc:  # noqa: BLE001 - reported to the caller, who decides how to fail
        return str(exc)
    return None


def install_triton_attn(config: TritonAttnConfig | None = None, stats: dict | None = None):
    """Install the sm_100a attention for every length it takes (the reference's
    ``VIGGLE_ATTN=triton``, attention_triton.py:348-353); None when the config is disabled."""
    config = TritonAttnConfig(enabled=True) if config is None else config
    return TritonAttnOverride(config, stats).install() if config.enabled else None


__all__ = [
    "DEFAULT_MIN_SEQ", "HEAD_DIM", "TritonAttnConfig", "TritonAttnOverride", "attention_heads", "attention_packed",
    "attention_quantized",
    "attn_scale", "install_triton_attn", "packed_geometry", "quantized_operands", "unwrap", "workspace_bytes",
]
