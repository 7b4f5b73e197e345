"""Device entry points on torch CUDA tensors (memory comes from torch's allocator; every
computation runs in libslimdit_b200.so).

* ``rotate_quant``  group-256 Hadamard rotation + per-row INT8 (slimdit/int8.py:39-52), in the
  reference's summation order (codes and scales identical to the reference's, for weights
  and for the per-token activation side of the runtime linear) or the butterfly order
* ``rotate``        rotation alone, fp32 out (slimdit/hadamard.py:45-58)
* ``quantize_rows`` quantisation alone (slimdit/int8.py:49-51)
* ``dequantize``    (q * scale) @ H^T (slimdit/int8.py:55-61)
* ``gemm_i8``       int8 GEMM + scale/bias(/GELU) epilogue
* ``int8_linear``   the convrot W8A8 linear, same call shape as the runtime op the reference
                    benchmarks (``comfy_kitchen.int8_linear``, tools/bench_int8.py:65-68)
* ``ffn_int8``      up-proj -> GELU-tanh -> rotate + requant -> down-proj
* ``swiglu_interleave`` / ``ffn_swiglu_int8``  the MiniMax-H3 FFN: fc1 with a fused SwiGLU
                    epilogue, rotate + requant, fc2
* ``int8_linear_host``  the linear on host-resident activations, copies and compute of row
                    chunks overlapped on three streams
* ``nvfp4_pack`` / ``nvfp4_quantize_act`` / ``nvfp4_dequantize`` / ``nvfp4_error`` /
  ``gemm_nvfp4`` / ``nvfp4_linear``  the NVFP4 format of slimdit/nvfp4.py and its linear
"""

from __future__ import annotations

import torch

from . import _native as nat

_DT = {torch.float32: nat.F32, torch.bfloat16: nat.BF16, torch.float16: nat.F16}
_ORDERS = {"reference": nat.ORDER_REFERENCE, "butterfly": nat.ORDER_BUTTERFLY}
_EPI = {None: nat.EPI_SCALE_BIAS, "none": nat.EPI_SCALE_BIAS, "gelu_tanh": nat.EPI_GELU_TANH,
        "swiglu": nat.EPI_SWIGLU}


def _cuda2d(t: torch.Tensor, name: str) -> torch.Tensor:
    nat.require_cuda()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dim() != 2:
        raise ValueError(f"expected a 2D {name}, got shape {tuple(t.shape)}")
    return t.contiguous()


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def rotate_quant(x: torch.Tensor, group_size: int = 256, order: str = "reference",
                 return_rotated: bool = False):
    """Rotate [rows, K] (f32/bf16/f16) and quantise per row -> (int8 [rows, K], f32 [rows, 1][, f32 rotated])."""
    x = _cuda2d(x, "input")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported dtype {x.dtype}")
    if order not in _ORDERS:
        raise ValueError(f"order must be one of {sorted(_ORDERS)}")
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.int8, device=x.device)
    scale = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    rot = torch.empty((rows, k), dtype=torch.float32, device=x.device) if return_rotated else None
    with torch.cuda.device(x.device):
        nat.check(nat.load().slim_rotate_quant_i8(x.data_ptr(), _DT[x.dtype], rows, k, group_size, _ORDERS[order],
                                                  q.data_ptr(), scale.data_ptr(), _ptr(rot), _stream(x)))
    return (q, scale, rot) if return_rotated else (q, scale)


def rotate(x: torch.Tensor, group_size: int = 256) -> torch.Tensor:
    """fp32 group-wise rotation W @ H^T in the reference order."""
    x = _cuda2d(x, "weight")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported dtype {x.dtype}")
    rows, k = x.shape
    out = torch.empty((rows, k), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        nat.check(nat.load().slim_rotate_f32(x.data_ptr(), _DT[x.dtype], rows, k, group_size, nat.ORDER_REFERENCE,
                                             out.data_ptr(), _stream(x)))
    return out


def quantize_rows(rotated: torch.Tensor):
    """Per-row symmetric INT8 of fp32 rows -> (int8 [rows, K], f32 [rows, 1])."""
    rotated = _cuda2d(rotated, "rotated")
    if rotated.dtype != torch.float32:
        raise TypeError("rotated rows must be float32")
    rows, k = rotated.shape
    q = torch.empty((rows, k), dtype=torch.int8, device=rotated.device)
    scale = torch.empty((rows, 1), dtype=torch.float32, device=rotated.device)
    with torch.cuda.device(rotated.device):
        nat.check(nat.load().slim_quantize_rows_i8(rotated.data_ptr(), rows, k, q.data_ptr(), scale.data_ptr(),
                                                   _stream(rotated)))
    return q, scale


def dequantize(q: torch.Tensor, scale: torch.Tensor, group_size: int = 256) -> torch.Tensor:
    """(q * scale) @ H^T in the reference order -> fp32 [rows, K]."""
    q = _cuda2d(q, "q")
    if q.dtype != torch.int8:
        raise TypeError("q must be int8")
    rows, k = q.shape
    scale = scale.to(device=q.device, dtype=torch.float32).contiguous().reshape(-1)
    if scale.numel() != rows:
        raise ValueError(f"scale has {scale.numel()} entries for {rows} rows")
    out = torch.empty((rows, k), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        nat.check(nat.load().slim_dequant_i8(q.data_ptr(), scale.data_ptr(), rows, k, group_size, out.data_ptr(),
                                             _stream(q)))
    return out


def _vec(t: torch.Tensor | None, n: int, dtype, device, name: str) -> torch.Tensor | None:
    if t is None:
        return None
    t = t.to(device=device, dtype=dtype).contiguous().reshape(-1)
    if t.numel() != n:
        raise ValueError(f"{name} has {t.numel()} entries, expected {n}")
    return t


def gemm_i8(a: torch.Tensor, b: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None = None,
            epilogue: str | None = None, return_acc: bool = False, out: torch.Tensor | None = None):
    """bf16(acc * sa[m] * sb[n] + bias[n]) (optionally GELU-tanh) for int8 a [M,K], b [N,K]."""
    a = _cuda2d(a, "a")
    b = _cuda2d(b, "b")
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise TypeError("a and b must be int8")
    m, k = a.shape
    n, kb = b.shape
    if k != kb:
        raise ValueError(f"K mismatch: a {tuple(a.shape)} vs b {tuple(b.shape)}")
    if epilogue not in _EPI:
        raise ValueError(f"epilogue must be one of {sorted(str(e) for e in _EPI)}")
    dev = a.device
    sa = _vec(sa, m, torch.float32, dev, "sa")
    sb = _vec(sb, n, torch.float32, dev, "sb")
    bias = _vec(bias, n, torch.bfloat16, dev, "bias")
    n_out = n // 2 if epilogue == "swiglu" else n
    if out is None:
        out = torch.empty((m, n_out), dtype=torch.bfloat16, device=dev)
    elif out.shape != (m, n_out) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous bf16 [{m}, {n_out}] tensor")
    acc = torch.empty((m, n), dtype=torch.int32, device=dev) if return_acc else None
    with torch.cuda.device(dev):
        nat.check(nat.load().slim_gemm_i8(a.data_ptr(), b.data_ptr(), sa.data_ptr(), sb.data_ptr(), _ptr(bias),
                                          out.data_ptr(), _ptr(acc), m, n, k, _EPI[epilogue], _stream(a)))
    return (out, acc) if return_acc else out


def int8_linear(x: torch.Tensor, qweight: torch.Tensor, wscales: torch.Tensor, convrot: bool = True,
                convrot_groupsize: int = 256, out_dtype: torch.dtype = torch.bfloat16,
                bias: torch.Tensor | None = None, epilogue: str | None = None,
                order: str = "reference") -> torch.Tensor:
    """Convrot W8A8 linear: y = rot(x) quantised per token @ (qweight * wscales)^T + bias.

    x: [..., K] bf16/f16/f32 CUDA; qweight: int8 [N, K] (pre-rotated, slimdit/int8.py:3-11);
    wscales: f32 [N, 1] or [N]. Same call shape as the runtime op the reference uses
    (tools/bench_int8.py:65-68). The output is computed in bf16 and cast if out_dtype differs.
    order="reference" (slim_int8_linear) quantises the activations exactly as the reference's
    rotate() + int8.py math would; order="butterfly" uses the fast transform alone
    (slim_rotate_quant_i8 + slim_gemm_i8).
    """
    nat.require_cuda()
    if not x.is_cuda:
        raise TypeError("x must be a CUDA tensor")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported activation dtype {x.dtype}")
    qweight = _cuda2d(qweight, "qweight")
    k = x.shape[-1]
    n = qweight.shape[0]
    if qweight.shape[1] != k:
        raise ValueError(f"in_features mismatch: x [..., {k}] vs qweight {tuple(qweight.shape)}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k).contiguous()
    m = x2.shape[0]
    dev = x2.device
    sw = _vec(wscales, n, torch.float32, dev, "wscales")
    b = _vec(bias, n, torch.bfloat16, dev, "bias")
    n_out = n // 2 if epilogue == "swiglu" else n
    out = torch.empty((m, n_out), dtype=torch.bfloat16, device=dev)
    if order not in _ORDERS:
        raise ValueError(f"order must be one of {sorted(_ORDERS)}")
    if convrot and order == "butterfly":
        xq, sx = rotate_quant(x2, convrot_groupsize, order="butterfly")
        gemm_i8(xq, qweight, sx, sw, b, epilogue=epilogue, out=out)
    elif convrot:
        xq = torch.empty((m, k), dtype=torch.int8, device=dev)
        sx = torch.empty((m,), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            nat.check(nat.load().slim_int8_linear(x2.data_ptr(), _DT[x2.dtype], qweight.data_ptr(), sw.data_ptr(),
                                                  _ptr(b), out.data_ptr(), xq.data_ptr(), sx.data_ptr(), m, n, k,
                                                  convrot_groupsize, _EPI[epilogue], _stream(x2)))
    else:
        if epilogue == "swiglu":
            raise ValueError("the SwiGLU epilogue needs convrot=True")
        xq, sx = quantize_rows(x2.float())
        gemm_i8(xq, qweight, sx, sw, b, epilogue=epilogue, out=out)
    out = out.reshape(*lead, n_out)
    return out if out_dtype == torch.bfloat16 else out.to(out_dtype)


def ffn_int8(x: torch.Tensor, w_up: torch.Tensor, s_up: torch.Tensor, w_down: torch.Tensor, s_down: torch.Tensor,
             b_up: torch.Tensor | None = None, b_down: torch.Tensor | None = None,
             order: str = "reference") -> torch.Tensor:
    """DiT FFN pair on the convrot linear: down(rotquant(gelu_tanh(up(x)))).

    The up-projection's epilogue applies GELU-tanh to its bf16 output (the same rounding as
    running the linear and then the activation on its bf16 result); the hidden activation
    is rotated and requantised per token before the down-projection. order="reference" runs
    slim_ffn_i8 (reference-order activation codes); order="butterfly" composes the two
    linears with the fast transform.
    """
    if order == "butterfly":
        h = int8_linear(x, w_up, s_up, bias=b_up, epilogue="gelu_tanh", order="butterfly")
        return int8_linear(h, w_down, s_down, bias=b_down, order="butterfly")
    if order != "reference":
        raise ValueError(f"order must be one of {sorted(_ORDERS)}")
    return _ffn(x, w_up, s_up, b_up, w_down, s_down, b_down, "gelu_tanh")


def _ffn(x, w_up, s_up, b_up, w_down, s_down, b_down, act: str) -> torch.Tensor:
    """Both projections of an FFN in one slim_ffn_i8 call (the C entry a plugin binds); the
    hidden activation and the quantised copies live in stream-ordered workspaces."""
    nat.require_cuda()
    if not x.is_cuda:
        raise TypeError("x must be a CUDA tensor")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported activation dtype {x.dtype}")
    w_up, w_down = _cuda2d(w_up, "w_up"), _cuda2d(w_down, "w_down")
    k = x.shape[-1]
    f = w_down.shape[1]
    n_up = 2 * f if act == "swiglu" else f
    if w_up.shape != (n_up, k) or w_down.shape != (k, f):
        raise ValueError(f"FFN weights {tuple(w_up.shape)} / {tuple(w_down.shape)} do not fit x [..., {k}] "
                         f"with the {act} activation")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k).contiguous()
    m, dev = x2.shape[0], x2.device
    su, sd = _vec(s_up, n_up, torch.float32, dev, "s_up"), _vec(s_down, k, torch.float32, dev, "s_down")
    bu, bd = _vec(b_up, n_up, torch.bfloat16, dev, "b_up"), _vec(b_down, k, torch.bfloat16, dev, "b_down")
    out = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    sx = torch.empty((m,), dtype=torch.float32, device=dev)
    h = torch.empty((m, f), dtype=torch.bfloat16, device=dev)
    hq = torch.empty((m, f), dtype=torch.int8, device=dev)
    sh = torch.empty((m,), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        nat.check(nat.load().slim_ffn_i8(x2.data_ptr(), _DT[x2.dtype], w_up.data_ptr(), su.data_ptr(), _ptr(bu),
                                         w_down.data_ptr(), sd.data_ptr(), _ptr(bd), out.data_ptr(), xq.data_ptr(),
                                         sx.data_ptr(), h.data_ptr(), hq.data_ptr(), sh.data_ptr(), m, k, f,
                                         _EPI[act], _stream(x2)))
    return out.reshape(*lead, k)


_PIPE_STREAMS: dict[int, tuple] = {}


def _pipe_streams(dev: torch.device):
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _PIPE_STREAMS:
        _PIPE_STREAMS[idx] = tuple(torch.cuda.Stream(device=idx) for _ in range(3))
    return _PIPE_STREAMS[idx]


def int8_linear_host(x: torch.Tensor, qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None = None,
                     out: torch.Tensor | None = None, chunk_rows: int = 4096, convrot_groupsize: int = 256,
                     epilogue: str | None = None) -> torch.Tensor:
    """The convrot linear for activations in host memory: y_host = int8_linear(x_host) on the
    weight's GPU, with the host->device copy, the linear and the device->host copy of
    successive row chunks overlapped on three streams (two device buffers per direction).

    x: host [M, K] bf16/f16/f32 (pinned for asynchronous copies); out: host bf16 [M, N]
    (allocated pinned when x is pinned, if not given). Token rows are independent, so the
    result equals int8_linear on the whole batch bit for bit. The copies into `out` are
    asynchronous with respect to the host, like non_blocking copies: synchronise the current
    stream before reading it.
    """
    nat.require_cuda()
    if x.is_cuda or x.dim() != 2:
        raise TypeError("x must be a 2-D host tensor")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported activation dtype {x.dtype}")
    qweight = _cuda2d(qweight, "qweight")
    dev = qweight.device
    m, k = x.shape
    n = qweight.shape[0]
    if qweight.shape[1] != k:
        raise ValueError(f"in_features mismatch: x [..., {k}] vs qweight {tuple(qweight.shape)}")
    if epilogue not in _EPI or epilogue == "swiglu":
        raise ValueError("epilogue must be None, 'none' or 'gelu_tanh' for the host-memory linear")
    if chunk_rows <= 0:
        raise ValueError("chunk_rows must be positive")
    sw = _vec(wscales, n, torch.float32, dev, "wscales")
    b = _vec(bias, n, torch.bfloat16, dev, "bias")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, pin_memory=x.is_pinned())
    elif out.is_cuda or out.shape != (m, n) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous host bf16 [M, N] tensor")
    if m == 0:
        return out
    x = x.contiguous()
    chunk = min(chunk_rows, m)
    s_h2d, s_cmp, s_d2h = _pipe_streams(dev)
    cur = torch.cuda.current_stream(dev)
    lib = nat.load()
    with torch.cuda.device(dev):
        xb = [torch.empty((chunk, k), dtype=x.dtype, device=dev) for _ in range(2)]
        yb = [torch.empty((chunk, n), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        xq = torch.empty((chunk, k), dtype=torch.int8, device=dev)
        sx = torch.empty((chunk,), dtype=torch.float32, device=dev)
        ev_h2d = [torch.cuda.Event() for _ in range(2)]
        ev_cmp = [torch.cuda.Event() for _ in range(2)]
        ev_d2h = [torch.cuda.Event() for _ in range(2)]
        for s in (s_h2d, s_cmp, s_d2h):
            s.wait_stream(cur)  # weights, scales and buffers come from the current stream
        for i, r0 in enumerate(range(0, m, chunk)):
            j = i % 2
            rows = min(chunk, m - r0)
            with torch.cuda.stream(s_h2d):
                if i >= 2:
                    s_h2d.wait_event(ev_cmp[j])      # the linear of chunk i-2 has read xb[j]
                xb[j][:rows].copy_(x[r0:r0 + rows], non_blocking=True)
                ev_h2d[j].record(s_h2d)
            s_cmp.wait_event(ev_h2d[j])
            if i >= 2:
                s_cmp.wait_event(ev_d2h[j])          # chunk i-2's output has left yb[j]
            nat.check(lib.slim_int8_linear(xb[j].data_ptr(), _DT[x.dtype], qweight.data_ptr(), sw.data_ptr(), _ptr(b),
                                           yb[j].data_ptr(), xq.data_ptr(), sx.data_ptr(), rows, n, k,
                                           convrot_groupsize, _EPI[epilogue], s_cmp.cuda_stream))
            ev_cmp[j].record(s_cmp)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(ev_cmp[j])
                out[r0:r0 + rows].copy_(yb[j][:rows], non_blocking=True)
                ev_d2h[j].record(s_d2h)
        for t in (*xb, *yb, xq, sx, sw, qweight, *( [b] if b is not None else [])):
            t.record_stream(s_h2d)
            t.record_stream(s_cmp)
            t.record_stream(s_d2h)
        cur.wait_stream(s_d2h)
        cur.wait_stream(s_cmp)
        cur.wait_stream(s_h2d)
    return out


def swiglu_interleave(qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None = None):
    """Reorder a gated projection's rows [up; gate] (N = 2F rows, ComfyUI's swiglu order,
    slimdit/mapping.py:96-97) into the SwiGLU epilogue's order: per 256-row tile, 128 up rows
    then the 128 matching gate rows. Pure data movement (2-D copies on the current stream);
    returns (qweight, wscales [N], bias [N] or None)."""
    qweight = _cuda2d(qweight, "qweight")
    n, k = qweight.shape
    if n % 256:
        raise ValueError(f"the gated projection needs a multiple of 256 rows, got {n}")
    dev = qweight.device
    f = n // 2
    sw = _vec(wscales, n, torch.float32, dev, "wscales")
    b = _vec(bias, n, torch.bfloat16, dev, "bias")
    lib = nat.load()
    st = _stream(qweight)
    outs = []
    with torch.cuda.device(dev):
        for t in (qweight, sw, b):
            if t is None:
                outs.append(None)
                continue
            row = (t.shape[1] if t.dim() == 2 else 1) * t.element_size()
            dst = torch.empty_like(t)
            for half in (0, 1):  # up rows -> first 128 of each tile, gate rows -> last 128
                nat.check(lib.slim_copy_2d(dst.data_ptr() + half * 128 * row, 256 * row,
                                           t.data_ptr() + half * f * row, 128 * row, 128 * row, f // 128, st))
            outs.append(dst)
    return outs[0], outs[1], outs[2]


def ffn_swiglu_int8(x: torch.Tensor, w_fc1: torch.Tensor, s_fc1: torch.Tensor, w_fc2: torch.Tensor,
                    s_fc2: torch.Tensor, b_fc1: torch.Tensor | None = None,
                    b_fc2: torch.Tensor | None = None) -> torch.Tensor:
    """The MiniMax-H3 FFN on the convrot linear: fc2(rotquant(swiglu(fc1(x)))).

    w_fc1/s_fc1/b_fc1 are the gated projection in :func:`swiglu_interleave` order (prepare once
    at load time); fc1's epilogue applies SwiGLU to its bf16 outputs and writes [M, F]; the
    result is rotated and requantised per token for fc2."""
    return _ffn(x, w_fc1, s_fc1, b_fc1, w_fc2, s_fc2, b_fc2, "swiglu")


# ---------------------------------------------------------------- NVFP4
# Format of slimdit/nvfp4.py:3-8 (weight uint8 [N, K/2], weight_scale uint8 [N, K/16] in the
# 128x4 tiled layout, weight_scale_2 fp32); the arithmetic runs in libslimdit_b200.so.

def _rows_pad(rows: int) -> int:
    return (rows + 127) // 128 * 128


def nvfp4_pack(w: torch.Tensor):
    """Per-tensor NVFP4 of a [N, K] weight (f32/bf16/f16 CUDA) -> (uint8 [N, K/2], uint8
    [N, K/16] tiled block scales, fp32 [1] global scale), as slimdit/nvfp4.py:72-87."""
    w = _cuda2d(w, "weight")
    if w.dtype not in _DT:
        raise TypeError(f"unsupported dtype {w.dtype}")
    n, k = w.shape
    q = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    sf = torch.empty((n, k // 16), dtype=torch.uint8, device=w.device)
    ts = torch.empty((1,), dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        nat.check(nat.load().slim_nvfp4_pack(w.data_ptr(), _DT[w.dtype], n, k, q.data_ptr(), sf.data_ptr(),
                                             ts.data_ptr(), _stream(w)))
    return q, sf, ts


def nvfp4_quantize_act(x: torch.Tensor, rotate: bool = False, out=None):
    """Per-token NVFP4 of activations [M, K] (optionally rotated first) -> (uint8 [M, K/2],
    uint8 [round_up(M, 128), K/16] tiled block scales, fp32 [M] row scales)."""
    x = _cuda2d(x, "input")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported dtype {x.dtype}")
    m, k = x.shape
    if out is None:
        q = torch.empty((m, k // 2), dtype=torch.uint8, device=x.device)
        sf = torch.empty((_rows_pad(m), k // 16), dtype=torch.uint8, device=x.device)
        rs = torch.empty((m,), dtype=torch.float32, device=x.device)
    else:
        q, sf, rs = out
    with torch.cuda.device(x.device):
        nat.check(nat.load().slim_quant_nvfp4_act(x.data_ptr(), _DT[x.dtype], m, k, int(bool(rotate)), q.data_ptr(),
                                                  sf.data_ptr(), rs.data_ptr(), _stream(x)))
    return q, sf, rs


def nvfp4_dequantize(q: torch.Tensor, sf: torch.Tensor, scale: torch.Tensor, per_row: bool = False) -> torch.Tensor:
    """code * (scale * block_scale) -> fp32 [rows, K]."""
    q = _cuda2d(q, "q")
    rows, k = q.shape[0], q.shape[1] * 2
    scale = scale.to(device=q.device, dtype=torch.float32).contiguous().reshape(-1)
    out = torch.empty((rows, k), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        nat.check(nat.load().slim_nvfp4_dequant(q.data_ptr(), sf.contiguous().data_ptr(), scale.data_ptr(),
                                                int(bool(per_row)), rows, k, out.data_ptr(), None, 0, None,
                                                _stream(q)))
    return out


def nvfp4_error(q: torch.Tensor, sf: torch.Tensor, scale: torch.Tensor, x: torch.Tensor) -> float:
    """Relative round-trip error ||dequant - x|| / ||x|| (slimdit/nvfp4.py:98-99), fp64 sums."""
    q = _cuda2d(q, "q")
    x = _cuda2d(x, "x")
    rows, k = q.shape[0], q.shape[1] * 2
    scale = scale.to(device=q.device, dtype=torch.float32).contiguous().reshape(-1)
    acc = torch.zeros((2,), dtype=torch.float64, device=q.device)
    with torch.cuda.device(q.device):
        nat.check(nat.load().slim_nvfp4_dequant(q.data_ptr(), sf.contiguous().data_ptr(), scale.data_ptr(), 0, rows, k,
                                                None, x.data_ptr(), _DT[x.dtype], acc.data_ptr(), _stream(q)))
    e2, x2 = acc.cpu().tolist()
    return float((e2 / x2) ** 0.5) if x2 > 0 else 0.0


def gemm_nvfp4(a: torch.Tensor, a_sf: torch.Tensor, a_scale: torch.Tensor, b: torch.Tensor, b_sf: torch.Tensor,
               b_scale: torch.Tensor, bias: torch.Tensor | None = None, epilogue: str | None = None,
               return_acc: bool = False, out: torch.Tensor | None = None):
    """bf16(acc * a_scale[m] * b_scale + bias[n]) for NVFP4 a [M, K/2] and b [N, K/2]."""
    a = _cuda2d(a, "a")
    b = _cuda2d(b, "b")
    if a.dtype != torch.uint8 or b.dtype != torch.uint8:
        raise TypeError("a and b must be uint8 (packed E2M1)")
    m, k = a.shape[0], a.shape[1] * 2
    n = b.shape[0]
    if b.shape[1] * 2 != k:
        raise ValueError(f"K mismatch: a {tuple(a.shape)} vs b {tuple(b.shape)}")
    if epilogue not in _EPI:
        raise ValueError(f"epilogue must be one of {sorted(str(e) for e in _EPI)}")
    dev = a.device
    if a_sf.numel() < _rows_pad(m) * (k // 16) or b_sf.numel() != n * (k // 16):
        raise ValueError("block-scale tensors have the wrong size")
    a_scale = _vec(a_scale, m, torch.float32, dev, "a_scale")
    b_scale = _vec(b_scale, 1, torch.float32, dev, "b_scale")
    bias = _vec(bias, n, torch.bfloat16, dev, "bias")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    acc = torch.empty((m, n), dtype=torch.float32, device=dev) if return_acc else None
    with torch.cuda.device(dev):
        nat.check(nat.load().slim_gemm_nvfp4(a.data_ptr(), a_sf.contiguous().data_ptr(), a_scale.data_ptr(),
                                             b.data_ptr(), b_sf.contiguous().data_ptr(), b_scale.data_ptr(),
                                             _ptr(bias), out.data_ptr(), _ptr(acc), m, n, k, _EPI[epilogue],
                                             _stream(a)))
    return (out, acc) if return_acc else out


def nvfp4_linear(x: torch.Tensor, qweight: torch.Tensor, block_scale: torch.Tensor, tensor_scale: torch.Tensor,
                 bias: torch.Tensor | None = None, rotate: bool = False, epilogue: str | None = None,
                 out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """NVFP4 linear on the checkpoint tensors of slimdit/nvfp4.py (weight, weight_scale,
    weight_scale_2): x [..., K] is quantised per token to NVFP4 (optionally after the
    group-256 rotation, for weights packed from rotated rows), then the block-scaled FP4 GEMM."""
    nat.require_cuda()
    if not x.is_cuda:
        raise TypeError("x must be a CUDA tensor")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported activation dtype {x.dtype}")
    qweight = _cuda2d(qweight, "qweight")
    k = x.shape[-1]
    n = qweight.shape[0]
    if qweight.shape[1] * 2 != k:
        raise ValueError(f"in_features mismatch: x [..., {k}] vs packed weight {tuple(qweight.shape)}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k).contiguous()
    m = x2.shape[0]
    dev = x2.device
    ts = _vec(tensor_scale, 1, torch.float32, dev, "tensor_scale")
    b = _vec(bias, n, torch.bfloat16, dev, "bias")
    bs = block_scale.to(dev).contiguous()
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    xq = torch.empty((m, k // 2), dtype=torch.uint8, device=dev)
    xsf = torch.empty((_rows_pad(m), k // 16), dtype=torch.uint8, device=dev)
    xs = torch.empty((m,), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        nat.check(nat.load().slim_nvfp4_linear(x2.data_ptr(), _DT[x2.dtype], qweight.data_ptr(), bs.data_ptr(),
                                               ts.data_ptr(), _ptr(b), out.data_ptr(), xq.data_ptr(), xsf.data_ptr(),
                                               xs.data_ptr(), m, n, k, int(bool(rotate)), _EPI[epilogue], _stream(x2)))
    out = out.reshape(*lead, n)
    return out if out_dtype == torch.bfloat16 else out.to(out_dtype)
