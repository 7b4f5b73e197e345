#!/usr/bin/env python
"""Benchmark of the convrot W8A8 linear on B200.

Workload (one "step"): the single convrot linear at the QKV shape — X bf16 [32768, 5120]
(Student-t(4) x 0.5, 16 outlier channels x30), W int8 [15360, 5120] pre-rotated codes with
fp32 row scales (converted by this library's reference-order converter from N(0, 0.02)
weights with outlier channels x50), bf16 bias [15360]. One step = per-token rotate +
quantise of X in the reference's order (the certified kernel: codes and scales identical to
the reference's rotate() + int8.py math) + tcgen05 INT8 GEMM with the dequant/bias epilogue
-> bf16 [32768, 15360]. Metric: int8 TOPS (2*M*N*K per step). The line also counts, on the
timed input, the codes and scales that the butterfly order alone would change.

Each secondary workload (config-2 FFN pair, real MiniMax-H3 shapes, NVFP4 up-projection,
converter kernels, attention, converter end to end) prints its own JSON line before the main
line; the main line (last) carries a compact summary of them.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU, each rank its own 32768-token batch with the
weights replicated (token rows are independent: no collective on the data path), so the
scaling is weak; `value` is the aggregate over ranks divided by the slowest rank's time.

--impl reference times the CPU restatement of the same linear (the reference's rotation,
np.matmul of the grouped rows with H^T, its per-row quantisation math + torch's CPU int8 GEMM)
on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "viggle-animate-workflow_b200"
for _p in (str(PKG), str(ROOT), str(ROOT / "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

M, N, K = 32768, 15360, 5120
OPS_PER_STEP = 2.0 * M * N * K
METRIC = "convrot INT8 linear TOPS (QKV shape, 32768x15360x5120)"
NOMINAL_I8_TOPS = 4500.0


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the FFN and converter measurements")
    ap.add_argument("--secondary-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU work in the cpu_baseline sample")
    ap.add_argument("--profile-case", choices=["nvfp4", "attn", "rotate", "actquant", "hidquant"], default=None,
                    help="run only a small case of one workload (for ncu captures; prints no bench line)")
    ap.add_argument("--tokens", type=int, default=16384, help="token rows of the --profile-case run")
    ap.add_argument("--heads", type=int, default=4, help="attention heads of the --profile-case attn run")
    ap.add_argument("--convert-blocks", type=int, default=4,
                    help="MiniMax-H3 blocks in the end-to-end converter line (0 skips it)")
    return ap.parse_args(argv)


def env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:  # noqa: BLE001
            pass
    return {}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples; only those taken inside [mark_start, mark_end] count."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.5)

    def mark_start(self):
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        self.t1 = datetime.datetime.now()

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.tmp.flush()
        rows = [line.split(",") for line in Path(self.tmp.name).read_text().splitlines() if line.strip()]
        os.unlink(self.tmp.name)
        sm, mx, power, reasons = [], 0.0, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        parsed = []
        for r in rows:
            try:
                r = [c.strip() for c in r]
                parsed.append((datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f"), r))
            except (ValueError, IndexError):
                continue
        inside = [(ts, r) for ts, r in parsed if self.t0 is None or self.t0 <= ts <= self.t1]
        in_window = bool(inside)
        if not inside and parsed and self.t0 is not None:
            # a timed region shorter than the 100 ms sampling period: the samples either side of it
            before = [x for x in parsed if x[0] < self.t0]
            after = [x for x in parsed if x[0] > self.t1]
            inside = before[-1:] + after[:1]
        for ts, r in inside:
            try:
                sm.append(float(r[2]))
                mx = max(mx, float(r[3]))
                power.append(float(r[4]))
                for name, val in zip(names, r[6:10]):
                    if val.lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": float(statistics.median(sm)), "sm_min_mhz": min(sm), "sm_max_mhz": mx,
                "power_w_median": float(statistics.median(power)) if power else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "inside the timed region" if in_window else "nearest samples around a short timed region"}


# ----------------------------------------------------------------------------- inputs
def make_inputs(torch, dev, seed: int = 0):
    """Synthetic tensors of the QKV linear (32768 x 15360 x 5120) generated on the device (same
    distributions as tests/synthetic.py)."""
    from slimdit import ops

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    z = torch.randn((M, K), generator=g, device=dev, dtype=torch.float32)
    chi2 = torch._standard_gamma(torch.full((M, K), 2.0, device=dev), generator=g) * 2.0  # Chi2(4)
    x = z / torch.sqrt(chi2 / 4.0) * 0.5
    del z, chi2
    chans = torch.randperm(K, generator=g, device=dev)[:16]
    x[:, chans] *= 30.0
    x = x.to(torch.bfloat16)
    w = torch.randn((N, K), generator=g, device=dev, dtype=torch.float32) * 0.02
    wch = torch.randperm(K, generator=g, device=dev)[:5]
    w[:, wch] *= 50.0
    qw, sw = ops.rotate_quant(w.to(torch.bfloat16), order="reference")
    bias = (torch.randn((N,), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    torch.cuda.synchronize(dev)
    return x, qw, sw.reshape(-1).contiguous(), bias


# ----------------------------------------------------------------------------- CPU baseline
def cpu_linear_sample(rows: int, seed: int = 0):
    """CPU restatement of the convrot linear on `rows` tokens of the QKV linear (K 5120, N 15360):
    the reference's rotation (np.matmul of the grouped rows with H^T, slimdit/hadamard.py:56-58,
    numpy/OpenBLAS on all host threads) + its per-row quantisation math (slimdit/int8.py:49-51) +
    torch's CPU int8 GEMM + fp32 dequant. Returns (seconds, threads)."""
    import numpy as np
    import torch

    import oracle
    import synthetic

    x = synthetic.activations(rows, K, seed=seed)
    rng = np.random.default_rng(seed)
    qw = torch.from_numpy(rng.integers(-127, 128, size=(N, K), dtype=np.int8))
    sw = torch.from_numpy((rng.random(N, dtype=np.float32) * 1e-3).astype(np.float32))
    t0 = time.perf_counter()
    h = oracle.build_hadamard(256)
    rot = np.matmul(x.reshape(rows, K // 256, 256), h.T).reshape(rows, K)
    qx, sx = oracle.quantize_rows(rot)
    acc = torch._int_mm(torch.from_numpy(qx), qw.t())
    y = (acc.float() * torch.from_numpy(sx) * sw[None, :]).to(torch.bfloat16)
    dt = time.perf_counter() - t0
    del y
    return dt, torch.get_num_threads()


def cpu_baseline(target_seconds: float) -> dict:
    rows = 256
    dt, _ = cpu_linear_sample(rows)
    rows = int(max(256, min(16384, rows * target_seconds / max(dt, 1e-3) / 2)))
    rows -= rows % 256
    total_t, total_rows, threads = 0.0, 0, 1
    while total_t < target_seconds * 0.5 or total_rows == 0:
        dt, threads = cpu_linear_sample(rows, seed=total_rows + 1)
        total_t += dt
        total_rows += rows
    value = 2.0 * total_rows * N * K / total_t / 1e12
    return {"value": round(value, 4), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{total_rows} tokens in chunks of {rows} through the 15360x5120 linear "
                      f"(the reference's np.matmul rotation + int8.py quantisation, torch CPU int8 GEMM), "
                      f"{total_t:.1f} s of CPU time"}


def run_reference(args) -> int:
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    for _ in range(max(1, args.warmup)):
        cpu_linear_sample(256)
    times, rows = [], 512
    threads = 1
    for s in range(args.steps):
        dt, threads = cpu_linear_sample(rows, seed=s + 1)
        times.append(dt)
    tot = sum(times)
    value = 2.0 * rows * N * K * args.steps / tot / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * tot / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "convrot linear 32768x15360x5120 (QKV), CPU sample of 512 tokens per step",
                   "M": M, "N": N, "K": K, "sample_rows_per_step": rows},
        "cpu_baseline": {"value": round(value, 4), "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": f"{rows} tokens per step x {args.steps} steps"},
        "e2e": {"value": round(value, 4), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ----------------------------------------------------------------------------- attention
ATTN_S, ATTN_H, ATTN_D = 30026, 56, 128  # MiniMax-H3 at 124 frames (attention_triton.py:19)


def attention_cpu_sample(target_seconds: float) -> dict:
    """The oracle's restatement of the same attention on a bounded slice of the workload: a few
    query rows of one head against all 30026 keys (numpy on the host cores)."""
    import numpy as np

    import oracle
    import oracle.attention as oa

    rng = np.random.default_rng(0)
    qkv = oracle.bf16_round((rng.standard_normal((ATTN_S, 3 * ATTN_D)) * 0.5).astype(np.float32))
    q, k, v = oa.split_packed(qkv, 1, ATTN_D)
    q8, qs = oa.quant_qk(q, True)
    k8, ks = oa.quant_qk(k, True)
    v8, amax = oa.quant_v(v)
    scale = oa.attn_scale(ATTN_D, True)
    rows, done, t_total = 64, 0, 0.0
    while t_total < target_seconds and done < ATTN_S:
        t0 = time.perf_counter()
        oa.flash(q8[done:done + rows], qs[done:done + rows], k8, ks, v8, amax, scale)
        t_total += time.perf_counter() - t0
        done += rows
    ops = 4.0 * done * ATTN_S * ATTN_D
    return {"value": round(ops / t_total / 1e12, 5), "unit": "TOPS", "kind": "port", "cores": os.cpu_count(),
            "sample": f"{done} query rows of 1 head x {ATTN_S} keys through the oracle's numpy flash "
                      f"restatement, {t_total:.1f} s"}


def run_attention(torch, dev, lib, world: int, rank: int, steps: int, barrier, reduce_max) -> dict:
    """S=30026 tokens, 56 heads of 128: quantise q/k (int8, rotated) and v (E4M3) from the packed
    bf16 buffer, then the tcgen05 flash kernel; heads split over the ranks (strong scaling), the V
    amax all-reduced so every rank uses the global scale."""
    from slimdit import attention

    g = torch.Generator(device=dev)
    g.manual_seed(7)
    qkv = (torch.randn((ATTN_S, 3 * ATTN_H * ATTN_D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    hl = ATTN_H // world
    out = torch.empty((ATTN_S, hl * ATTN_D), dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev)
    for _ in range(2):
        attention.attention_heads(qkv, ATTN_H, rank, world, out=out)
    torch.cuda.synchronize(dev)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n = max(1, min(steps, 5))
    e0.record(st)
    for _ in range(n):
        attention.attention_heads(qkv, ATTN_H, rank, world, out=out)
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms = reduce_max(e0.elapsed_time(e1) / n)
    # the flash kernel alone on this rank's quantised heads
    seq_pad = (ATTN_S + 127) // 128 * 128
    ops = attention.quantized_operands(qkv[:, :], ATTN_H, rotate=True) if world == 1 else None
    flash_ms = None
    if ops is not None:
        scale = attention.attn_scale(ATTN_D, True)
        attention.attention_quantized(ops, ATTN_S, ATTN_H, scale, out=out)
        torch.cuda.synchronize(dev)
        e0.record(st)
        for _ in range(n):
            attention.attention_quantized(ops, ATTN_S, ATTN_H, scale, out=out)
        e1.record(st)
        torch.cuda.synchronize(dev)
        flash_ms = e0.elapsed_time(e1) / n
        del ops
    total_ops = 4.0 * ATTN_S * ATTN_S * ATTN_H * ATTN_D  # QK^T and PV, 2 ops per multiply-add
    peak = float(measured_peaks().get("bf16_tflops", 1590.0)) * 2.0  # dense INT8/FP8 rate = 2x bf16 (burst)
    res = {"workload": f"packed qkv [{ATTN_S}, 3x{ATTN_H}x{ATTN_D}] bf16 -> int8 q/k (rotated) + E4M3 v -> "
                       f"flash attention, heads split {world} ways, V amax all-reduced",
           "ms_per_step": round(ms, 3), "value": round(total_ops / (ms * 1e-3) / 1e12, 1), "unit": "TOPS",
           "scaling": "strong", "steps": n, "seq_pad": seq_pad,
           "reference_published_ms": {"value": 74.1, "hardware": "RTX 5090", "source": "attention_triton.py:21"}}
    if flash_ms is not None:
        res["flash_ms"] = round(flash_ms, 3)
        res["tensor_frac_of_int8_peak"] = round(total_ops / (flash_ms * 1e-3) / 1e12 / peak, 3)
        res["peak_tops"] = round(peak, 1)
    return res


# ----------------------------------------------------------------------------- converter end to end
def run_convert_e2e(torch, dev, blocks: int) -> dict:
    """The whole converter on real-shape shards: `blocks` MiniMax-H3 blocks (hidden 5120, FFN
    13824) plus the global tensors as bf16 safetensors in a temporary directory (random
    N(0, 0.02) weights drawn on the GPU), converted twice: ops one at a time, then pipelined
    (reads, GPU work and writes overlapped); the two files must be byte-identical."""
    import contextlib
    import hashlib
    import shutil

    import numpy as np

    import synthetic
    from slimdit.convert import convert

    work = Path(tempfile.mkdtemp(prefix="slim_convert_e2e_"))
    try:
        src = work / "official"
        src.mkdir()
        shapes = synthetic.official_shapes(blocks, 5120, 13824, 256)
        g = torch.Generator(device=dev)
        g.manual_seed(3)
        names = sorted(shapes)
        per = (len(names) + 1) // 2
        src_bytes = 0
        for s_i in range(2):
            part = {}
            for name in names[s_i * per:(s_i + 1) * per]:
                if name == "rope.inv_freq":
                    part[name] = (1.0 / (10000.0 ** (np.arange(16, dtype=np.float32) / 16))).astype(np.float32)
                else:
                    t = (torch.randn(shapes[name], generator=g, device=dev) * 0.02).to(torch.bfloat16)
                    part[name] = t.view(torch.int16).cpu().numpy().view(np.uint16)
                src_bytes += part[name].nbytes
            synthetic._write_safetensors(src / f"diffusion_pytorch_model-{s_i + 1:05d}-of-00002.safetensors", part)
            del part
        res = {"workload": f"{blocks} MiniMax-H3 blocks (hidden 5120, FFN 13824) + global tensors: bf16 shards -> "
                           f"adaLN curve + INT8 convrot file, rank 8, grid 1025, error report on",
               "source_gb": round(src_bytes / 1e9, 3), "unit": "GB/s", "source": "page-cache resident shards"}
        digests = {}
        # each mode twice: the first run in a process pays pinned allocations and library set-up
        for mode in ("sequential", "pipelined"):
            for attempt in ("cold", "warm"):
                out = work / f"{mode}.safetensors"
                with contextlib.redirect_stdout(sys.stderr):
                    t0 = time.perf_counter()
                    convert(src, out, rank=8, grid=1025, pipeline=(mode == "pipelined"))
                    dt = time.perf_counter() - t0
                res[f"{mode}_s" if attempt == "warm" else f"{mode}_cold_s"] = round(dt, 3)
                h = hashlib.sha256()
                with out.open("rb") as fh:
                    for chunk in iter(lambda: fh.read(1 << 24), b""):
                        h.update(chunk)
                digests[f"{mode}/{attempt}"] = h.hexdigest()
                res["output_gb"] = round(out.stat().st_size / 1e9, 3)
                out.unlink()
        res["identical"] = len(set(digests.values())) == 1
        res["value"] = round(src_bytes / 1e9 / res["pipelined_s"], 3)
        res["sequential_gbs"] = round(src_bytes / 1e9 / res["sequential_s"], 3)
        return res
    finally:
        shutil.rmtree(work, ignore_errors=True)


# ----------------------------------------------------------------------------- secondary workloads
FFN_TOKENS, FFN_H, FFN_F = 115200, 5120, 13824
CONVERT_BLOCKS = 40
CONVERT_SHAPES = [(15360, 5120), (5120, 5120), (13824, 5120), (5120, 13824)]  # qkv, out, fc1, fc2


def run_secondary(torch, dev, lib, world: int, rank: int, steps: int, barrier, reduce_max) -> dict:
    """The DiT FFN pair (115200 tokens row-sharded over the ranks: strong scaling), the
    MiniMax-H3 linears, the NVFP4 up-projection, and the converter's per-linear kernels over 40
    blocks (blocks split over the ranks)."""
    from slimdit import _native, ops

    out: dict = {}
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    # ---- DiT FFN pair: up-proj -> GELU-tanh -> rotate + requant -> down-proj
    m = (FFN_TOKENS + world - 1) // world
    g = torch.Generator(device=dev)
    g.manual_seed(100 + rank)
    x = (torch.randn((m, FFN_H), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    wu = (torch.randn((FFN_F, FFN_H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wd = (torch.randn((FFN_H, FFN_F), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    qu, su = ops.rotate_quant(wu, order="reference")
    qd, sd = ops.rotate_quant(wd, order="reference")
    su, sd = su.reshape(-1).contiguous(), sd.reshape(-1).contiguous()
    del wu, wd
    xq = torch.empty((m, FFN_H), dtype=torch.int8, device=dev)
    sx = torch.empty((m,), dtype=torch.float32, device=dev)
    h = torch.empty((m, FFN_F), dtype=torch.bfloat16, device=dev)
    hq = torch.empty((m, FFN_F), dtype=torch.int8, device=dev)
    sh = torch.empty((m,), dtype=torch.float32, device=dev)
    y = torch.empty((m, FFN_H), dtype=torch.bfloat16, device=dev)

    def ffn_step():
        _native.check(lib.slim_ffn_i8(x.data_ptr(), _native.BF16, qu.data_ptr(), su.data_ptr(), None, qd.data_ptr(),
                                      sd.data_ptr(), None, y.data_ptr(), xq.data_ptr(), sx.data_ptr(), h.data_ptr(),
                                      hq.data_ptr(), sh.data_ptr(), m, FFN_H, FFN_F, _native.EPI_GELU_TANH, sp))

    for _ in range(3):
        ffn_step()
    torch.cuda.synchronize(dev)
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        ffn_step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = reduce_max(a.elapsed_time(b) / steps)
    ops_total = 2 * 2.0 * FFN_TOKENS * FFN_H * FFN_F
    out["ffn_pair"] = {"workload": "115200 tokens, 5120 -> 13824 (GELU-tanh, requant) -> 5120, int8 convrot",
                       "tokens_per_gpu": m, "ms_per_step": round(ms, 4), "value": round(ops_total / (ms * 1e-3) / 1e12, 1),
                       "unit": "TOPS", "scaling": "strong", "steps": steps}
    del xq, sx, h, hq, sh, y, qu, qd
    torch.cuda.empty_cache()

    # ---- the real MiniMax-H3 linears (tools/bench_int8.py:23-28) at the same token count:
    # qkv, out_proj, and the SwiGLU FFN (fc1 with the fused SwiGLU epilogue, requant, fc2)
    mm = (FFN_TOKENS + world - 1) // world
    xh = (torch.randn((mm, 5376), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    xo = (torch.randn((mm, 7168), generator=g, device=dev) * 0.5).to(torch.bfloat16)

    def qweight(n, k):
        w = (torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        q, s_ = ops.rotate_quant(w, order="butterfly")
        return q, s_.reshape(-1).contiguous()

    shapes = {"qkv": (21504, 5376, xh), "out_proj": (5376, 7168, xo)}
    res = {}
    for name, (n_, k_, xin) in shapes.items():
        q, s_ = qweight(n_, k_)
        for _ in range(2):
            ops.int8_linear(xin, q, s_)
        torch.cuda.synchronize(dev)
        barrier()
        a.record(stream)
        for _ in range(steps):
            ops.int8_linear(xin, q, s_)
        b.record(stream)
        torch.cuda.synchronize(dev)
        ms = reduce_max(a.elapsed_time(b) / steps)
        res[name] = {"M": mm, "N": n_, "K": k_, "ms": round(ms, 4),
                     "TOPS": round(world * 2.0 * mm * n_ * k_ / (ms * 1e-3) / 1e12, 1)}
        del q, s_
    q1, s1 = qweight(28672, 5376)
    q1, s1, _ = ops.swiglu_interleave(q1, s1)
    q2, s2 = qweight(5376, 14336)
    for _ in range(2):
        ops.ffn_swiglu_int8(xh, q1, s1, q2, s2)
    torch.cuda.synchronize(dev)
    barrier()
    a.record(stream)
    for _ in range(steps):
        ops.ffn_swiglu_int8(xh, q1, s1, q2, s2)
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = reduce_max(a.elapsed_time(b) / steps)
    ffn_ops = 2.0 * FFN_TOKENS * 28672 * 5376 + 2.0 * FFN_TOKENS * 5376 * 14336
    res["ffn_swiglu"] = {"M": mm, "fc1": [28672, 5376], "fc2": [5376, 14336], "ms": round(ms, 4),
                         "TOPS": round(ffn_ops / (ms * 1e-3) / 1e12, 1)}
    # the layer's linears together: their ops over the sum of their times
    layer_ops = 2.0 * FFN_TOKENS * (21504 * 5376 + 5376 * 7168) + ffn_ops
    layer_ms = sum(v["ms"] for v in res.values())
    out["minimax_h3"] = {"workload": f"MiniMax-H3 linears at {FFN_TOKENS} tokens (split over the ranks): qkv, "
                                     "out_proj, and the FFN fc1 -> fused SwiGLU -> rotate+requant -> fc2",
                         "shapes": res, "ms_per_step": round(layer_ms, 4),
                         "value": round(layer_ops / (layer_ms * 1e-3) / 1e12, 1), "unit": "TOPS",
                         "scaling": "strong", "steps": steps}
    del xh, xo, q1, s1, q2, s2
    torch.cuda.empty_cache()

    # ---- NVFP4 up-proj (rotate + per-token NVFP4 of x, block-scaled FP4 GEMM)
    wu = (torch.randn((FFN_F, FFN_H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    pw, pws, pwg = ops.nvfp4_pack(wu)
    del wu
    pad = (m + 127) // 128 * 128
    xq4 = torch.empty((m, FFN_H // 2), dtype=torch.uint8, device=dev)
    xsf4 = torch.empty((pad, FFN_H // 16), dtype=torch.uint8, device=dev)
    xs4 = torch.empty((m,), dtype=torch.float32, device=dev)
    h4 = torch.empty((m, FFN_F), dtype=torch.bfloat16, device=dev)

    def fp4_quant():
        _native.check(lib.slim_quant_nvfp4_act(x.data_ptr(), _native.BF16, m, FFN_H, 1, xq4.data_ptr(), xsf4.data_ptr(),
                                               xs4.data_ptr(), sp))

    def fp4_gemm():
        _native.check(lib.slim_gemm_nvfp4(xq4.data_ptr(), xsf4.data_ptr(), xs4.data_ptr(), pw.data_ptr(),
                                          pws.data_ptr(), pwg.data_ptr(), None, h4.data_ptr(), None, m, FFN_F, FFN_H,
                                          _native.EPI_SCALE_BIAS, sp))

    for _ in range(3):
        fp4_quant()
        fp4_gemm()
    torch.cuda.synchronize(dev)
    barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    gq = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    evs[0].record(stream)
    for i in range(steps):
        fp4_quant()
        gq[i].record(stream)
        fp4_gemm()
        evs[i + 1].record(stream)
    torch.cuda.synchronize(dev)
    ms = reduce_max(evs[0].elapsed_time(evs[-1]) / steps)
    gemm_ms = reduce_max(sum(gq[i].elapsed_time(evs[i + 1]) for i in range(steps)) / steps)
    ops_up = 2.0 * FFN_TOKENS * FFN_H * FFN_F
    out["nvfp4_up_proj"] = {
        "workload": "115200 tokens x 5120 -> 13824, x rotated + per-token NVFP4, W NVFP4 (E2M1 + UE4M3/16 + fp32)",
        "tokens_per_gpu": m, "ms_per_step": round(ms, 4), "gemm_ms": round(gemm_ms, 4),
        "value": round(ops_up / (ms * 1e-3) / 1e12, 1), "gemm_value": round(ops_up / (gemm_ms * 1e-3) / 1e12, 1),
        "unit": "TOPS", "scaling": "strong", "steps": steps}
    del x, xq4, xsf4, xs4, h4, pw, pws, pwg
    torch.cuda.empty_cache()

    # ---- attention: the in-place INT8/FP8 override at the production geometry (heads split over ranks)
    out["attention_packed"] = run_attention(torch, dev, lib, world, rank, steps, barrier, reduce_max)
    torch.cuda.empty_cache()

    # ---- converter kernels (rotate + per-row INT8 of each block linear)
    my_blocks = len([i for i in range(CONVERT_BLOCKS) if i % world == rank])
    ws = [(torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16) for shape in CONVERT_SHAPES]
    qs = [torch.empty(shape, dtype=torch.int8, device=dev) for shape in CONVERT_SHAPES]
    ss = [torch.empty((shape[0],), dtype=torch.float32, device=dev) for shape in CONVERT_SHAPES]
    block_bytes = sum(r * k * 3 + r * 4 for r, k in CONVERT_SHAPES)
    for order_name, order in (("reference_order", _native.ORDER_REFERENCE), ("butterfly_order", _native.ORDER_BUTTERFLY)):
        def block(order=order):
            for w, q, sc, (r, k) in zip(ws, qs, ss, CONVERT_SHAPES):
                _native.check(lib.slim_rotate_quant_i8(w.data_ptr(), _native.BF16, r, k, 256, order, q.data_ptr(),
                                                       sc.data_ptr(), None, sp))
        block()
        torch.cuda.synchronize(dev)
        barrier()
        a.record(stream)
        for _ in range(my_blocks):
            block()
        b.record(stream)
        torch.cuda.synchronize(dev)
        ms = reduce_max(a.elapsed_time(b))
        total = CONVERT_BLOCKS * block_bytes
        out[f"convert_{order_name}"] = {
            "workload": "40 blocks x {qkv 15360x5120, out 5120x5120, fc1 13824x5120, fc2 5120x13824} bf16 -> int8 + scales",
            "ms_total": round(ms, 3), "value": round(total / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "algorithmic_bytes": total, "scaling": "strong"}
    # NVFP4 weights: per-tensor amax pass + pack (bf16 read twice, 0.5 + 1/16 B written per element)
    del qs, ss
    pq = [torch.empty((r, k // 2), dtype=torch.uint8, device=dev) for r, k in CONVERT_SHAPES]
    psf = [torch.empty((r, k // 16), dtype=torch.uint8, device=dev) for r, k in CONVERT_SHAPES]
    pts = torch.empty((len(CONVERT_SHAPES),), dtype=torch.float32, device=dev)

    def block_fp4():
        for i, (w, (r, k)) in enumerate(zip(ws, CONVERT_SHAPES)):
            _native.check(lib.slim_nvfp4_pack(w.data_ptr(), _native.BF16, r, k, pq[i].data_ptr(), psf[i].data_ptr(),
                                              pts[i:].data_ptr(), sp))

    block_fp4()
    torch.cuda.synchronize(dev)
    barrier()
    a.record(stream)
    for _ in range(my_blocks):
        block_fp4()
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = reduce_max(a.elapsed_time(b))
    elems = CONVERT_BLOCKS * sum(r * k for r, k in CONVERT_SHAPES)
    fp4_bytes = elems * (2 + 0.5 + 1 / 16)
    out["convert_nvfp4"] = {
        "workload": "40 blocks x {qkv, out, fc1, fc2} bf16 -> NVFP4 (per-tensor amax pass + pack)",
        "ms_total": round(ms, 3), "value": round(fp4_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
        "algorithmic_bytes": int(fp4_bytes), "bytes_moved_two_pass": int(fp4_bytes + 2 * elems), "scaling": "strong"}
    del ws, pq, psf, pts
    torch.cuda.empty_cache()

    # ---- output-column split (N > 1 only): the QKV linear (32768 x 15360 x 5120), weight rows
    # split over the ranks, x replicated, column blocks all-gathered over NVLink (NCCL), "blocks" layout
    if world > 1:
        import torch.distributed as dist

        from slimdit import colsplit

        xs, qw, sw, bias = make_inputs(torch, dev, seed=200)
        q_s, s_s, b_s = colsplit.shard_weight(qw, sw, bias, rank, world)
        del qw, sw, bias
        nl = N // world
        y_loc = torch.empty((M, nl), dtype=torch.bfloat16, device=dev)
        blocks = torch.empty((world * M, nl), dtype=torch.bfloat16, device=dev)
        xq = torch.empty((M, K), dtype=torch.int8, device=dev)
        sx = torch.empty((M,), dtype=torch.float32, device=dev)

        def cs_step(ev_mid=None):
            _native.check(lib.slim_int8_linear(xs.data_ptr(), _native.BF16, q_s.data_ptr(), s_s.data_ptr(),
                                               b_s.data_ptr(), y_loc.data_ptr(), xq.data_ptr(), sx.data_ptr(), M, nl,
                                               K, 256, _native.EPI_SCALE_BIAS, sp))
            if ev_mid is not None:
                ev_mid.record(stream)
            dist.all_gather_into_tensor(blocks, y_loc)

        for _ in range(3):
            cs_step()
        torch.cuda.synchronize(dev)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        mids = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        e0.record(stream)
        for i in range(steps):
            cs_step(mids[i])
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
        ms = reduce_max(e0.elapsed_time(ends[-1]) / steps)
        gather_ms = reduce_max(sum(mids[i].elapsed_time(ends[i]) for i in range(steps)) / steps)
        out["colsplit_linear"] = {
            "workload": f"QKV linear 32768 x 15360 x 5120, W rows split {world} ways, x replicated, NCCL all-gather of "
                        f"[{M},{nl}] bf16 blocks ([G,M,N/G] layout)",
            "ms_per_step": round(ms, 4), "allgather_ms": round(gather_ms, 4),
            "value": round(OPS_PER_STEP / (ms * 1e-3) / 1e12, 1), "unit": "TOPS", "scaling": "strong",
            "allgather_busbw_gbs": round((world - 1) * M * nl * 2 / (gather_ms * 1e-3) / 1e9, 1), "steps": steps}
        del y_loc, blocks, xq, sx
        torch.cuda.empty_cache()
        # the same split with the all-gather inside the GEMM epilogue (peer stores over NVLink)
        for mode, layout, what in (
                ("dma", "blocks", "[G,M,N/G] blocks like NCCL's; 4096-row chunks, each pushed to every peer as one "
                                  "contiguous copy by the copy engines while the next chunk computes"),
                ("dma", "rows", "[M,N]; 4096-row chunks pushed as 2-D copies while the next chunk computes"),
                ("stores", "rows", "[M,N]; the GEMM epilogue stores each tile into every peer's output")):
            fused = colsplit.PeerColumnSplit(M, N, K, device=dev, mode=mode, layout=layout)
            for _ in range(3):
                fused(xs, q_s, s_s, b_s)
            torch.cuda.synchronize(dev)
            barrier()
            e0.record(stream)
            for i in range(steps):
                fused(xs, q_s, s_s, b_s)
            ends[0].record(stream)
            torch.cuda.synchronize(dev)
            ms = reduce_max(e0.elapsed_time(ends[0]) / steps)
            out[f"colsplit_linear_peer_{mode}_{layout}"] = {
                "workload": f"QKV linear 32768 x 15360 x 5120, W rows split {world} ways, x replicated, written into all {world} "
                            f"GPUs' outputs over NVLink (CUDA IPC mappings), M={M} N={N}: {what}",
                "ms_per_step": round(ms, 4), "value": round(OPS_PER_STEP / (ms * 1e-3) / 1e12, 1), "unit": "TOPS",
                "scaling": "strong", "nvlink_bytes_out_per_gpu": (world - 1) * M * nl * 2, "steps": steps}
            fused.close()
            del fused
        del xs, q_s, s_s, b_s
        torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- profiling cases
def run_profile_quant(args, hidden: bool) -> int:
    """The linears' activation quantiser (reference order, certified kernel) alone on `--tokens`
    rows: config-1 activations (K 5120), or with `hidden` the config-2 FFN hidden (K 13824, GELU-
    tanh of twice the config-1 distribution). Warm-up + `--steps` calls, for ncu captures."""
    import torch

    from slimdit import _native, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    k = 13824 if hidden else K
    g = torch.Generator(device=dev)
    g.manual_seed(12)
    z = torch.randn((args.tokens, k), generator=g, device=dev)
    chi2 = torch._standard_gamma(torch.full((args.tokens, k), 2.0, device=dev), generator=g) * 2.0
    x = z / torch.sqrt(chi2 / 4.0) * 0.5
    del z, chi2
    x[:, torch.randperm(k, generator=g, device=dev)[:16]] *= 30.0
    if hidden:
        x = torch.nn.functional.gelu(2.0 * x, approximate="tanh")
    x = x.to(torch.bfloat16)
    warm = max(1, args.warmup)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for i in range(warm + args.steps):
        if i == warm:
            ev[0].record()
        ops.rotate_quant(x, order="reference")
    ev[1].record()
    torch.cuda.synchronize(dev)
    assert _native.device_error() == 0
    ms = ev[0].elapsed_time(ev[1]) / max(1, args.steps)
    print(json.dumps({"profile_case": "hidden_quant" if hidden else "activation_quant", "rows": args.tokens, "K": k,
                      "steps": args.steps, "ms": round(ms, 4),
                      "GBs": round(args.tokens * (3 * k + 4) / (ms * 1e-3) / 1e9, 1)}))
    return 0


def run_profile_rotate(args) -> int:
    """The reference-order weight rotation + INT8 of one linear (W bf16 [tokens, 5120], the QKV
    linear's 15360 rows by default in captures): warm-up + `--steps` calls, for ncu captures."""
    import torch

    from slimdit import _native, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    w = (torch.randn((args.tokens, 5120), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    warm = max(1, args.warmup)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(warm + args.steps + 1)]
    for i in range(warm + args.steps):
        ev[i].record()
        ops.rotate_quant(w, order="reference")
    ev[-1].record()
    torch.cuda.synchronize(dev)
    assert _native.device_error() == 0
    ms = ev[warm].elapsed_time(ev[-1]) / max(1, args.steps)
    print(json.dumps({"profile_case": "rotate_reference_order", "rows": args.tokens, "K": 5120, "steps": args.steps,
                      "ms": round(ms, 4)}))
    return 0


def run_profile_attn(args) -> int:
    """A small case of the attention (packed qkv [tokens, 3*heads*128]): the quantisers once,
    then warm-up + `--steps` launches of the flash kernel, for ncu captures."""
    import torch

    from slimdit import _native, attention

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s_len, heads = args.tokens, args.heads
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    qkv = (torch.randn((s_len, 3 * heads * ATTN_D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    ops = attention.quantized_operands(qkv, heads)
    scale = attention.attn_scale(ATTN_D, True)
    out = torch.empty((s_len, heads * ATTN_D), dtype=torch.bfloat16, device=dev)
    warm = max(1, args.warmup)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(warm + args.steps + 1)]
    for i in range(warm + args.steps):
        ev[i].record()
        attention.attention_quantized(ops, s_len, heads, scale, out=out)
    ev[-1].record()
    torch.cuda.synchronize(dev)
    assert _native.device_error() == 0
    ms = ev[warm].elapsed_time(ev[-1]) / max(1, args.steps)
    print(json.dumps({"profile_case": "attention", "tokens": s_len, "heads": heads, "steps": args.steps,
                      "flash_ms": round(ms, 4),
                      "flash_tops": round(4.0 * s_len * s_len * heads * ATTN_D / (ms * 1e-3) / 1e12, 1)}))
    return 0


def run_profile_case(args) -> int:
    """A small case of the NVFP4 up-proj (x [tokens, 5120] rotated + per-token
    NVFP4, FP4 GEMM against W [13824, 5120]): warm-up + `--steps` launches of each kernel, for
    ncu captures that must stay a few GB. Prints a JSON line marked "profile_case"."""
    import torch

    from slimdit import _native, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _native.load()
    sp = torch.cuda.current_stream(dev).cuda_stream
    m = args.tokens
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    x = (torch.randn((m, FFN_H), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    w = (torch.randn((FFN_F, FFN_H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    pw, pws, pwg = ops.nvfp4_pack(w)
    xq = torch.empty((m, FFN_H // 2), dtype=torch.uint8, device=dev)
    xsf = torch.empty(((m + 127) // 128 * 128, FFN_H // 16), dtype=torch.uint8, device=dev)
    xs = torch.empty((m,), dtype=torch.float32, device=dev)
    h = torch.empty((m, FFN_F), dtype=torch.bfloat16, device=dev)
    warm = max(3, args.warmup)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(warm + args.steps)]
    for i in range(warm + args.steps):
        ev[i][0].record()
        _native.check(lib.slim_quant_nvfp4_act(x.data_ptr(), _native.BF16, m, FFN_H, 1, xq.data_ptr(), xsf.data_ptr(),
                                               xs.data_ptr(), sp))
        ev[i][1].record()
        _native.check(lib.slim_gemm_nvfp4(xq.data_ptr(), xsf.data_ptr(), xs.data_ptr(), pw.data_ptr(), pws.data_ptr(),
                                          pwg.data_ptr(), None, h.data_ptr(), None, m, FFN_F, FFN_H,
                                          _native.EPI_SCALE_BIAS, sp))
        ev[i][2].record()
    torch.cuda.synchronize(dev)
    assert _native.device_error() == 0
    timed = ev[warm:]
    qms = statistics.mean(e[0].elapsed_time(e[1]) for e in timed) if timed else 0.0
    gms = statistics.mean(e[1].elapsed_time(e[2]) for e in timed) if timed else 0.0
    print(json.dumps({"profile_case": "nvfp4_up_proj", "tokens": m, "steps": args.steps,
                      "quant_ms": round(qms, 4), "gemm_ms": round(gms, 4),
                      "quant_gbs": round((m * FFN_H * 2 + m * FFN_H * 0.5625) / (qms * 1e-3) / 1e9, 1) if qms else None,
                      "gemm_tops": round(2.0 * m * FFN_H * FFN_F / (gms * 1e-3) / 1e12, 1) if gms else None}))
    return 0


# ----------------------------------------------------------------------------- ours
def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    from slimdit import _native

    rank, world, local = env_rank()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = _native.load()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    x, qw, sw, bias = make_inputs(torch, dev, seed=rank)
    xq = torch.empty((M, K), dtype=torch.int8, device=dev)
    sx = torch.empty((M,), dtype=torch.float32, device=dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

    def quant(order=_native.ORDER_REFERENCE):
        # the activation side of slim_int8_linear: reference-order codes (certified kernel)
        _native.check(lib.slim_rotate_quant_i8(x.data_ptr(), _native.BF16, M, K, 256, order,
                                               xq.data_ptr(), sx.data_ptr(), None, sp))

    def gemm():
        _native.check(lib.slim_gemm_i8(xq.data_ptr(), qw.data_ptr(), sx.data_ptr(), sw.data_ptr(), bias.data_ptr(),
                                       out.data_ptr(), None, M, N, K, _native.EPI_SCALE_BIAS, sp))

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, args.warmup)):
        quant()
        gemm()
    torch.cuda.synchronize(dev)
    # activation parity on this input: the butterfly order against the reference order the step
    # uses (outside the timed region), and the butterfly quantiser's own time for comparison
    q_ref, s_ref = xq.clone(), sx.clone()
    quant(_native.ORDER_BUTTERFLY)
    torch.cuda.synchronize(dev)
    parity = {"order_timed": "reference", "rows": M, "K": K,
              "butterfly_codes_differ": int((xq != q_ref).sum().item()),
              "butterfly_code_max_abs_diff": int((xq.int() - q_ref.int()).abs().max().item()),
              "butterfly_scales_differ": int((sx != s_ref).sum().item())}
    bf_a, bf_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    bf_a.record(stream)
    for _ in range(5):
        quant(_native.ORDER_BUTTERFLY)
    bf_b.record(stream)
    torch.cuda.synchronize(dev)
    parity["butterfly_quant_ms"] = round(bf_a.elapsed_time(bf_b) / 5, 4)
    del q_ref, s_ref
    quant()
    torch.cuda.synchronize(dev)
    barrier()

    steps = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(visible.split(",")[local] if visible else local)
    clocks.start()
    launches0 = _native.launch_count()
    torch.cuda.synchronize(dev)
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks.mark_start()
    torch.cuda.nvtx.range_push(f"timed region: {steps} steps")  # for a profiler's timeline
    t_start.record(stream)
    for i in range(steps):
        ev[i][0].record(stream)
        quant()
        ev[i][1].record(stream)
        gemm()
        ev[i][2].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    torch.cuda.nvtx.range_pop()
    clocks.mark_end()
    barrier()
    launches = _native.launch_count() - launches0
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    quant_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    gemm_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)

    # end to end through the public API with host buffers (pinned), copies in the timed region
    e2e = None
    if args.e2e_steps > 0:
        from slimdit import ops

        x_h = x.cpu().pin_memory()
        out_h = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
        x_d = None

        def e2e_step():
            ops.int8_linear_host(x_h, qw, sw, bias=bias, out=out_h)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = a.elapsed_time(b) / args.e2e_steps
        e2e = {"ms": e2e_ms, "h2d": x.numel() * 2, "d2h": M * N * 2}
        del x_h, out_h, x_d

    def reduce_max(v: float) -> float:
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    secondary = None
    if not args.no_secondary:
        secondary = run_secondary(torch, dev, lib, world, rank, args.secondary_steps, barrier, reduce_max)
        if world == 1 and args.convert_blocks > 0:
            secondary["convert_e2e"] = run_convert_e2e(torch, dev, args.convert_blocks)

    # max over ranks
    vals = torch.tensor([total_ms, gemm_ms, quant_ms, e2e["ms"] if e2e else 0.0], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, gemm_ms, quant_ms, e2e_ms = [float(v) for v in vals.cpu()]
    if _native.device_error() != 0:
        raise RuntimeError("device error word set during the benchmark")

    if rank == 0:
        ms_per_step = total_ms / steps
        value = world * OPS_PER_STEP / (ms_per_step * 1e-3) / 1e12
        peaks = measured_peaks()
        # A timed region longer than half a second runs under the power cap: compare with the
        # sustained figure; a short burst with the burst figure.
        sustained = total_ms > 500.0
        key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
        regime = "sustained (seconds-long loop)" if sustained else "burst"
        if key in peaks:
            peak = 2.0 * float(peaks[key])
            peak_src = (f"2 x measured bf16 cuBLAS {regime} (MEASURED_PEAKS.json {key}); "
                        "kind::i8 issues at twice kind::f16's rate")
        else:
            peak = 2.0 * (1400.0 if sustained else 1590.0)
            peak_src = f"2 x fallback bf16 {regime}"
        gemm_tops = OPS_PER_STEP / (gemm_ms * 1e-3) / 1e12
        # DRAM traffic of one GEMM launch is read from the committed summary of an offline ncu
        # capture of the same shape (a profiler cannot run inside this timed benchmark)
        traffic = None
        prof = ROOT / "profiles" / "gemm_i8_pair_qkv_32768x15360x5120.md"
        if prof.exists():
            for ln in prof.read_text().splitlines():
                if ln.startswith("dram_bytes_per_launch:"):
                    traffic = int(ln.split(":", 1)[1])
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TOPS", "n_gpus": world, "steps": steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "convrot W8A8 linear, QKV shape: X bf16 [32768,5120] -> rotate+quant -> "
                                   "int8 GEMM vs W [15360,5120] -> bf16 [32768,15360] (+bias)",
                       "M": M, "N": N, "K": K, "tokens_per_gpu": M, "parallelism": f"token rows x{world}, no collective",
                       "l2": "inputs+outputs 1.5 GB per step > 126 MB L2 (no flush needed)"},
            "roofline": {"bound": "tensor", "kernel": "gemm_i8_pair_kernel (tcgen05 kind::i8, cta_group::2)",
                         "achieved": round(gemm_tops, 2), "peak": round(peak, 1), "unit": "TOPS",
                         "frac": round(gemm_tops / peak, 4), "peak_source": peak_src,
                         "frac_of_nominal_4500": round(gemm_tops / NOMINAL_I8_TOPS, 4), "traffic": traffic,
                         "traffic_source": "offline ncu capture (dram__bytes_read.sum + dram__bytes_write.sum of one "
                                           "launch): profiles/gemm_i8_pair_qkv_32768x15360x5120.md",
                         "avg_launch_ms": round(gemm_ms, 4)},
            "kernels_ms_per_step": {"rotate_quant_reference_order": round(quant_ms, 4), "gemm_i8": round(gemm_ms, 4)},
            "activation_parity": parity,
            "act_quant_gbs": round((M * K * 2 + M * K + M * 4) / (quant_ms * 1e-3) / 1e9, 1),
            "gpu_launches": int(launches),
            "clocks": clk,
        }
        if secondary is not None:
            peak_hbm = float(peaks.get("hbm_gbs", 6650.0))
            for key in ("convert_reference_order", "convert_butterfly_order", "convert_nvfp4"):
                secondary[key]["frac_of_measured_hbm"] = round(secondary[key]["value"] / (world * peak_hbm), 4)
            for key in ("ffn_pair", "minimax_h3"):
                if "value" in secondary.get(key, {}):
                    secondary[key]["frac_of_i8_peak"] = round(secondary[key]["value"] / (world * peak), 4)
            # dense FP4 (kind::mxf4nvf4) issues at four times kind::f16's rate
            fp4_peak = 2.0 * peak
            nv = secondary["nvfp4_up_proj"]
            nv["fp4_peak"] = round(fp4_peak, 1)
            nv["frac_of_fp4_peak"] = round(nv["value"] / (world * fp4_peak), 4)
            nv["gemm_frac_of_fp4_peak"] = round(nv["gemm_value"] / (world * fp4_peak), 4)
            # each secondary workload on its own line (printed below, before this one); this line
            # keeps a compact summary of their headline figures
            summary_keys = ("value", "unit", "ms_per_step", "ms_total", "frac_of_i8_peak", "frac_of_fp4_peak",
                            "gemm_frac_of_fp4_peak", "frac_of_measured_hbm", "tensor_frac_of_int8_peak")
            line["secondary"] = {name: {k: v[k] for k in summary_keys if k in v} for name, v in secondary.items()
                                 if isinstance(v, dict)}
        if e2e is not None:
            line["e2e"] = {"value": round(world * OPS_PER_STEP / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOPS",
                           "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                           "ms_per_step": round(e2e_ms, 3),
                           "api": "slimdit.ops.int8_linear_host: pinned host x and out, H2D / linear / D2H of "
                                  "4096-row chunks overlapped on three streams"}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
            if secondary is not None and "attention_packed" in secondary:
                secondary["attention_packed"]["cpu_baseline"] = attention_cpu_sample(min(args.cpu_seconds, 8.0))
        if secondary is not None:
            for name, v in secondary.items():
                print(json.dumps({"secondary": name, **v} if isinstance(v, dict) else {"secondary": name, "value": v}),
                      flush=True)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    if args.profile_case == "rotate":
        return run_profile_rotate(args)
    if args.profile_case in ("actquant", "hidquant"):
        return run_profile_quant(args, hidden=args.profile_case == "hidquant")
    if args.profile_case == "attn":
        return run_profile_attn(args)
    if args.profile_case:
        return run_profile_case(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
