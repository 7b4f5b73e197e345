"""GPU parity of the tcgen05 INT8 GEMM and the convrot linear.

* INT32 accumulators: bit-exact against exact integer math (oracle.int8_gemm_i32).
* bf16 output: |y - ref| <= 1 bf16 ulp of ref, ref = fp64 dequant (acc * sa * sb + bias).
* GELU epilogue: within 2 bf16 ulp (+ the tanh cancellation term) of GELU(bf16(linear))
  evaluated in fp32 on the CPU.
"""

import numpy as np
import pytest
import torch

import oracle
import synthetic

pytestmark = pytest.mark.gpu


def rand_i8(rng, shape):
    return rng.integers(-127, 128, size=shape, dtype=np.int8)


def check_bf16_within_one_ulp(y_bf16: torch.Tensor, ref: np.ndarray, what: str = "", term: np.ndarray | None = None):
    """|y - ref| <= 1 bf16 ulp(ref) + 2^-21 |term|; term = the acc*sa*sb product whose fp32
    rounding (int->float, scale product, fused multiply-add) matters only where the bias
    cancels it to near zero."""
    y = y_bf16.float().cpu().numpy().astype(np.float64)
    err = np.abs(y - ref)
    ulp = oracle.bf16_ulp(ref)
    if term is not None:
        ulp = ulp + np.abs(term) * 2.0**-21
    bad = err > ulp
    assert not bad.any(), f"{what}: {int(bad.sum())} outputs beyond 1 bf16 ulp; worst {float((err / ulp).max()):.3f} ulp"


@pytest.mark.parametrize("m,n,k", [
    (128, 256, 128),      # one tile, one k-block
    (256, 512, 5120),     # several tiles, config K
    (300, 264, 384),      # ragged M and N tails (N % 256 != 0), 3 k-blocks
    (1, 8, 16),           # minimal: K and N below one tile, TMA zero fill
    (129, 520, 1040),     # K not a multiple of 128
    (1024, 1024, 13824),  # FFN down-proj K
])
def test_gemm_int32_accumulators_bit_exact_and_bf16_epilogue(cuda, m, n, k):
    from slimdit import ops
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a, b = rand_i8(rng, (m, k)), rand_i8(rng, (n, k))
    sa = (rng.random(m, dtype=np.float32) * 0.02 + 1e-3).astype(np.float32)
    sb = (rng.random(n, dtype=np.float32) * 0.002 + 1e-4).astype(np.float32)
    bias = synthetic.bf16_round_f32(rng.standard_normal(n).astype(np.float32) * 0.02)
    at, bt = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    y, acc = ops.gemm_i8(at, bt, torch.from_numpy(sa), torch.from_numpy(sb),
                         torch.from_numpy(bias).to(torch.bfloat16), return_acc=True)
    acc_ref = oracle.int8_gemm_i32(a, b)
    assert np.array_equal(acc.cpu().numpy(), acc_ref)
    check_bf16_within_one_ulp(y, oracle.linear_reference_f64(acc_ref, sa, sb, bias), "scale+bias",
                              term=oracle.linear_reference_f64(acc_ref, sa, sb, None))
    y2 = ops.gemm_i8(at, bt, torch.from_numpy(sa), torch.from_numpy(sb))
    check_bf16_within_one_ulp(y2, oracle.linear_reference_f64(acc_ref, sa, sb, None), "scale only")


def test_gemm_extreme_codes_saturate_nothing(cuda):
    """All -128 / 127 codes at K=13824: |acc| up to 2.26e8 < 2^31 is exact."""
    from slimdit import ops
    m, n, k = 128, 256, 13824
    a = np.full((m, k), -128, np.int8)
    b = np.full((n, k), -128, np.int8)
    b[1::2] = 127
    _, acc = ops.gemm_i8(torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda),
                         torch.ones(m), torch.ones(n), return_acc=True)
    assert np.array_equal(acc.cpu().numpy(), oracle.int8_gemm_i32(a, b))


def test_gemm_gelu_epilogue(cuda):
    from slimdit import ops
    rng = np.random.default_rng(5)
    m, n, k = 256, 512, 1024
    a, b = rand_i8(rng, (m, k)), rand_i8(rng, (n, k))
    sa = np.full(m, 0.01, np.float32)
    sb = (rng.random(n, dtype=np.float32) * 1e-3).astype(np.float32)
    y, acc = ops.gemm_i8(torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda), torch.from_numpy(sa),
                         torch.from_numpy(sb), epilogue="gelu_tanh", return_acc=True)
    acc = acc.cpu().numpy()
    lin = oracle.bf16_round((acc.astype(np.float32) * (sa[:, None] * sb[None, :])).astype(np.float32))
    ref = oracle.gelu_tanh_f32(lin).astype(np.float64)
    yv = y.float().cpu().numpy().astype(np.float64)
    err = np.abs(yv - ref)
    # CUDA tanhf and numpy's float32 tanh may differ by a few fp32 ulp. Near tanh = -1
    # (x below about -3) 0.5*x*(1 + tanh) cancels, so such a difference is an absolute error
    # of ~0.5*|x|*2^-24 per ulp, large relative to the tiny output; elsewhere it can move the
    # bf16 rounding by one step. Tolerance: 2 bf16 ulp + 4 fp32 tanh ulp scaled by |x|.
    tol = 2 * oracle.bf16_ulp(ref) + 4 * 2.0**-24 * np.abs(lin.astype(np.float64))
    assert np.all(err <= tol), float((err / tol).max())


def test_gemm_shape_errors(cuda):
    from slimdit import ops
    a = torch.zeros((4, 64), dtype=torch.int8, device=cuda)
    with pytest.raises(ValueError):
        ops.gemm_i8(a, torch.zeros((12, 64), dtype=torch.int8, device=cuda), torch.ones(4), torch.ones(12))
    with pytest.raises(ValueError):
        ops.gemm_i8(a, torch.zeros((16, 32), dtype=torch.int8, device=cuda), torch.ones(4), torch.ones(16))
    y = ops.gemm_i8(a[:0], torch.zeros((16, 64), dtype=torch.int8, device=cuda), torch.ones(0), torch.ones(16))
    assert y.shape == (0, 16)
    from slimdit import _native
    assert _native.device_error() == 0


@pytest.mark.parametrize("m,n,k", [(256, 768, 5120), (77, 512, 1024), (4096, 1536, 5120)])
def test_int8_linear_end_to_end_vs_oracle(cuda, m, n, k):
    """x bf16 -> rotate + per-token INT8 (the reference's order) -> GEMM -> bf16; weights from
    the reference converter path. Codes bit-exact with the oracle's; output within 1 bf16 ulp of
    the fp64 dequant of those codes."""
    from slimdit import ops
    from slimdit.int8 import quantize_convrot_weight
    x = synthetic.activations(m, k, seed=m + n)
    w = synthetic.weight(n, k, seed=n + k)
    bias = synthetic.bf16_round_f32(np.random.default_rng(1).standard_normal(n).astype(np.float32) * 0.02)
    qw, sw = quantize_convrot_weight(w)
    xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    y = ops.int8_linear(xt, torch.from_numpy(qw).to(cuda), torch.from_numpy(sw).to(cuda),
                        bias=torch.from_numpy(bias).to(cuda).to(torch.bfloat16))
    assert y.dtype == torch.bfloat16 and y.shape == (m, n)
    qx, sx = oracle.quantize_activations(x)
    acc = oracle.int8_gemm_i32(qx, qw)
    check_bf16_within_one_ulp(y, oracle.linear_reference_f64(acc, sx.reshape(-1), sw.reshape(-1), bias), "linear",
                              term=oracle.linear_reference_f64(acc, sx.reshape(-1), sw.reshape(-1), None))
    # accuracy of the whole convrot linear against the unquantised bf16 product
    exact = x.astype(np.float64) @ w.astype(np.float64).T + bias
    rel = np.linalg.norm(y.float().cpu().numpy() - exact) / np.linalg.norm(exact)
    assert rel < 0.05


def test_int8_linear_3d_input_and_out_dtype(cuda):
    from slimdit import ops
    from slimdit.int8 import quantize_convrot_weight
    x = synthetic.activations(2 * 33, 512, seed=3).reshape(2, 33, 512)
    w = synthetic.weight(256, 512, seed=4)
    qw, sw = quantize_convrot_weight(w)
    xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    y = ops.int8_linear(xt, torch.from_numpy(qw).to(cuda), torch.from_numpy(sw).to(cuda), out_dtype=torch.float32)
    assert y.shape == (2, 33, 256) and y.dtype == torch.float32
    y2 = ops.int8_linear(xt.reshape(66, 512), torch.from_numpy(qw).to(cuda), torch.from_numpy(sw).to(cuda))
    assert torch.equal(y.reshape(66, 256).to(torch.bfloat16), y2)


def test_ffn_pair_vs_oracle(cuda):
    """up-proj -> GELU-tanh -> rotate + requant -> down-proj, against the same pipeline on the
    CPU (oracle codes, exact int32 GEMMs, fp32 GELU): outputs within 2 bf16 ulp + the effect
    of hidden codes that differ by GELU rounding (checked via relative error)."""
    from slimdit import ops
    from slimdit.int8 import quantize_convrot_weight
    m, hdim, f = 256, 512, 1024
    x = synthetic.activations(m, hdim, seed=11)
    wu, wd = synthetic.weight(f, hdim, seed=12), synthetic.weight(hdim, f, seed=13)
    qu, su = quantize_convrot_weight(wu)
    qd, sd = quantize_convrot_weight(wd)
    dev = cuda
    y = ops.ffn_int8(torch.from_numpy(x).to(dev).to(torch.bfloat16), torch.from_numpy(qu).to(dev),
                     torch.from_numpy(su).to(dev), torch.from_numpy(qd).to(dev), torch.from_numpy(sd).to(dev))
    qx, sx = oracle.quantize_activations(x)
    acc1 = oracle.int8_gemm_i32(qx, qu)
    h = oracle.bf16_round(oracle.gelu_tanh_f32(oracle.bf16_round(
        (acc1.astype(np.float32) * (sx.reshape(-1, 1) * su.reshape(1, -1))).astype(np.float32))))
    qh, sh = oracle.quantize_activations(h)
    acc2 = oracle.int8_gemm_i32(qh, qd)
    ref = oracle.linear_reference_f64(acc2, sh.reshape(-1), sd.reshape(-1), None)
    yv = y.float().cpu().numpy()
    rel = np.linalg.norm(yv - ref) / np.linalg.norm(ref)
    assert rel < 1e-2, rel


@pytest.mark.parametrize("m,chunk,pinned", [(10000, 4096, True), (300, 128, False), (5, 4096, True)])
def test_int8_linear_host_pipelined_equals_device_call(cuda, m, chunk, pinned):
    """Host-memory activations through the chunked, stream-overlapped path: the same bytes as
    the single device call (token rows are independent)."""
    from slimdit import ops
    from slimdit.int8 import quantize_convrot_weight
    x = synthetic.activations(m, 1024, seed=m)
    w = synthetic.weight(768, 1024, seed=9)
    qw, sw = quantize_convrot_weight(w)
    qw_d, sw_d = torch.from_numpy(qw).to(cuda), torch.from_numpy(sw).to(cuda)
    bias = torch.from_numpy(np.random.default_rng(4).standard_normal(768).astype(np.float32) * 0.02).to(torch.bfloat16)
    xh = torch.from_numpy(x).to(torch.bfloat16)
    if pinned:
        xh = xh.pin_memory()
    y = ops.int8_linear_host(xh, qw_d, sw_d, bias=bias, chunk_rows=chunk)
    torch.cuda.current_stream(cuda).synchronize()
    ref = ops.int8_linear(xh.to(cuda), qw_d, sw_d, bias=bias.to(cuda)).cpu()
    assert y.device.type == "cpu" and torch.equal(y, ref)


def test_swiglu_epilogue_and_minimax_ffn(cuda):
    """fc1 with the fused SwiGLU epilogue (weights in swiglu_interleave order) against the
    plain linear's bf16 up/gate outputs followed by bf16(up * bf16(silu(gate))) in fp32; then
    the whole FFN (fc1 -> SwiGLU -> rotate + requant -> fc2)."""
    from slimdit import ops
    from slimdit.int8 import quantize_convrot_weight
    m, hdim, f = 300, 512, 1024
    x = synthetic.activations(m, hdim, seed=41)
    w1 = synthetic.weight(2 * f, hdim, seed=42)
    w2 = synthetic.weight(hdim, f, seed=43)
    b1 = synthetic.bf16_round_f32(np.random.default_rng(44).standard_normal(2 * f).astype(np.float32) * 0.02)
    q1, s1 = quantize_convrot_weight(w1)
    q2, s2 = quantize_convrot_weight(w2)
    xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    q1d, s1d = torch.from_numpy(q1).to(cuda), torch.from_numpy(s1).to(cuda)
    b1d = torch.from_numpy(b1).to(cuda).to(torch.bfloat16)
    q2d, s2d = torch.from_numpy(q2).to(cuda), torch.from_numpy(s2).to(cuda)
    qi, si, bi = ops.swiglu_interleave(q1d, s1d, b1d)
    qi_h, si_h = qi.cpu().numpy(), si.cpu().numpy()
    for t in range(2 * f // 256):
        assert np.array_equal(qi_h[256 * t:256 * t + 128], q1[128 * t:128 * t + 128])
        assert np.array_equal(qi_h[256 * t + 128:256 * t + 256], q1[f + 128 * t:f + 128 * t + 128])
        assert np.array_equal(si_h[256 * t:256 * t + 128], s1.reshape(-1)[128 * t:128 * t + 128])
    lin = ops.int8_linear(xt, q1d, s1d, bias=b1d).float().cpu().numpy()
    up, gate = lin[:, :f].astype(np.float32), lin[:, f:].astype(np.float32)
    silu = oracle.bf16_round((gate / (np.float32(1.0) + np.exp(-gate))).astype(np.float32))
    ref = oracle.bf16_round((up * silu).astype(np.float32))
    y = ops.int8_linear(xt, qi, si, bias=bi, epilogue="swiglu")
    assert y.shape == (m, f)
    yv = y.float().cpu().numpy()
    diff = np.abs(yv - ref)
    assert np.all(diff <= oracle.bf16_ulp(ref) + 1e-30), "SwiGLU beyond 1 bf16 ulp"
    assert (diff > 0).mean() < 1e-3  # only expf/np.exp last-bit differences may remain
    yf = ops.ffn_swiglu_int8(xt, qi, si, q2d, s2d, bi, None)
    ref_f = ops.int8_linear(y, q2d, s2d)
    assert torch.equal(yf, ref_f)
    with pytest.raises(ValueError):  # rows not a multiple of 256
        ops.swiglu_interleave(q1d[:384], s1d[:384])


@pytest.mark.parametrize("act", ["gelu_tanh", "swiglu"])
@pytest.mark.parametrize("lead", [(1,), (3,), (2, 130), (1000,)])
def test_ffn_c_entry_equals_two_linears(cuda, act, lead):
    """slim_ffn_i8 (one C call: up-proj with the activation epilogue, rotate + requant, down-proj)
    gives the same bytes as the two convrot linears run one after the other, biases included."""
    from slimdit import _native as nat
    from slimdit import ops
    from slimdit.int8 import quantize_convrot_weight
    hdim, f = 512, 768
    n_up = 2 * f if act == "swiglu" else f
    rows = int(np.prod(lead))
    x = synthetic.activations(rows, hdim, seed=51 + rows)
    qu, su = quantize_convrot_weight(synthetic.weight(n_up, hdim, seed=52))
    qd, sd = quantize_convrot_weight(synthetic.weight(hdim, f, seed=53))
    rng = np.random.default_rng(54)
    bu = torch.from_numpy(rng.standard_normal(n_up).astype(np.float32) * 0.02).to(cuda).to(torch.bfloat16)
    bd = torch.from_numpy(rng.standard_normal(hdim).astype(np.float32) * 0.02).to(cuda).to(torch.bfloat16)
    xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16).reshape(*lead, hdim)
    qud, sud = torch.from_numpy(qu).to(cuda), torch.from_numpy(su).to(cuda)
    qdd, sdd = torch.from_numpy(qd).to(cuda), torch.from_numpy(sd).to(cuda)
    if act == "swiglu":
        qud, sud, bu = ops.swiglu_interleave(qud, sud, bu)
        y = ops.ffn_swiglu_int8(xt, qud, sud, qdd, sdd, bu, bd)
    else:
        y = ops.ffn_int8(xt, qud, sud, qdd, sdd, bu, bd)
    h = ops.int8_linear(xt, qud, sud, bias=bu, epilogue=act)
    ref = ops.int8_linear(h, qdd, sdd, bias=bd)
    assert y.shape == (*lead, hdim) and torch.equal(y, ref)
    # the C entry rejects an activation that is not an FFN's
    z = torch.empty(1, device=cuda)
    rc = nat.load().slim_ffn_i8(xt.data_ptr(), 1, qud.data_ptr(), sud.data_ptr(), None, qdd.data_ptr(),
                                sdd.data_ptr(), None, z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(),
                                z.data_ptr(), z.data_ptr(), rows, hdim, f, nat.EPI_SCALE_BIAS, 0)
    assert rc != 0
    with pytest.raises(ValueError):
        ops.ffn_int8(xt, qdd, sdd, qud, sud)


_THREADS_SCRIPT = r"""
import sys, threading
sys.path[:0] = sys.argv[1:]
import numpy as np, torch
import synthetic
from slimdit import ops, attention, _native
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
qw, sw = ops.rotate_quant(torch.from_numpy(synthetic.weight(512, 1024, seed=1)).to(dev).to(torch.bfloat16))
xs = [torch.from_numpy(synthetic.activations(64 + 97 * i, 1024, seed=i)).to(dev).to(torch.bfloat16) for i in range(8)]
qkv = (torch.randn((300, 3 * 2 * 128), generator=torch.Generator().manual_seed(3)) * 0.5).to(torch.bfloat16).to(dev)
torch.cuda.synchronize()
outs, errors = [None] * 8, []
start = threading.Barrier(8)
def work(i):
    try:
        s = torch.cuda.Stream(device=dev)
        start.wait()  # the first library calls of the process, all at once
        with torch.cuda.stream(s):
            y = ops.int8_linear(xs[i], qw, sw)
            a = attention.attention_packed(qkv, 2) if i % 2 else None
        s.synchronize()
        outs[i] = (y, a)
    except Exception as exc:  # reported below
        errors.append(repr(exc))
threads = [threading.Thread(target=work, args=(i,)) for i in range(8)]
[t.start() for t in threads]
[t.join() for t in threads]
assert not errors, errors
for i in range(8):
    assert torch.equal(outs[i][0], ops.int8_linear(xs[i], qw, sw)), i
    if i % 2:
        assert torch.equal(outs[i][1], attention.attention_packed(qkv, 2)), i
assert _native.device_error() == 0
print("threads ok")
"""


def test_first_calls_from_many_threads_at_once(cuda):
    """Eight host threads, each on its own stream, make the process's first library calls at the
    same moment (the lazy per-device caches race for real only then): every result equals the
    one a single thread gets afterwards."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    paths = [str(root / "viggle-animate-workflow_b200"), str(root), str(root / "tests")]
    r = subprocess.run([sys.executable, "-c", _THREADS_SCRIPT, *paths], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "threads ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_ffn_config2_slice_stage_by_stage(cuda):
    """The config-2 FFN on 2048 tokens (5120 -> 13824 -> 5120, GELU-tanh), through the C entry
    slim_ffn_i8 with the test's own workspaces, checked stage by stage:
    * activation codes/scales = the reference-order quantisation of x (bit-exact);
    * hidden bf16 h: within 1 bf16 ulp of GELU-tanh (fp64) of the epilogue's exact bf16
      pre-activation, and at most 1 in 10^4 beyond half an ulp (the epilogue's hardware exponential
      and reciprocal are approximations);
    * hidden codes/scales = the reference-order quantisation of the GPU's own h (bit-exact), and
      against the codes of the oracle's fp32 GELU: the approximate exponential in the epilogue
      changes at most 1 in 10^4 codes, each by one;
    * output within 1 bf16 ulp of the fp64 dequant of the GPU's own hidden codes."""
    from slimdit import _native
    from slimdit.int8 import quantize_convrot_weight
    m, k, f = 2048, 5120, 13824
    x = synthetic.activations(m, k, seed=21)
    qu, su = quantize_convrot_weight(synthetic.weight(f, k, seed=22))
    qd, sd = quantize_convrot_weight(synthetic.weight(k, f, seed=23))
    dev = cuda
    xt = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    t = {name: torch.from_numpy(a).to(dev) for name, a in (("qu", qu), ("su", su.reshape(-1)), ("qd", qd),
                                                           ("sd", sd.reshape(-1)))}
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    sx = torch.empty((m,), dtype=torch.float32, device=dev)
    h = torch.empty((m, f), dtype=torch.bfloat16, device=dev)
    hq = torch.empty((m, f), dtype=torch.int8, device=dev)
    sh = torch.empty((m,), dtype=torch.float32, device=dev)
    out = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
    lib = _native.load()
    _native.check(lib.slim_ffn_i8(xt.data_ptr(), _native.BF16, t["qu"].data_ptr(), t["su"].data_ptr(), None,
                                  t["qd"].data_ptr(), t["sd"].data_ptr(), None, out.data_ptr(), xq.data_ptr(),
                                  sx.data_ptr(), h.data_ptr(), hq.data_ptr(), sh.data_ptr(), m, k, f,
                                  _native.EPI_GELU_TANH, None))
    torch.cuda.synchronize()
    # stage 1: activation codes
    qx, sxo = oracle.quantize_activations(x)
    assert np.array_equal(xq.cpu().numpy(), qx)
    assert np.array_equal(sx.cpu().numpy().view(np.uint32), sxo.reshape(-1).view(np.uint32))
    # stage 2: the hidden activation. The epilogue's pre-activation is the fp32 chain
    # bf16(fma(float(acc), sa * sb, 0)); restated exactly (an fp32 x fp32 product is exact in fp64,
    # so one rounding to fp32 equals the fused multiply-add). GELU near x = -4 moves by tens of
    # output ulps per input ulp, so the pre-activation must match bit for bit, not within an ulp.
    acc1 = oracle.int8_gemm_i32(qx, qu)
    s_prod = (sxo.reshape(-1, 1).astype(np.float32) * su.reshape(1, -1).astype(np.float32)).astype(np.float32)
    lin = oracle.bf16_round((acc1.astype(np.float32).astype(np.float64) * s_prod.astype(np.float64)).astype(np.float32))
    lin_f64 = oracle.bf16_round((acc1.astype(np.float64) * sxo.reshape(-1, 1) * su.reshape(1, -1)).astype(np.float32))
    assert (lin != lin_f64).mean() <= 1e-3  # the fp32 scale product moves rare pre-activations by one ulp
    l64 = lin.astype(np.float64)
    # GELU-tanh as x / (1 + exp(-2u)) (= 0.5 x (1 + tanh u) exactly): no cancellation where tanh -> -1
    with np.errstate(over="ignore"):  # exp -> inf for very negative x: GELU -> -0
        gelu64 = l64 / (1.0 + np.exp(-2.0 * 0.7978845608028654 * (l64 + 0.044715 * l64 ** 3)))
    hv = h.cpu().float().numpy().astype(np.float64)
    # the epilogue's reciprocal flushes results below 2^-126 to zero: |GELU| < 2^-122 may read as 0
    err = np.abs(hv - gelu64) - np.where(np.abs(gelu64) < 2.0**-122, np.abs(gelu64), 0.0)
    ulp = oracle.bf16_ulp(gelu64)
    assert np.all(err <= ulp), float((err / ulp).max())
    assert (err > 0.5 * ulp * (1 + 2.0**-5)).mean() <= 1e-4  # correctly rounded bar the approximations
    # stage 3: hidden codes of the GPU's own h, and against the oracle's fp32 GELU
    h_gpu = h.cpu().float().numpy()
    qh, sho = oracle.quantize_activations(h_gpu)
    hq_n = hq.cpu().numpy()
    assert np.array_equal(hq_n, qh)
    assert np.array_equal(sh.cpu().numpy().view(np.uint32), sho.reshape(-1).view(np.uint32))
    qh_o, _ = oracle.quantize_activations(oracle.bf16_round(oracle.gelu_tanh_f32(lin)))
    diff = hq_n.astype(np.int32) - qh_o.astype(np.int32)
    assert np.abs(diff).max() <= 1
    assert (diff != 0).mean() <= 1e-4, int((diff != 0).sum())
    # stage 4: the output against the GPU's own hidden codes
    acc2 = oracle.int8_gemm_i32(hq_n, qd)
    check_bf16_within_one_ulp(out, oracle.linear_reference_f64(acc2, sho.reshape(-1), sd.reshape(-1), None), "ffn out")


def test_minimax_swiglu_ffn_slice_stage_by_stage(cuda):
    """The MiniMax-H3 FFN at its real widths (5376 -> 2 x 14336 with the fused SwiGLU -> 5376,
    tools/bench_int8.py:23-28, slimdit/mapping.py:99-101) on 1024 tokens, through the C entry
    slim_ffn_i8 with the test's own workspaces, stage by stage:
    * activation codes/scales = the reference-order quantisation of x (bit-exact);
    * hidden h: within 2 bf16 ulp of bf16(up * bf16(silu(gate))) evaluated in fp64 from the
      epilogue's bf16 up and gate (fp32 pre-activation chain restated exactly; one ulp for a
      flip of the rounded silu, one for the final rounding), at most 1 in 10^3 beyond half an ulp;
    * hidden codes/scales = the reference-order quantisation of the GPU's own h (bit-exact);
    * output within 1 bf16 ulp of the fp64 dequant of those codes."""
    from slimdit import _native, ops
    from slimdit.int8 import quantize_convrot_weight
    m, k, f = 1024, 5376, 14336
    x = synthetic.activations(m, k, seed=61)
    q1, s1 = quantize_convrot_weight(synthetic.weight(2 * f, k, seed=62))  # rows [up; gate]
    q2, s2 = quantize_convrot_weight(synthetic.weight(k, f, seed=63))
    b1 = synthetic.bf16_round_f32(np.random.default_rng(64).standard_normal(2 * f).astype(np.float32) * 0.02)
    dev = cuda
    q1i, s1i, b1i = ops.swiglu_interleave(torch.from_numpy(q1).to(dev), torch.from_numpy(s1.reshape(-1)).to(dev),
                                          torch.from_numpy(b1).to(dev).to(torch.bfloat16))
    q2d, s2d = torch.from_numpy(q2).to(dev), torch.from_numpy(s2.reshape(-1)).to(dev)
    xt = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    sx = torch.empty((m,), dtype=torch.float32, device=dev)
    h = torch.empty((m, f), dtype=torch.bfloat16, device=dev)
    hq = torch.empty((m, f), dtype=torch.int8, device=dev)
    sh = torch.empty((m,), dtype=torch.float32, device=dev)
    out = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
    lib = _native.load()
    _native.check(lib.slim_ffn_i8(xt.data_ptr(), _native.BF16, q1i.data_ptr(), s1i.data_ptr(), b1i.data_ptr(),
                                  q2d.data_ptr(), s2d.data_ptr(), None, out.data_ptr(), xq.data_ptr(), sx.data_ptr(),
                                  h.data_ptr(), hq.data_ptr(), sh.data_ptr(), m, k, f, _native.EPI_SWIGLU, None))
    torch.cuda.synchronize()
    # stage 1: activation codes
    qx, sxo = oracle.quantize_activations(x)
    assert np.array_equal(xq.cpu().numpy(), qx)
    assert np.array_equal(sx.cpu().numpy().view(np.uint32), sxo.reshape(-1).view(np.uint32))
    # stage 2: the hidden activation from the epilogue's bf16 up and gate,
    # bf16(fma(float(acc), sa * sb, bias)) with the fp32 scale product
    acc1 = oracle.int8_gemm_i32(qx, q1)

    def lin(cols):
        sp = (sxo.reshape(-1, 1).astype(np.float32) * s1.reshape(-1)[cols].reshape(1, -1)).astype(np.float32)
        v = acc1[:, cols].astype(np.float32).astype(np.float64) * sp.astype(np.float64) + b1[cols].astype(np.float64)
        return oracle.bf16_round(v.astype(np.float32)).astype(np.float64)

    up, gate = lin(slice(0, f)), lin(slice(f, 2 * f))
    silu = oracle.bf16_round((gate / (1.0 + np.exp(-gate))).astype(np.float32)).astype(np.float64)
    ref = up * silu
    hv = h.cpu().float().numpy().astype(np.float64)
    ulp = oracle.bf16_ulp(ref)
    err = np.abs(hv - ref)
    assert np.all(err <= 2 * ulp), float((err / ulp).max())
    assert (err > 0.5 * ulp * (1 + 2.0**-5)).mean() <= 1e-3
    # stage 3: hidden codes of the GPU's own h
    qh, sho = oracle.quantize_activations(h.cpu().float().numpy())
    hq_n = hq.cpu().numpy()
    assert np.array_equal(hq_n, qh)
    assert np.array_equal(sh.cpu().numpy().view(np.uint32), sho.reshape(-1).view(np.uint32))
    # stage 4: the output against the GPU's own hidden codes
    acc2 = oracle.int8_gemm_i32(hq_n, q2)
    check_bf16_within_one_ulp(out, oracle.linear_reference_f64(acc2, sho.reshape(-1), s2.reshape(-1), None), "swiglu out")
