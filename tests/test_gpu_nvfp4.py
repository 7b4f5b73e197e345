"""GPU parity of the NVFP4 path (slimdit/nvfp4.py format, the NVFP4 up-projection) through the C ABI.

* weight packing and activation quantisation: packed codes, tiled block-scale bytes and
  global scales bit-exact with the oracle's restatement (oracle/nvfp4.py);
* block-scaled FP4 GEMM (tcgen05 kind::mxf4nvf4): raw fp32 accumulators within the fp32
  accumulation bound of the exact fp64 sum, bf16 outputs within 1 bf16 ulp of the fp64
  dequant reference plus that bound (tolerances written below);
* the NVFP4 linear end to end, the numpy API and the converter with --quant nvfp4.
"""

import hashlib

import numpy as np
import pytest
import torch

import oracle
import synthetic
from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu

# fp32 accumulation bound of the tensor cores' block-scaled sums: |acc - exact| <= ACC_TOL * T
# with T = sum_k |a_k * b_k| (the dequantised products, fp64). 2^-20 allows for ~K/64 fp32
# roundings of partial sums that are each at most T.
ACC_TOL = 2.0 ** -20


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def to_dev(a: np.ndarray, device, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("rows,k,dtype", [(128, 64, torch.float32), (256, 5120, torch.bfloat16),
                                          (384, 13824, torch.bfloat16), (128, 320, torch.float16)])
def test_weight_pack_bit_exact_vs_oracle(cuda, rows, k, dtype):
    from slimdit import ops
    w = synthetic.weight(rows, k, seed=rows + k)
    wt = to_dev(w, cuda, dtype)
    q, sf, ts = ops.nvfp4_pack(wt)
    qo, sfo, gso = onv.quantize_nvfp4_weight(wt.float().cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(sf.cpu().numpy(), sfo)
    assert bits(ts.cpu().numpy())[0] == bits(np.array([gso], np.float32))[0]


def test_pack_codes_at_rounding_ties(cuda):
    """Elements placed exactly on every E2M1 rounding boundary of their block (x = theta *
    total, theta in {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5}) and 1-2 ulps either side: the codes
    must still equal the oracle's (IEEE quotient, half-to-even), whatever shortcut the kernel
    takes for the division."""
    from slimdit import ops
    rng = np.random.default_rng(77)
    w = synthetic.weight(256, 512, seed=77)
    n, k = w.shape
    w[:, ::16] = np.float32(0.05) * np.sign(rng.standard_normal((n, k // 16))).astype(np.float32)  # block maxima
    gs = onv.global_scale(np.abs(w).max())
    blocks = w.reshape(n, k // 16, 16)
    bamax = np.abs(blocks).max(axis=2)
    sf = onv.e4m3_encode(np.minimum(((bamax / np.float32(6)).astype(np.float32) / gs).astype(np.float32),
                                    np.float32(448)))
    total = (gs * onv.e4m3_decode(sf)).astype(np.float32)
    thetas = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    for j in range(1, 16):
        th = thetas[rng.integers(0, len(thetas), size=(n, k // 16))]
        x = (th * total).astype(np.float32)
        step = rng.integers(-2, 3, size=x.shape)
        for _ in range(2):
            x = np.where(step > 0, np.nextafter(x, np.float32(np.inf)), x)
            x = np.where(step < 0, np.nextafter(x, np.float32(0)), x)
            step = step - np.sign(step)
        sign = np.where(rng.random(x.shape) < 0.5, np.float32(-1), np.float32(1))
        blocks[:, :, j] = np.where(np.abs(x) < bamax, sign * x, blocks[:, :, j])
    w = blocks.reshape(n, k)
    q, sfd, ts = ops.nvfp4_pack(to_dev(w, cuda))
    qo, sfo, gso = onv.quantize_nvfp4_weight(w)
    assert np.array_equal(sfd.cpu().numpy(), sfo) and ts.cpu().numpy()[0] == gso
    got, want = onv.unpack_nibbles(q.cpu().numpy()), onv.unpack_nibbles(qo)
    assert np.array_equal(got, want), f"{int((got != want).sum())} codes differ at rounding ties"


@pytest.mark.parametrize("m,k,rotate,dtype", [
    (1, 64, False, torch.bfloat16),        # one row, one scale tile column
    (77, 5120, True, torch.bfloat16),      # ragged rows, config K, rotated
    (300, 1024, False, torch.float32),
    (128, 13824, True, torch.bfloat16),    # FFN hidden width
    (200, 256, True, torch.float16),
    (40, 16384, True, torch.float32),      # widest row: fewer rows staged in shared memory
    (130, 1280, True, torch.bfloat16),     # two blocks per thread, odd group count (idle y lanes)
    (33, 7936, True, torch.float16),       # 31 groups, two blocks per thread
    (65, 8192, True, torch.float32),       # fp32 rows: the one-block-per-thread kernel
    (50, 10240, True, torch.bfloat16),     # the two-block kernel's widest rows
])
def test_activation_quant_bit_exact_vs_oracle(cuda, m, k, rotate, dtype):
    from slimdit import ops
    x = synthetic.activations(m, k, seed=m * 3 + k)
    if m > 5:
        x[5] = 0.0                           # an all-zero token row
    xt = to_dev(x, cuda, dtype)
    q, sf, rs = ops.nvfp4_quantize_act(xt, rotate=rotate)
    qo, sfo, rso = onv.quantize_nvfp4_rows(xt.float().cpu().numpy(), rotate=rotate)
    assert sf.shape == ((m + 127) // 128 * 128, k // 16)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(sf.cpu().numpy(), sfo)
    assert np.array_equal(bits(rs.cpu().numpy()), bits(rso))


def test_dequant_and_error_report(cuda):
    from slimdit import ops
    w = synthetic.weight(256, 1024, seed=9)
    wt = to_dev(w, cuda)
    q, sf, ts = ops.nvfp4_pack(wt)
    deq = ops.nvfp4_dequantize(q, sf, ts).cpu().numpy()
    qn, sfn, gs = q.cpu().numpy(), sf.cpu().numpy(), np.float32(ts.cpu().numpy()[0])
    codes = onv.unpack_nibbles(qn)
    bsc = np.repeat(onv.e4m3_decode(onv.from_blocked(sfn, 256, 64)), 16, axis=1)
    expect = (onv.e2m1_decode(codes) * (gs * bsc).astype(np.float32)).astype(np.float32)
    assert np.array_equal(bits(deq), bits(expect))
    err = ops.nvfp4_error(q, sf, ts, wt)
    ref = float(np.linalg.norm(expect.astype(np.float64) - w) / np.linalg.norm(w.astype(np.float64)))
    assert abs(err - ref) <= 1e-9 + 1e-7 * ref
    assert 0.02 < err < 0.2


def _operands(m, n, k, seed):
    x = synthetic.activations(m, k, seed=seed)
    w = synthetic.weight(n, k, seed=seed + 1)
    qa, sfa, sa = onv.quantize_nvfp4_rows(x)
    qb, sfb, gb = onv.quantize_nvfp4_weight(w)
    return (qa, sfa, sa), (qb, sfb, gb)


@pytest.mark.parametrize("m,n,k", [
    (128, 256, 256),      # one tile, one k-block
    (256, 512, 5120),     # several tiles, config K
    (300, 384, 1024),     # ragged M; N % 256 == 128 (half B tile)
    (1, 128, 64),         # one row, one 64-wide K step
    (129, 256, 320),      # K not a multiple of 256 (last k-block has one MMA)
    (512, 768, 13824),    # FFN down-proj K
    (700, 640, 2048),     # several CTA-pair tiles, the last pair's second CTA partly past M
])
def test_gemm_accumulators_and_epilogue_vs_fp64(cuda, m, n, k):
    from slimdit import ops
    (qa, sfa, sa), (qb, sfb, gb) = _operands(m, n, k, seed=m + n + k)
    bias = synthetic.bf16_round_f32(np.random.default_rng(k).standard_normal(n).astype(np.float32) * 0.02)
    y, acc = ops.gemm_nvfp4(to_dev(qa, cuda), to_dev(sfa, cuda), to_dev(sa, cuda), to_dev(qb, cuda),
                            to_dev(sfb, cuda), torch.tensor([gb]), to_dev(bias, cuda, torch.bfloat16),
                            return_acc=True)
    exact, tsum = onv.gemm_reference_f64(qa, sfa, 1.0, qb, sfb, 1.0)
    acc = acc.cpu().numpy().astype(np.float64)
    aerr = np.abs(acc - exact)
    bound = ACC_TOL * tsum + 1e-30
    assert np.all(aerr <= bound), f"accumulators: worst {float((aerr / bound).max()):.3f} of the bound"
    alpha = (sa.astype(np.float32) * np.float32(gb)).astype(np.float64).reshape(-1, 1)
    ref = exact * sa.astype(np.float64).reshape(-1, 1) * np.float64(gb) + bias.astype(np.float64)
    yv = y.float().cpu().numpy().astype(np.float64)
    tol = oracle.bf16_ulp(ref) + 2.0 * ACC_TOL * tsum * alpha
    bad = np.abs(yv - ref) > tol
    assert not bad.any(), f"{int(bad.sum())} outputs beyond 1 bf16 ulp + accumulation bound"
    # GELU epilogue: GELU-tanh of the bf16-rounded linear output, bf16 result
    yg = ops.gemm_nvfp4(to_dev(qa, cuda), to_dev(sfa, cuda), to_dev(sa, cuda), to_dev(qb, cuda), to_dev(sfb, cuda),
                        torch.tensor([gb]), to_dev(bias, cuda, torch.bfloat16), epilogue="gelu_tanh")
    g = oracle.gelu_tanh_f32(yv.astype(np.float32)).astype(np.float64)
    gerr = np.abs(yg.float().cpu().numpy() - g)
    assert np.all(gerr <= 2 * oracle.bf16_ulp(g) + 4 * 2.0 ** -24 * np.abs(yv) + 1e-6)


def test_gemm_rejects_bad_shapes(cuda):
    from slimdit import _native, ops
    a = torch.zeros((4, 32), dtype=torch.uint8, device=cuda)
    sfa = torch.zeros((128, 4), dtype=torch.uint8, device=cuda)
    with pytest.raises(ValueError):   # N not a multiple of 128
        ops.gemm_nvfp4(a, sfa, torch.ones(4), torch.zeros((64, 32), dtype=torch.uint8, device=cuda),
                       torch.zeros((64, 4), dtype=torch.uint8, device=cuda), torch.ones(1))
    with pytest.raises(ValueError):   # K = 48 not a multiple of 64
        ops.nvfp4_quantize_act(torch.zeros((4, 48), dtype=torch.bfloat16, device=cuda))
    with pytest.raises(ValueError):   # rotation needs K % 256 == 0
        ops.nvfp4_quantize_act(torch.zeros((4, 64), dtype=torch.bfloat16, device=cuda), rotate=True)
    y = ops.gemm_nvfp4(a[:0], sfa[:0], torch.ones(0), torch.zeros((128, 32), dtype=torch.uint8, device=cuda),
                       torch.zeros((128, 4), dtype=torch.uint8, device=cuda), torch.ones(1))
    assert y.shape == (0, 128)
    assert _native.device_error() == 0


@pytest.mark.parametrize("m,n,k,rotate", [(77, 512, 5120, False), (256, 1024, 5120, True), (64, 256, 13824, True)])
def test_nvfp4_linear_end_to_end(cuda, m, n, k, rotate):
    """x bf16 -> per-token NVFP4 (optionally rotated) -> FP4 GEMM -> bf16, against the oracle
    pipeline; for rotate=True the weight is packed from its reference-order rotation, so the
    product approximates x @ w^T."""
    from slimdit import ops
    x = synthetic.bf16_round_f32(synthetic.activations(m, k, seed=m + k))
    w = synthetic.weight(n, k, seed=n + k)
    wq = oracle.rotate_reference(w) if rotate else w
    qb, sfb, gb = onv.quantize_nvfp4_weight(wq)
    bias = synthetic.bf16_round_f32(np.random.default_rng(2).standard_normal(n).astype(np.float32) * 0.02)
    y = ops.nvfp4_linear(to_dev(x, cuda, torch.bfloat16), to_dev(qb, cuda), to_dev(sfb, cuda), torch.tensor([gb]),
                         bias=to_dev(bias, cuda, torch.bfloat16), rotate=rotate)
    qa, sfa, sa = onv.quantize_nvfp4_rows(x, rotate=rotate)
    exact, tsum = onv.gemm_reference_f64(qa, sfa, 1.0, qb, sfb, 1.0)
    ref = exact * sa.astype(np.float64).reshape(-1, 1) * np.float64(gb) + bias
    alpha = (sa.astype(np.float64) * gb).reshape(-1, 1)
    yv = y.float().cpu().numpy()
    assert np.all(np.abs(yv - ref) <= oracle.bf16_ulp(ref) + 2.0 * ACC_TOL * tsum * alpha)
    true = x.astype(np.float64) @ w.astype(np.float64).T + bias
    rel = np.linalg.norm(yv - true) / np.linalg.norm(true)
    assert rel < 0.25, rel


def test_numpy_api_matches_oracle(cuda):
    from slimdit import nvfp4
    w = synthetic.weight(256, 512, seed=21)
    assert nvfp4.nvfp4_available()
    q, bs, s = nvfp4.quantize_nvfp4_weight(w)
    qo, bso, so = onv.quantize_nvfp4_weight(w)
    assert q.dtype == np.uint8 and bs.dtype == np.uint8 and s.dtype == np.float32 and s.shape == ()
    assert np.array_equal(q, qo) and np.array_equal(bs, bso) and s == so
    q2, bs2, s2, err = nvfp4.quantize_nvfp4_with_error(w)
    assert np.array_equal(q2, qo) and np.array_equal(bs2, bso) and s2 == so
    ref = np.linalg.norm(onv.dequantize(qo, bso, so) - w) / np.linalg.norm(w)
    assert abs(err - ref) <= 1e-6 * ref


def test_converter_nvfp4_layers_match_oracle(cuda, golden_meta, tmp_path):
    """convert(--quant nvfp4): the manifest is the reference's (tests/golden), and every
    quantised linear's bytes are the oracle's pack of the reference-mapped weight."""
    from slimdit import mapping
    from slimdit.convert import convert
    from slimdit.safetensors_io import ShardSet, read_header
    case = golden_meta["convert"]["case"]
    src_dir = synthetic.official_checkpoint(tmp_path / "official", **case)
    out = tmp_path / "nvfp4.safetensors"
    report = convert(src_dir, out, rank=8, grid=65, quant="nvfp4")
    header = read_header(out)
    raw = out.read_bytes()
    base = 8 + int.from_bytes(raw[:8], "little")
    names = [k for k in header if k != "__metadata__"]
    assert [[n, header[n]["dtype"], header[n]["shape"]] for n in names] == golden_meta["nvfp4"]["output_manifest"]
    src = ShardSet(src_dir)
    quant_ops = [op for op in mapping.build_plan(src.manifest.keys()) if op.kind == "quant"]
    assert len(report.quant_errors) == len(quant_ops)
    for op in quant_ops:
        parts = [src.get(s).float().numpy() for s in op.src]
        w = np.concatenate(parts, axis=0)
        if op.swap_halves:
            h = w.shape[0] // 2
            w = np.concatenate([w[h:], w[:h]], axis=0)
        qo, sfo, so = onv.quantize_nvfp4_weight(w)
        stem = op.out[0][: -len(".weight")]

        def tensor_bytes(name):
            b0, b1 = header[name]["data_offsets"]
            return raw[base + b0: base + b1]

        assert tensor_bytes(f"{stem}.weight") == qo.tobytes(), stem
        assert tensor_bytes(f"{stem}.weight_scale") == sfo.tobytes(), stem
        assert tensor_bytes(f"{stem}.weight_scale_2") == np.float32(so).tobytes(), stem
        assert tensor_bytes(f"{stem}.comfy_quant") == b'{"format": "nvfp4"}'
    assert all(0.02 < e < 0.2 for e in report.quant_errors)


def test_cross_check_against_flashinfer_nvfp4(cuda):
    """Independent cross-check of the NVFP4 bytes against flashinfer's fp4_quantize (NVIDIA's
    NVFP4 quantiser, 16-element blocks, UE4M3 scales in the 128x4 swizzled layout, global scale
    passed as 448*6/amax): scale bytes identical; E2M1 codes identical except where the two
    rounding sequences (x / (s2*sf) here, x * rcp(sf * rcp(1/s2)) there) straddle a grid
    midpoint: those differ by one grid step with the same sign."""
    flashinfer = pytest.importorskip("flashinfer")
    import torch

    from slimdit import ops

    dev = torch.device("cuda", 0)
    for m, k, seed in ((256, 512, 0), (1024, 5120, 1)):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        w = (torch.randn((m, k), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w[:, 7] *= 50
        q, sf, s2 = ops.nvfp4_pack(w)
        gsc = (448.0 * 6.0 / w.float().abs().max()).reshape(1).to(torch.float32)
        fq, fsf = flashinfer.fp4_quantize(w, gsc, sf_vec_size=16, sf_use_ue8m0=False, is_sf_swizzled_layout=True)
        torch.cuda.synchronize()
        fq = fq.view(torch.uint8).reshape(m, k // 2).cpu().numpy()
        fsf = fsf.view(torch.uint8).reshape(-1)[: m * k // 16].reshape(m, k // 16).cpu().numpy()
        assert np.array_equal(sf.cpu().numpy().reshape(m, k // 16), fsf), "block scale bytes differ"
        # flashinfer packs element 2i in the low nibble (the hardware's own operand order); the
        # stored layout here is high nibble first, so the codes are compared element by element
        a = onv.unpack_nibbles(q.cpu().numpy()).astype(np.int16)
        b = np.stack([fq & 15, fq >> 4], -1).reshape(m, k).astype(np.int16)
        diff = a != b
        assert diff.mean() < 1e-3, diff.mean()
        # every difference: same sign, adjacent magnitudes on the E2M1 grid
        assert np.all((a[diff] & 8) == (b[diff] & 8))
        assert np.all(np.abs((a[diff] & 7) - (b[diff] & 7)) == 1)
