"""GPU parity of the rotation / quantisation kernels against the reference's golden
outputs and the oracle, through the C ABI (ops.* call libslimdit_b200.so directly)."""

import hashlib

import numpy as np
import pytest
import torch

import oracle
import synthetic

pytestmark = pytest.mark.gpu

WEIGHT_CASES = ["w_k256", "w_k512", "w_k768", "w_k1024", "w_k1280", "w_k5120", "w_k13824"]


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def bf16_tensor(bits16: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits16).view(np.int16)).to(device).view(torch.bfloat16)


@pytest.mark.parametrize("name", WEIGHT_CASES)
def test_weight_codes_scales_rotation_bit_exact_vs_reference(cuda, golden, name):
    from slimdit import ops
    x = bf16_tensor(golden[f"{name}_in_bf16"], cuda)
    q, s, rot = ops.rotate_quant(x, order="reference", return_rotated=True)
    assert np.array_equal(q.cpu().numpy(), golden[f"{name}_q"])
    assert np.array_equal(bits(s.cpu().numpy()), bits(golden[f"{name}_scale"]))
    assert np.array_equal(bits(rot.cpu().numpy()), bits(golden[f"{name}_rot"]))
    # fused path (no rotated copy) gives the same codes
    q2, s2 = ops.rotate_quant(x, order="reference")
    assert torch.equal(q2, q) and torch.equal(s2, s)


@pytest.mark.parametrize("name", WEIGHT_CASES)
def test_numpy_api_drop_in_matches_reference(cuda, golden, name):
    from slimdit.hadamard import build_hadamard, rotate
    from slimdit.int8 import quantize_convrot_weight
    w = synthetic.bf16_bits_to_f32(golden[f"{name}_in_bf16"])
    q, s = quantize_convrot_weight(w)
    assert q.dtype == np.int8 and s.dtype == np.float32 and s.shape == (w.shape[0], 1)
    assert np.array_equal(q, golden[f"{name}_q"])
    assert np.array_equal(bits(s), bits(golden[f"{name}_scale"]))
    r = rotate(w, build_hadamard(256), 256)
    assert np.array_equal(bits(r), bits(golden[f"{name}_rot"]))


@pytest.mark.parametrize("name", ["w_k512", "w_k5120"])
def test_dequantize_bit_exact_vs_reference(cuda, golden, name):
    from slimdit.int8 import dequantize_convrot_weight
    d = dequantize_convrot_weight(golden[f"{name}_q"], golden[f"{name}_scale"])
    assert np.array_equal(bits(d), bits(golden[f"{name}_deq"]))


def test_config0_full_weight_bit_exact(cuda, golden_meta):
    """The 5120 x 5120 weight: W bf16 [5120, 5120] ~ N(0, 0.02), 5 outlier channels x50 -> codes and scales
    identical to the reference's quantize_convrot_weight (SHA-256)."""
    from slimdit import ops
    meta = golden_meta["config0"]
    w0 = synthetic.weight(5120, 5120, seed=0)
    b16 = synthetic.f32_to_bf16_bits(w0)
    assert hashlib.sha256(b16.tobytes()).hexdigest() == meta["sha256_input_bf16"]
    q, s = ops.rotate_quant(bf16_tensor(b16, cuda), order="reference")
    assert hashlib.sha256(q.cpu().numpy().tobytes()).hexdigest() == meta["sha256_q"]
    assert hashlib.sha256(s.cpu().numpy().tobytes()).hexdigest() == meta["sha256_scale"]


@pytest.mark.parametrize("rows,k", [(1, 256), (3, 512), (5, 1024), (7, 1280), (33, 5120), (4, 13824), (2, 16384),
                                    (2, 20480)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_reference_order_vs_oracle_shapes_and_dtypes(cuda, rows, k, dtype):
    from slimdit import ops
    x = synthetic.activations(rows, k, seed=rows * 31 + k)
    xt = torch.from_numpy(x).to(cuda).to(dtype)
    xin = xt.float().cpu().numpy()
    q, s, rot = ops.rotate_quant(xt, order="reference", return_rotated=True)
    ref_rot = oracle.rotate_reference(xin)
    qo, so = oracle.quantize_rows(ref_rot)
    assert np.array_equal(bits(rot.cpu().numpy()), bits(ref_rot))
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(bits(s.cpu().numpy()), bits(so))
    q2, s2 = ops.rotate_quant(xt, order="reference")
    assert torch.equal(q2, q) and torch.equal(s2, s)


@pytest.mark.parametrize("rows,k", [(1, 256), (3, 512), (9, 768), (64, 5120), (17, 13824), (5, 16384)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_butterfly_bit_exact_vs_oracle(cuda, rows, k, dtype):
    from slimdit import ops
    x = synthetic.activations(rows, k, seed=rows + k)
    xt = torch.from_numpy(x).to(cuda).to(dtype)
    xin = xt.float().cpu().numpy()
    q, s, rot = ops.rotate_quant(xt, order="butterfly", return_rotated=True)
    ref_rot = oracle.rotate_butterfly(xin)
    qo, so = oracle.quantize_rows(ref_rot)
    assert np.array_equal(bits(rot.cpu().numpy()), bits(ref_rot))
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(bits(s.cpu().numpy()), bits(so))


@pytest.mark.parametrize("name", ["x_k5120", "x_k13824"])
def test_butterfly_within_tolerance_of_reference_rotation(cuda, golden, name):
    """Activation order vs the reference's own rotation: |diff| <= 2^-20 * row absmax, codes +-1."""
    from slimdit import ops
    x = bf16_tensor(golden[f"{name}_in_bf16"], cuda)
    q, s, rot = ops.rotate_quant(x, order="butterfly", return_rotated=True)
    ref = golden[f"{name}_rot"]
    tol = np.abs(ref).max(axis=1, keepdims=True) * 2.0**-20
    assert np.all(np.abs(rot.cpu().numpy() - ref) <= tol)
    assert np.abs(q.cpu().numpy().astype(np.int32) - golden[f"{name}_q"]).max() <= 1


def test_quantize_stage_bit_exact_given_reference_rotation(cuda, golden):
    """Quantisation alone, fed the reference's own rotated fp32 rows."""
    from slimdit import ops
    for name in ["w_k5120", "x_k5120", "x_k13824", "w_k256"]:
        rot = torch.from_numpy(golden[f"{name}_rot"]).to(cuda)
        q, s = ops.quantize_rows(rot)
        assert np.array_equal(q.cpu().numpy(), golden[f"{name}_q"]), name
        assert np.array_equal(bits(s.cpu().numpy()), bits(golden[f"{name}_scale"])), name


def test_edge_rows_zero_constant_and_huge(cuda):
    from slimdit import ops
    k = 1280
    x = np.zeros((6, k), np.float32)
    x[1] = 1.0                      # constant row
    x[2, 7] = -3.0                  # single spike
    x[3] = np.float32(1e35)         # large but finite through the whole chain
    x[4, ::2] = 1e-30               # tiny
    x[5] = synthetic.activations(1, k, seed=9)[0]
    for order, rot_fn in (("reference", oracle.rotate_reference), ("butterfly", oracle.rotate_butterfly)):
        q, s, rot = ops.rotate_quant(torch.from_numpy(x).to(cuda), order=order, return_rotated=True)
        ro = rot_fn(x)
        qo, so = oracle.quantize_rows(ro)
        assert np.array_equal(bits(rot.cpu().numpy()), bits(ro)), order
        assert np.array_equal(q.cpu().numpy(), qo), order
        assert np.array_equal(bits(s.cpu().numpy()), bits(so)), order
    assert s.cpu().numpy()[0, 0] == np.float32(1e-30)


def test_empty_and_error_cases(cuda):
    from slimdit import ops
    q, s = ops.rotate_quant(torch.empty((0, 512), device=cuda, dtype=torch.bfloat16))
    assert q.shape == (0, 512) and s.shape == (0, 1)
    with pytest.raises(ValueError):
        ops.rotate_quant(torch.zeros((2, 300), device=cuda))
    with pytest.raises(ValueError):
        ops.rotate_quant(torch.zeros((2, 512), device=cuda), group_size=128)
    with pytest.raises(ValueError):
        ops.rotate_quant(torch.zeros((2, 32768), device=cuda, dtype=torch.bfloat16), order="butterfly")
    from slimdit import _native
    assert _native.device_error() == 0


def test_butterfly_quantiser_near_rounding_boundaries(cuda):
    """Rows whose rotated values sit on or next to half-integer multiples of the row scale:
    the quantiser's reciprocal fast path must hand these to the exact division."""
    from slimdit import ops
    rng = np.random.default_rng(77)
    k = 5120
    rows = []
    for r in range(48):
        target = (rng.integers(-127, 127, size=k) + 0.5).astype(np.float64)
        target[0] = 127.0
        target *= 10.0 ** rng.uniform(-3, 2) / 127.0
        # pre-image under the rotation (H is its own inverse); fp32 inputs keep the ties
        rows.append(oracle.rotate_reference(target.astype(np.float32)[None])[0])
    x = np.stack(rows)
    xt = torch.from_numpy(x).to(cuda)
    q, s, rot = ops.rotate_quant(xt, order="butterfly", return_rotated=True)
    ro = oracle.rotate_butterfly(x)
    qo, so = oracle.quantize_rows(ro)
    assert np.array_equal(bits(rot.cpu().numpy()), bits(ro))
    assert np.array_equal(bits(s.cpu().numpy()), bits(so))
    assert np.array_equal(q.cpu().numpy(), qo)
    # the construction really produced near-ties
    frac = np.abs(ro / so - np.round(ro / so))
    assert (np.abs(frac - 0.5) < 1e-3).mean() > 0.1


# ---- the properties the reference's own tests state for the rotation and the weight
# quantiser (tests/test_int8.py:23-55), here on the sm_100a kernels behind the same API


def test_rotation_is_an_involution_and_stays_within_its_group(cuda):
    from slimdit.hadamard import build_hadamard, rotate
    rng = np.random.default_rng(0)
    w = rng.standard_normal((32, 512)).astype(np.float32)
    h = build_hadamard(256)
    back = rotate(rotate(w, h, 256), h, 256)
    assert np.abs(back - w).max() < 1e-4
    moved = w.copy()
    moved[:, 256:] += 5.0  # only the second group's inputs change
    a, b = rotate(w, h, 256), rotate(moved, h, 256)
    assert np.array_equal(a[:, :256], b[:, :256])
    assert not np.allclose(a[:, 256:], b[:, 256:])


@pytest.mark.parametrize("k, on_device", [(256, False), (256, True)])
def test_convrot_beats_the_plain_grid_on_outlier_rows(cuda, k, on_device):
    """One huge channel per row: after the rotation the row quantises far better than on the
    plain per-row INT8 grid (error below a fifth of it, and below 1 %)."""
    from slimdit.int8 import dequantize_convrot_weight, quantize_convrot_weight
    rng = np.random.default_rng(1)
    w = rng.standard_normal((8, k)).astype(np.float32) * 0.05
    w[:, 0] = 40.0
    if on_device:
        w = oracle.bf16_round(w)
        q, scale = quantize_convrot_weight(torch.from_numpy(w).to(cuda).to(torch.bfloat16), 256)
        back = dequantize_convrot_weight(q, scale, 256)
        back = back.cpu().numpy() if isinstance(back, torch.Tensor) else back
    else:
        q, scale = quantize_convrot_weight(w, 256)
        back = dequantize_convrot_weight(q, scale, 256)
    rotated_err = np.linalg.norm(back - w) / np.linalg.norm(w)
    plain_scale = np.maximum(np.abs(w).max(axis=1, keepdims=True) / np.float32(127), np.float32(1e-30))
    plain_back = np.clip(np.rint(w / plain_scale), -128, 127) * plain_scale
    plain_err = np.linalg.norm(plain_back - w) / np.linalg.norm(w)
    assert rotated_err < plain_err / 5 and rotated_err < 0.01, (rotated_err, plain_err)


def test_dequantize_from_unaligned_codes_matches_aligned(cuda):
    """slim_dequant_i8 takes int8 codes at any address: codes one byte past an aligned address
    (read element by element, not with 16-byte vector loads) give the same fp32 bits."""
    from slimdit import ops
    n, k = 96, 5120
    rng = np.random.default_rng(12)
    q = torch.from_numpy(rng.integers(-128, 128, size=(n, k), dtype=np.int8)).to(cuda)
    scale = torch.from_numpy((rng.random(n, dtype=np.float32) * 1e-3 + 1e-5).astype(np.float32)).to(cuda)
    buf = torch.empty(n * k + 1, dtype=torch.int8, device=cuda)
    shifted = buf[1:].view(n, k)
    shifted.copy_(q)
    assert shifted.data_ptr() % 16 != 0
    assert torch.equal(ops.dequantize(shifted, scale).view(torch.int32), ops.dequantize(q, scale).view(torch.int32))


@pytest.mark.parametrize("name", ["act_8192x5120", "hidden_2048x13824"])
def test_reference_order_activations_at_scale_vs_reference_digests(cuda, golden_meta, name):
    """Per-token codes and scales in the reference order at scale: SHA-256 equal to the
    reference's own outputs; the butterfly order's differences from them are counted exactly."""
    from slimdit import ops
    meta = golden_meta["at_scale"][name]
    x = getattr(synthetic, meta["generator"])(meta["rows"], meta["K"], seed=meta["seed"])
    b16 = synthetic.f32_to_bf16_bits(x)
    assert hashlib.sha256(b16.tobytes()).hexdigest() == meta["sha256_input_bf16"]
    xt = bf16_tensor(b16, cuda)
    q, s = ops.rotate_quant(xt, order="reference")
    qn, sn = q.cpu().numpy(), s.cpu().numpy()
    assert hashlib.sha256(qn.tobytes()).hexdigest() == meta["sha256_q"]
    assert hashlib.sha256(sn.tobytes()).hexdigest() == meta["sha256_scale"]
    qb, sb = ops.rotate_quant(xt, order="butterfly")
    qb, sb = qb.cpu().numpy(), sb.cpu().numpy()
    assert int((qn != qb).sum()) == meta["butterfly_codes_differ"]
    assert int(np.abs(qn.astype(np.int32) - qb.astype(np.int32)).max()) == meta["butterfly_code_max_abs_diff"]
    assert int((bits(sn) != bits(sb)).sum()) == meta["butterfly_scales_differ"]


def _stress_rows(k: int, dtype) -> np.ndarray:
    """Rows that drive every branch of the certified quantiser: wide dynamic ranges (many
    inexact groups and queued outputs), integer rows (exact ties), a spike over tiny noise (many
    outputs tied for the row maximum), zero, constant, tiny and heavy-tailed rows."""
    rng = np.random.default_rng(k)
    hi = 12 if dtype == torch.float16 else 40
    lo = -12 if dtype == torch.float16 else -40
    rows = []
    for _ in range(24):  # log-uniform magnitudes with random signs
        mag = np.exp2(rng.uniform(lo, hi, size=k))
        rows.append(mag * rng.choice([-1.0, 1.0], size=k))
    for _ in range(8):
        rows.append(rng.integers(-3, 4, size=k).astype(np.float64))
    for _ in range(4):
        r = rng.standard_normal(k) * 1e-3
        r[rng.integers(0, k)] = 50.0
        rows.append(r)
    rows.append(np.zeros(k))
    rows.append(np.full(k, 0.75))
    rows.append(rng.standard_normal(k) * (1e-4 if dtype == torch.float16 else 1e-30))
    rows.extend(synthetic.activations(16, k, seed=k + 5).astype(np.float64))
    rows.extend(synthetic.ffn_hidden(16, k, seed=k + 6).astype(np.float64))
    return np.stack(rows).astype(np.float32)


@pytest.mark.parametrize("k", [1280, 2816, 5120, 7168, 10240, 10496, 13824, 16384])  # 10240 / 10496: either side of
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])     # the narrow/wide switch
def test_certified_reference_order_stress_vs_oracle(cuda, k, dtype):
    from slimdit import ops
    xt = torch.from_numpy(_stress_rows(k, dtype)).to(cuda).to(dtype)
    xin = xt.float().cpu().numpy()
    q, s = ops.rotate_quant(xt, order="reference")
    qo, so = oracle.quantize_rows(oracle.rotate_reference(xin))
    assert np.array_equal(bits(s.cpu().numpy()), bits(so))
    assert np.array_equal(q.cpu().numpy(), qo)


@pytest.mark.parametrize("rows", [1, 3, 997, 4096])
def test_certified_reference_order_many_rows_vs_oracle(cuda, rows):
    """Row counts below, near and far above the persistent grid (queues carried across rows)."""
    from slimdit import ops
    x = synthetic.ffn_hidden(rows, 5120, seed=rows)
    xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    q, s = ops.rotate_quant(xt, order="reference")
    qo, so = oracle.quantize_convrot_weight(x)
    assert np.array_equal(bits(s.cpu().numpy()), bits(so))
    assert np.array_equal(q.cpu().numpy(), qo)
