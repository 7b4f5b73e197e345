"""Host-side logic of the attention override (no GPU): the packed-layout check and tensor
unwrapping of the reference's attention_triton.py, the install posture when the kernel cannot
run, and the oracle's own consistency (its quantiser against a per-row restatement, its
online softmax against a one-pass softmax over the same FP8-rounded weights)."""

import sys
import types

import numpy as np
import pytest
import torch

import oracle
import oracle.attention as oa

D = 128


def _views(seq=16, heads=2, dim=D, dtype=torch.bfloat16):
    buf = torch.zeros((seq, 3 * heads * dim), dtype=dtype)
    view = buf.view(1, seq, 3, heads, dim)
    return buf, [view[:, :, i].permute(0, 2, 1, 3) for i in range(3)]


def test_packed_geometry_accepts_the_packed_views():
    from slimdit.attention import packed_geometry

    _, (q, k, v) = _views()
    g = packed_geometry(q, k, v, 2)
    assert g == {"seq": 16, "heads": 2, "dim": D, "row_stride": 3 * 2 * D, "head_stride": D, "row_bytes": 2 * D * 2}


def test_packed_geometry_rejects_other_layouts():
    from slimdit.attention import packed_geometry

    _, (q, k, v) = _views()
    assert packed_geometry(q.contiguous(), k, v, 2) is None          # a copy
    assert packed_geometry(q, k, v, 3) is None                       # wrong head count
    assert packed_geometry(q, v, k, 2) is None                       # k/v swapped
    assert packed_geometry(None, k, v, 2) is None
    _, (q32, k32, v32) = _views(dtype=torch.float32)
    assert packed_geometry(q32, k32, v32, 2) is None                 # not bf16
    _, (q3, k3, v3) = _views(dim=96)
    assert packed_geometry(q3, k3, v3, 2) is None                    # dim not a power of two


def test_unwrap():
    from slimdit.attention import unwrap

    t = torch.zeros(3)
    assert unwrap(t) is t

    class Box:
        def __init__(self, x):
            self.x = x

        def take(self):
            return self.x

    assert unwrap(Box(t)) is t
    assert unwrap(5) == 5


def test_config_and_override_rules():
    from slimdit.attention import DEFAULT_MIN_SEQ, TritonAttnConfig, TritonAttnOverride

    cfg = TritonAttnConfig()
    assert not cfg.enabled and cfg.min_seq == DEFAULT_MIN_SEQ and cfg.rotate
    assert set(cfg.describe()) == {"kernel", "min_seq", "rotate"}
    with pytest.raises(ValueError):
        TritonAttnOverride(cfg)


def _fake_comfy(monkeypatch):
    mod = types.ModuleType("comfy.ldm.minimax.model")
    mod.optimized_attention = lambda *a, **k: "dense"
    for name in ("comfy", "comfy.ldm", "comfy.ldm.minimax"):
        monkeypatch.setitem(sys.modules, name, types.ModuleType(name))
    monkeypatch.setitem(sys.modules, "comfy.ldm.minimax.model", mod)
    return mod


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the posture when no GPU can run the kernel")
def test_install_without_a_gpu(monkeypatch, capsys):
    from slimdit.attention import TritonAttnConfig, install_triton_attn

    mod = _fake_comfy(monkeypatch)
    original = mod.optimized_attention
    ov = install_triton_attn(TritonAttnConfig(enabled=True))
    assert mod.optimized_attention is original          # fail open: the model keeps its attention
    assert "disabled" in capsys.readouterr().out
    with pytest.raises(RuntimeError):
        install_triton_attn(TritonAttnConfig(enabled=True, fail_closed=True))
    assert install_triton_attn(TritonAttnConfig(enabled=False)) is None
    # the override still routes calls it cannot take to the original function
    _, (q, k, v) = _views()
    ov.dense = original
    assert ov(q, k, v, 2, mask=torch.ones(1), skip_reshape=True) == "dense"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the error without a GPU")
def test_compute_entry_fails_loudly_without_a_gpu():
    from slimdit import _native
    from slimdit.attention import attention_packed

    buf, _ = _views()
    with pytest.raises(_native.NativeUnavailable):
        attention_packed(buf, 2)


def test_sylvester_is_symmetric_and_orthogonal():
    h = oa.sylvester(D)
    assert np.array_equal(h, h.T)
    assert np.array_equal(h @ h, D * np.eye(D))
    with pytest.raises(ValueError):
        oa.sylvester(96)


def test_oracle_quantiser_matches_a_per_row_restatement():
    rng = np.random.default_rng(0)
    x = oracle.bf16_round(rng.standard_normal((5, 3, D)).astype(np.float32) * 3)
    h = oa.sylvester(D)
    q8, qs = oa.quant_qk(x, True)
    for t in range(5):
        for hd in range(3):
            y = np.float32(x[t, hd].astype(np.float64) @ h)
            s = np.float32(max(np.float32(np.abs(y).max()), np.float32(1e-8)) / np.float32(127))
            assert qs[t, hd] == s
            codes = np.clip(np.floor(np.float32(y / s) + np.float32(0.5)), -127, 127)
            assert np.array_equal(q8[t, hd], codes.astype(np.int8))
    zero, zs = oa.quant_qk(np.zeros((1, 1, D), np.float32), True)
    assert not zero.any() and zs[0, 0] == np.float32(np.float32(1e-8) / np.float32(127))


def test_oracle_online_softmax_equals_one_pass_softmax():
    """With one key tile the online recurrence is a plain softmax over FP8-rounded weights."""
    rng = np.random.default_rng(1)
    seq = 100
    x = oracle.bf16_round(rng.standard_normal((seq, 3 * D)).astype(np.float32))
    q, k, v = oa.split_packed(x, 1, D)
    q8, qs = oa.quant_qk(q, True)
    k8, ks = oa.quant_qk(k, True)
    v8, amax = oa.quant_v(v)
    scale = oa.attn_scale(D, True)
    out = oa.flash(q8, qs, k8, ks, v8, amax, scale)[:, 0]
    s = (q8[:, 0].astype(np.float64) @ k8[:, 0].astype(np.float64).T).astype(np.float32)
    y = s * ks[:, 0][None, :]
    ra = np.float32(np.float32(qs[:, 0] * scale) * oa.LOG2E)
    m = (y.max(axis=1) * ra).astype(np.float32)
    p = np.exp2((y.astype(np.float64) * ra[:, None] - m[:, None]).astype(np.float32).astype(np.float64))
    from oracle.nvfp4 import e4m3_decode, e4m3_encode
    pq = e4m3_decode(e4m3_encode(p.astype(np.float32))).astype(np.float64)
    ref = (pq @ e4m3_decode(v8[:, 0]).astype(np.float64)) * float(oa.v_scale_of(amax)) / pq.sum(axis=1, keepdims=True)
    assert np.abs(out - ref).max() <= np.abs(ref).max() * 2.0 ** -7


def test_oracle_quality_against_dense_attention():
    rng = np.random.default_rng(2)
    x = oracle.bf16_round((rng.standard_t(4, size=(300, 3 * 2 * D)) * 0.5).astype(np.float32))
    got = oa.attention_packed(x, 2, D)
    dense = oa.dense_attention_f64(x, 2, D)
    cos = (got * dense).sum() / np.linalg.norm(got) / np.linalg.norm(dense)
    assert cos > 0.999


def _golden_cases():
    import json
    from pathlib import Path

    d = Path(__file__).resolve().parent / "golden"
    meta = json.loads((d / "attention_quant_golden.json").read_text())
    data = np.load(d / "attention_quant_golden.npz")
    return meta["cases"], data


def test_oracle_pinned_to_reference_quantiser_golden():
    """The oracle's unrotated Q/K quantiser and V amax equal the reference's own Triton kernels
    (quant_int8_rows with ROT=False, tensor_amax) run by tests/golden/make_attention_golden.py."""
    cases, data = _golden_cases()
    for c in cases:
        key, seq, heads = c["key"], c["seq"], c["heads"]
        x = oracle.bf16_to_f32(data[f"{key}_input_bf16"])
        q, k, v = oa.split_packed(x, heads, D)
        for name, t in (("q", q), ("k", k)):
            codes, scales = oa.quant_qk(t, rotate=False)
            assert np.array_equal(codes.reshape(seq, -1), data[f"{key}_{name}_codes"]), (key, name)
            assert np.array_equal(scales.view(np.uint32), data[f"{key}_{name}_scales"].view(np.uint32)), (key, name)
        _, amax = oa.quant_v(v)
        assert np.float32(amax) == data[f"{key}_v_amax"][0], key
