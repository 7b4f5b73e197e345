"""GPU checks of the ComfyUI linear hook: calls made through the runtime's op name
(comfy_kitchen.int8_linear, installed over a stand-in module) give the bytes of
slimdit.ops.int8_linear; SlimInt8Linear / SlimSwiGLUFFN built from converted-checkpoint
tensors give the bytes of the ops they wrap, and the FFN applies SiLU to the gate half
(ComfyUI's [up; gate] order)."""

import sys
import types

import numpy as np
import pytest
import torch

import oracle
import synthetic
from slimdit import comfy_ops, int8

pytestmark = pytest.mark.gpu


def _kitchen(monkeypatch):
    mod = types.ModuleType("comfy_kitchen")
    mod.int8_linear = lambda *a, **k: "runtime"
    monkeypatch.setitem(sys.modules, "comfy_kitchen", mod)
    return mod


def _weights(cuda, n, k, seed):
    from slimdit import ops
    w = torch.from_numpy(synthetic.weight(n, k, seed=seed)).to(cuda).to(torch.bfloat16)
    q, s = ops.rotate_quant(w, order="reference")
    return q, s


def test_runtime_op_name_runs_the_sm100_linear(cuda, monkeypatch):
    from slimdit import ops
    mod = _kitchen(monkeypatch)
    ov = comfy_ops.install_int8_linear()
    try:
        assert mod.int8_linear is ov
        q, s = _weights(cuda, 768, 1024, 3)
        bias = (torch.randn(768, generator=torch.Generator().manual_seed(4)) * 0.02).to(cuda).to(torch.bfloat16)
        x = torch.from_numpy(synthetic.activations(300, 1024, seed=5)).to(cuda).to(torch.bfloat16)
        y = mod.int8_linear(x, q, s, convrot=True, convrot_groupsize=256, out_dtype=torch.bfloat16, bias=bias)
        assert torch.equal(y, ops.int8_linear(x, q, s, bias=bias))
        x3 = x.reshape(3, 100, 1024)
        y3 = mod.int8_linear(x3, q, s, convrot=True, convrot_groupsize=256, out_dtype=torch.float32)
        assert y3.shape == (3, 100, 768) and y3.dtype == torch.float32
        assert torch.equal(y3.reshape(300, 768), ops.int8_linear(x, q, s, out_dtype=torch.float32))
        assert mod.int8_linear(x, q, s, convrot=False) == "runtime"  # not the convrot linear: the runtime's op
        assert ov.stats["kernel_calls"] == 2 and ov.stats["fallback_calls"] == 1
    finally:
        ov.uninstall()
    assert mod.int8_linear(None, None, None) == "runtime"


def _checkpoint(n, k, seed, bias=True):
    rng = np.random.default_rng(seed)
    q, s = oracle.quantize_convrot_weight(synthetic.weight(n, k, seed=seed))
    sd = {"weight": q, "weight_scale": s, "comfy_quant": int8.comfy_quant_blob()}
    if bias:
        sd["bias"] = oracle.bf16_round(rng.standard_normal(n).astype(np.float32) * 0.02)
    return sd


def _prefixed(prefix, sd):
    return {prefix + key: value for key, value in sd.items()}


def test_slim_linear_from_a_checkpoint(cuda):
    from slimdit import ops
    sd = _prefixed("blocks.0.attn.out_proj.", _checkpoint(512, 768, 7))
    lin = comfy_ops.SlimInt8Linear.from_state_dict(sd, "blocks.0.attn.out_proj.", device=cuda)
    x = torch.from_numpy(synthetic.activations(129, 768, seed=8)).to(cuda).to(torch.bfloat16)
    want = ops.int8_linear(x, lin.weight, lin.weight_scale, bias=lin.bias)
    assert torch.equal(lin(x), want)


def test_swiglu_ffn_from_a_checkpoint(cuda):
    from slimdit import ops
    hdim, f, m = 512, 1024, 260
    sd = {}
    sd.update(_prefixed("mlp.fc1.", _checkpoint(2 * f, hdim, 21)))  # [up; gate]
    sd.update(_prefixed("mlp.fc2.", _checkpoint(hdim, f, 22, bias=False)))
    ffn = comfy_ops.SlimSwiGLUFFN.from_state_dict(sd, "mlp.fc1.", "mlp.fc2.", device=cuda)
    x = torch.from_numpy(synthetic.activations(m, hdim, seed=23)).to(cuda).to(torch.bfloat16)
    y = ffn(x)
    fc1 = comfy_ops.SlimInt8Linear.from_state_dict(sd, "mlp.fc1.", device=cuda)
    fc2 = comfy_ops.SlimInt8Linear.from_state_dict(sd, "mlp.fc2.", device=cuda)
    w1, s1, b1 = ops.swiglu_interleave(fc1.weight, fc1.weight_scale, fc1.bias)
    assert torch.equal(y, ops.ffn_swiglu_int8(x, w1, s1, fc2.weight, fc2.weight_scale, b1, None))
    # unfused: fc1 in bf16, then up * silu(gate) with the gate the second half, then fc2
    h = fc1(x).float()
    up, gate = h[:, :f], h[:, f:]
    act = (up * torch.nn.functional.silu(gate).to(torch.bfloat16).float()).to(torch.bfloat16)
    ref = fc2(act).float()
    rel = (torch.linalg.vector_norm(y.float() - ref) / torch.linalg.vector_norm(ref)).item()
    assert rel < 1e-2, rel
    swapped = (gate * torch.nn.functional.silu(up).to(torch.bfloat16).float()).to(torch.bfloat16)
    wrong = fc2(swapped).float()
    assert (torch.linalg.vector_norm(y.float() - wrong) / torch.linalg.vector_norm(wrong)).item() > 0.1
