"""Host-side logic of the ComfyUI linear hook (no GPU): the install posture when the kernel
cannot run, which calls the override hands to the runtime's own op, and the checkpoint
descriptor checks of SlimInt8Linear."""

import sys
import types

import numpy as np
import pytest
import torch

import oracle
from slimdit import comfy_ops, int8


def _fake_kitchen(monkeypatch):
    mod = types.ModuleType("comfy_kitchen")
    calls = []

    def int8_linear(x, qweight, wscales, **kwargs):
        calls.append(kwargs)
        return "runtime"

    mod.int8_linear = int8_linear
    monkeypatch.setitem(sys.modules, "comfy_kitchen", mod)
    return mod, calls


def test_config_rules():
    assert comfy_ops.install_int8_linear(comfy_ops.Int8LinearConfig(enabled=False)) is None
    with pytest.raises(ValueError):
        comfy_ops.Int8LinearOverride(comfy_ops.Int8LinearConfig(enabled=False))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the posture when no GPU can run the kernel")
def test_install_without_a_gpu_keeps_the_runtime_op(monkeypatch, capsys):
    mod, _ = _fake_kitchen(monkeypatch)
    original = mod.int8_linear
    ov = comfy_ops.install_int8_linear()
    assert mod.int8_linear is original  # fail open
    assert "disabled" in capsys.readouterr().out
    with pytest.raises(RuntimeError):
        comfy_ops.install_int8_linear(comfy_ops.Int8LinearConfig(fail_closed=True))
    ov.uninstall()
    assert mod.int8_linear is original


def test_calls_it_cannot_take_go_to_the_runtime_op(monkeypatch):
    mod, calls = _fake_kitchen(monkeypatch)
    ov = comfy_ops.Int8LinearOverride()
    ov._module, ov._original = mod, mod.int8_linear
    x = torch.zeros((4, 256), dtype=torch.bfloat16)
    q = torch.zeros((16, 256), dtype=torch.int8)
    s = torch.ones((16, 1))
    # host tensors, convrot off, another group size, an unknown argument: all forwarded intact
    assert ov(x, q, s, convrot=True, convrot_groupsize=256, out_dtype=torch.float32) == "runtime"
    assert ov(x, q, s, convrot=False) == "runtime"
    assert ov(x, q, s, convrot=True, convrot_groupsize=128) == "runtime"
    assert ov(x, q, s, convrot=True, some_flag=1) == "runtime"
    assert calls[0] == {"convrot": True, "convrot_groupsize": 256, "out_dtype": torch.float32}
    assert calls[1] == {"convrot": False, "convrot_groupsize": 256}
    assert calls[3] == {"some_flag": 1, "convrot": True, "convrot_groupsize": 256}
    assert ov.stats["calls"] == 4 and ov.stats["fallback_calls"] == 4 and ov.stats["kernel_calls"] == 0


def _state(n=16, k=256, blob=None, bias=True):
    rng = np.random.default_rng(0)
    q, s = oracle.quantize_convrot_weight(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    sd = {"blk.weight": q, "blk.weight_scale": s, "blk.comfy_quant": int8.comfy_quant_blob() if blob is None else blob}
    if bias:
        sd["blk.bias"] = rng.standard_normal(n).astype(np.float32)
    return sd


def test_slim_linear_reads_a_converted_checkpoint():
    lin = comfy_ops.SlimInt8Linear.from_state_dict(_state(), "blk.", device="cpu")
    assert (lin.out_features, lin.in_features) == (16, 256)
    assert lin.weight.dtype == torch.int8 and lin.weight_scale.shape == (16, 1)
    assert lin.bias.dtype == torch.bfloat16
    assert isinstance(lin, torch.nn.Module) and set(dict(lin.named_buffers())) == {"weight", "weight_scale", "bias"}


def test_slim_linear_rejects_other_layers():
    with pytest.raises(KeyError):
        comfy_ops.SlimInt8Linear.from_state_dict({"blk.weight": np.zeros((16, 256), np.int8)}, "blk.", device="cpu")
    from slimdit import nvfp4
    with pytest.raises(ValueError):
        comfy_ops.SlimInt8Linear.from_state_dict(_state(blob=nvfp4.comfy_quant_blob()), "blk.", device="cpu")
    with pytest.raises(ValueError):
        comfy_ops.SlimInt8Linear.from_state_dict(_state(blob=np.full(72, 0xFF, np.uint8)), "blk.", device="cpu")
    with pytest.raises(ValueError):  # in_features not a multiple of the rotation group
        comfy_ops.SlimInt8Linear(torch.zeros((16, 320), dtype=torch.int8), torch.ones(16))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the error without a GPU")
def test_forward_fails_loudly_without_a_gpu():
    from slimdit import _native
    lin = comfy_ops.SlimInt8Linear.from_state_dict(_state(), "blk.", device="cpu")
    with pytest.raises(_native.NativeUnavailable):
        lin(torch.zeros((2, 256), dtype=torch.bfloat16))
