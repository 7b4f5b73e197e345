"""ComfyUI runtime hook for the convrot INT8 linear: the node pack's linears on the sm_100a kernels.

At run time ComfyUI evaluates every linear whose checkpoint carries an ``int8_tensorwise``
``comfy_quant`` descriptor through ``comfy_kitchen.int8_linear(x, qweight, wscales,
convrot=True, convrot_groupsize=256, out_dtype=...)`` (the call of tools/bench_int8.py:65-68;
the checkpoint layout is docs/DEV_NOTES.md:45-53). This module provides:

* ``Int8LinearOverride`` / ``install_int8_linear``: replaces that module attribute with the
  sm_100a linear (``slimdit.ops.int8_linear``: butterfly rotate + per-token INT8, tcgen05 GEMM
  with the dequantising epilogue) for the calls it can take, and hands every other call to the
  original function. Installing it is what makes the models ComfyUI loads from converted
  checkpoints, the MiniMax-H3 DiT included, run their quantised linears here. Like the
  attention override it fails open: without the library or an sm_100 device it prints why and
  leaves the original in place (``fail_closed=True`` raises instead).
* ``SlimInt8Linear``: the same linear as a ``torch.nn.Module`` built straight from a converted
  checkpoint's ``<name>.weight`` / ``<name>.weight_scale`` / ``<name>.comfy_quant`` (and an
  optional ``<name>.bias``), for code that owns its model instead of going through ComfyUI.
* ``SlimSwiGLUFFN``: the MiniMax-H3 FFN ``linear_input_act(fc2, fc1(x), "swiglu")``
  (docs/DEV_NOTES.md:82-87) from two such linears: fc1 stores ``[up; gate]`` (ComfyUI's swiglu
  order, slimdit/mapping.py:99-100), interleaved once at construction for the fused SwiGLU
  epilogue, then one ``slim_ffn_i8`` call per forward.

The NVFP4 twin is not hooked: the reference names no runtime symbol for its NVFP4 linear.
"""

from __future__ import annotations

import time

import numpy as np
import torch

from . import int8

#: The module and attribute the runtime calls for a convrot INT8 linear.
RUNTIME_MODULE = "comfy_kitchen"
RUNTIME_OP = "int8_linear"
GROUP_SIZE = 256


class Int8LinearConfig:
    """Knobs of the override: ``enabled`` as for the attention override, ``fail_closed`` to
    raise instead of keeping the original op when the kernel cannot run, ``min_tokens`` to
    leave tiny calls (below the rows at which a launch pays) to the original op."""

    def __init__(self, enabled=True, fail_closed=False, min_tokens=1):
        self.enabled = enabled
        self.fail_closed = fail_closed
        self.min_tokens = min_tokens


def _descriptor_ok(blob) -> bool:
    try:
        fields = int8.descriptor_fields(blob)
    except (ValueError, UnicodeDecodeError):
        return False
    return (fields.get("format") == "int8_tensorwise" and fields.get("convrot") is True
            and fields.get("convrot_groupsize") == GROUP_SIZE)


class Int8LinearOverride:
    """Replaces ``comfy_kitchen.int8_linear`` while installed. Takes a call when it is the
    convrot linear with group size 256 on an sm_100 CUDA device with a bf16/f16/f32 input,
    int8 [N, K] weights, K % 256 == 0 and N % 8 == 0, and no argument it does not know; every
    other call goes to the original op unchanged. ``stats`` counts both."""

    def __init__(self, config=None, stats=None):
        config = config if config is not None else Int8LinearConfig()
        if not config.enabled:
            raise ValueError("Int8LinearOverride requires an enabled config")
        self.config = config
        self.stats = stats if stats is not None else {}
        for key in ("calls", "kernel_calls", "fallback_calls", "kernel_dispatch_seconds"):
            self.stats.setdefault(key, 0 if key.endswith("calls") else 0.0)
        self._module = None
        self._original = None

    def install(self):
        import importlib

        module = importlib.import_module(RUNTIME_MODULE)
        self._module = module
        self._original = getattr(module, RUNTIME_OP)
        try:
            from . import _native

            _native.load()
            _native.require_cuda()
        except Exception as exc:  # environment dependent: no library or no sm_100 device
            if self.config.fail_closed:
                raise RuntimeError(f"sm_100a int8 linear unavailable: {exc}") from exc
            print(f"[slim-linear] disabled, kernel unavailable: {exc}", flush=True)
            return self
        setattr(module, RUNTIME_OP, self)
        return self

    def uninstall(self):
        if self._module is not None and getattr(self._module, RUNTIME_OP, None) is self:
            setattr(self._module, RUNTIME_OP, self._original)

    def takes(self, x, qweight, wscales, convrot, convrot_groupsize, bias, kwargs) -> bool:
        """Whether the sm_100a linear takes this call (the rest go to the original op)."""
        from . import ops

        if kwargs or not convrot or convrot_groupsize != GROUP_SIZE:
            return False
        if not all(isinstance(t, torch.Tensor) for t in (x, qweight, wscales)):
            return False
        if bias is not None and not isinstance(bias, torch.Tensor):
            return False
        if not (x.is_cuda and qweight.is_cuda and wscales.is_cuda) or x.dtype not in ops._DT:
            return False
        if qweight.device != x.device or wscales.device != x.device:
            return False
        if qweight.dtype != torch.int8 or qweight.dim() != 2 or x.dim() < 1:
            return False
        n, k = qweight.shape
        if x.shape[-1] != k or k % GROUP_SIZE or n % 8 or wscales.numel() != n:
            return False
        if bias is not None and (bias.numel() != n or bias.device != x.device):
            return False
        if x.numel() // k < self.config.min_tokens:
            return False
        return torch.cuda.get_device_capability(x.device)[0] == 10  # sm_100 only

    def __call__(self, x, qweight, wscales, convrot=True, convrot_groupsize=GROUP_SIZE, out_dtype=None,
                 bias=None, **kwargs):
        self.stats["calls"] += 1
        if not self.takes(x, qweight, wscales, convrot, convrot_groupsize, bias, kwargs):
            self.stats["fallback_calls"] += 1
            call_kwargs = dict(kwargs, convrot=convrot, convrot_groupsize=convrot_groupsize)
            if out_dtype is not None:
                call_kwargs["out_dtype"] = out_dtype
            if bias is not None:
                call_kwargs["bias"] = bias
            return self._original(x, qweight, wscales, **call_kwargs)
        from . import ops

        started = time.perf_counter()
        y = ops.int8_linear(x, qweight, wscales, convrot=True, convrot_groupsize=GROUP_SIZE,
                            out_dtype=out_dtype if out_dtype is not None else torch.bfloat16, bias=bias)
        self.stats["kernel_calls"] += 1
        self.stats["kernel_dispatch_seconds"] += time.perf_counter() - started
        return y


def install_int8_linear(config=None, stats=None):
    """Route ComfyUI's convrot INT8 linears to the sm_100a kernels (see Int8LinearOverride).
    Returns the installed override, or None when the config is disabled."""
    config = config if config is not None else Int8LinearConfig()
    if not config.enabled:
        return None
    return Int8LinearOverride(config, stats).install()


def _tensor(value, device):
    if isinstance(value, torch.Tensor):
        return value.to(device)
    return torch.from_numpy(np.ascontiguousarray(value)).to(device)


class SlimInt8Linear(torch.nn.Module):
    """A converted checkpoint's convrot INT8 linear as a module: ``y = int8_linear(x, weight,
    weight_scale, bias)`` on the sm_100a kernels. ``from_state_dict`` validates the
    ``comfy_quant`` descriptor (int8_tensorwise, convrot, group size 256) and the shapes."""

    def __init__(self, qweight, wscales, bias=None):
        super().__init__()
        if qweight.dtype != torch.int8 or qweight.dim() != 2:
            raise ValueError(f"weight must be int8 [N, K], got {qweight.dtype} {tuple(qweight.shape)}")
        n, k = qweight.shape
        if k % GROUP_SIZE:
            raise ValueError(f"in_features {k} is not a multiple of the rotation group {GROUP_SIZE}")
        if wscales.numel() != n:
            raise ValueError(f"weight_scale has {wscales.numel()} entries for {n} rows")
        self.in_features, self.out_features = k, n
        self.register_buffer("weight", qweight.contiguous())
        self.register_buffer("weight_scale", wscales.reshape(n, 1).to(torch.float32).contiguous())
        self.register_buffer("bias", None if bias is None else bias.reshape(n).to(torch.bfloat16).contiguous())

    @classmethod
    def from_state_dict(cls, state_dict, prefix, device="cuda"):
        """Build from ``<prefix>weight``, ``<prefix>weight_scale``, ``<prefix>comfy_quant`` and
        the optional ``<prefix>bias`` of a converted checkpoint (numpy arrays or tensors)."""
        blob = state_dict.get(prefix + "comfy_quant")
        if blob is None:
            raise KeyError(f"{prefix}comfy_quant missing: not a quantised linear")
        blob = blob.cpu().numpy() if hasattr(blob, "cpu") else np.asarray(blob)
        if not _descriptor_ok(blob):
            raise ValueError(f"{prefix}comfy_quant is not an int8_tensorwise convrot-256 descriptor")
        bias = state_dict.get(prefix + "bias")
        return cls(_tensor(state_dict[prefix + "weight"], device), _tensor(state_dict[prefix + "weight_scale"], device),
                   None if bias is None else _tensor(bias, device))

    def forward(self, x, out_dtype=None):
        from . import ops

        return ops.int8_linear(x, self.weight, self.weight_scale, bias=self.bias,
                               out_dtype=out_dtype if out_dtype is not None else torch.bfloat16)


class SlimSwiGLUFFN(torch.nn.Module):
    """The MiniMax-H3 FFN ``fc2(swiglu(fc1(x)))`` from two ``SlimInt8Linear`` (fc1 [2F, K] in
    ComfyUI's ``[up; gate]`` order, fc2 [K, F]): fc1's rows are interleaved once for the fused
    SwiGLU epilogue, then each forward is one ``slim_ffn_i8`` call (fc1 with the SwiGLU
    epilogue, rotate + requant of the hidden, fc2)."""

    def __init__(self, fc1, fc2):
        from . import ops

        super().__init__()
        if fc1.out_features != 2 * fc2.in_features or fc2.out_features != fc1.in_features:
            raise ValueError(f"fc1 [{fc1.out_features}, {fc1.in_features}] and fc2 [{fc2.out_features}, "
                             f"{fc2.in_features}] are not a gated FFN pair")
        w1, s1, b1 = ops.swiglu_interleave(fc1.weight, fc1.weight_scale, fc1.bias)
        self.register_buffer("w_fc1", w1)
        self.register_buffer("s_fc1", s1)
        self.register_buffer("b_fc1", b1)
        self.fc2 = fc2

    @classmethod
    def from_state_dict(cls, state_dict, fc1_prefix, fc2_prefix, device="cuda"):
        return cls(SlimInt8Linear.from_state_dict(state_dict, fc1_prefix, device),
                   SlimInt8Linear.from_state_dict(state_dict, fc2_prefix, device))

    def forward(self, x):
        from . import ops

        return ops.ffn_swiglu_int8(x, self.w_fc1, self.s_fc1, self.fc2.weight, self.fc2.weight_scale,
                                   self.b_fc1, self.fc2.bias)


__all__ = [
    "GROUP_SIZE", "Int8LinearConfig", "Int8LinearOverride", "RUNTIME_MODULE", "RUNTIME_OP", "SlimInt8Linear",
    "SlimSwiGLUFFN", "install_int8_linear",
]
