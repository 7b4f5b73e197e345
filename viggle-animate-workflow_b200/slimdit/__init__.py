"""slimdit (B200) — the convrot W8A8 linear and the convrot weight converter on sm_100a.

Drop-in for the reference's ``slimdit`` package on its hot path: the module names and
signatures of ``hadamard``, ``int8``, ``mapping``, ``safetensors_io``, ``convert``,
``curve`` and ``rope`` are the reference's; the rotation, quantisation and GEMM run as
hand-written CUDA kernels in ``libslimdit_b200.so`` (``ops`` exposes them on torch CUDA
tensors). There is no CPU fallback.
"""

from . import hadamard, int8

__all__ = ["hadamard", "int8"]
__version__ = "0.1.0+b200"
