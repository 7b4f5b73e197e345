"""Loader and thin ctypes binding of libslimdit_b200.so (the sm_100a kernels' C ABI).

There is no CPU fallback: every compute entry point of this package goes through this
library, and importing a compute function on a machine without the built library or
without a CUDA device raises immediately with the reason.
"""

from __future__ import annotations

import ctypes
import subprocess
import threading
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
CSRC = PKG_ROOT / "csrc"
LIB_DIR = PKG_ROOT / "lib"
LIB_PATH = LIB_DIR / "libslimdit_b200.so"
INCLUDE_DIR = PKG_ROOT.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]

# status codes (include/slimdit_b200.h)
SLIM_OK = 0
SLIM_ERR_SHAPE = -1
SLIM_ERR_ALIGN = -2
SLIM_ERR_GROUP = -3
SLIM_ERR_ARCH = -4
SLIM_ERR_CUDA = -5
SLIM_ERR_DTYPE = -6
SLIM_ERR_NULL = -7

F32, BF16, F16 = 0, 1, 2
ORDER_REFERENCE, ORDER_BUTTERFLY = 0, 1
EPI_SCALE_BIAS, EPI_GELU_TANH, EPI_SWIGLU = 0, 1, 2


class NativeUnavailable(RuntimeError):
    """The CUDA library is not built, or no sm_100 device is present."""


class SlimError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"slimdit_b200 error {code}: {message}")
        self.code = code


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE_DIR / "slimdit_b200.h"]


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/ into lib/libslimdit_b200.so for sm_100a (nvcc cross-compiles; no GPU needed)."""
    newest = max(p.stat().st_mtime for p in sources())
    if LIB_PATH.exists() and not force and LIB_PATH.stat().st_mtime >= newest:
        return LIB_PATH
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = ["nvcc", *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "slimdit_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    tmp.replace(LIB_PATH)
    return LIB_PATH


_lib = None
_lock = threading.Lock()

_SIGS = {
    "slim_version": (ctypes.c_int, []),
    "slim_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
    "slim_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint)]),
    "slim_launch_count": (ctypes.c_uint64, []),
    "slim_rotate_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "slim_rotate_quant_i8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p]),
    "slim_quantize_rows_i8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p]),
    "slim_dequant_i8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_void_p]),
    "slim_gemm_i8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]),
    "slim_int8_linear": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_void_p]),
    "slim_ffn_i8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]),
    "slim_int8_linear_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "slim_peer_buffer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    "slim_peer_buffer_free": (ctypes.c_int, [ctypes.c_void_p]),
    "slim_copy_2d": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_int64, ctypes.c_void_p]),
    "slim_peer_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p)]),
    "slim_peer_close": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64]),
    "slim_int8_linear_colsplit": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                                 ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                                 ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_void_p]),
    "slim_rel_l2_int8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    "slim_rel_l2": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                   ctypes.c_void_p, ctypes.c_void_p]),
    "slim_nvfp4_pack": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "slim_quant_nvfp4_act": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "slim_nvfp4_dequant": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                          ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                          ctypes.c_void_p, ctypes.c_void_p]),
    "slim_gemm_nvfp4": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_void_p]),
    "slim_nvfp4_linear": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "slim_attn_workspace_bytes": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                 ctypes.POINTER(ctypes.c_uint64)]),
    "slim_attn_quant_qk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                          ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                          ctypes.c_void_p]),
    "slim_attn_quant_v": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                         ctypes.c_void_p]),
    "slim_attn_v_amax": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    "slim_attn_quant_v_scaled": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                                ctypes.c_void_p, ctypes.c_void_p]),
    "slim_attn_int8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "slim_attn_packed": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
}


def exported_symbols() -> list[str]:
    return list(_SIGS)


def load() -> ctypes.CDLL:
    """Load the library (no device needed). Raises NativeUnavailable if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeUnavailable(
                    f"{LIB_PATH} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
                    "(or slimdit._native.build_library()) — there is no CPU fallback")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().slim_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(rc: int) -> None:
    if rc == SLIM_OK:
        return
    msg = last_error()
    if rc in (SLIM_ERR_SHAPE, SLIM_ERR_GROUP, SLIM_ERR_ALIGN, SLIM_ERR_NULL):
        raise ValueError(msg)
    if rc == SLIM_ERR_DTYPE:
        raise TypeError(msg)
    if rc == SLIM_ERR_ARCH:
        raise NativeUnavailable(msg)
    raise SlimError(rc, msg)


def require_cuda():
    """Return torch with a usable CUDA device, or raise NativeUnavailable."""
    import torch

    if not torch.cuda.is_available():
        raise NativeUnavailable("slimdit_b200 needs a CUDA device (B200, sm_100a); there is no CPU fallback")
    load()
    return torch


def stream_ptr(torch_mod, device=None) -> int:
    return torch_mod.cuda.current_stream(device).cuda_stream


def device_error() -> int:
    """Synchronise and return (then clear) the kernels' device error word (0 = none)."""
    code = ctypes.c_uint(0)
    check(load().slim_device_error(ctypes.byref(code)))
    return int(code.value)


def launch_count() -> int:
    return int(load().slim_launch_count())
