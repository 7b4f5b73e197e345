"""Host-side API and ABI checks that need no GPU (the reference's tests/test_int8.py:9-26
and the C-ABI boundary)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent

REFERENCE_BLOB = b'{"format": "int8_tensorwise", "convrot": true, "convrot_groupsize": 256}'


def test_descriptor_matches_the_runtime_blob():
    from slimdit.int8 import BLOB_LEN, comfy_quant_blob, descriptor_fields
    blob = comfy_quant_blob()
    assert blob.dtype == np.uint8 and blob.shape == (BLOB_LEN,)
    assert bytes(blob[: len(REFERENCE_BLOB)]) == REFERENCE_BLOB
    assert bytes(blob[len(REFERENCE_BLOB):]) == b"\x00" * (BLOB_LEN - len(REFERENCE_BLOB))
    assert descriptor_fields(blob) == {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256}


def test_descriptor_matches_golden(golden):
    from slimdit.int8 import comfy_quant_blob
    assert np.array_equal(comfy_quant_blob(), golden["blob"])


def test_descriptor_rejects_other_groups():
    from slimdit.int8 import comfy_quant_blob
    with pytest.raises(ValueError):
        comfy_quant_blob(128)


def test_hadamard_is_orthonormal_symmetric_and_equals_oracle():
    import oracle
    from slimdit.hadamard import build_hadamard
    h = build_hadamard(256)
    assert h.dtype == np.float32
    assert np.allclose(h, h.T)
    assert np.allclose(h @ h, np.eye(256), atol=1e-5)
    assert np.array_equal(h, oracle.build_hadamard(256))
    assert build_hadamard(256) is h  # cached


@pytest.mark.parametrize("size", [2, 8, 32, 128, 100])
def test_hadamard_rejects_non_powers_of_four(size):
    from slimdit.hadamard import build_hadamard
    with pytest.raises(ValueError):
        build_hadamard(size)


def test_rotate_shape_errors_raise_before_any_device_work():
    from slimdit.hadamard import build_hadamard, rotate
    h = build_hadamard(256)
    with pytest.raises(ValueError):
        rotate(np.zeros((4,), np.float32), h)
    with pytest.raises(ValueError):
        rotate(np.zeros((4, 300), np.float32), h)
    with pytest.raises(ValueError):
        rotate(np.zeros((4, 256), np.float32), np.eye(256, dtype=np.float32))


def test_quantize_shape_errors_raise():
    from slimdit.int8 import quantize_convrot_weight
    with pytest.raises(ValueError):
        quantize_convrot_weight(np.zeros((3,), np.float32))
    with pytest.raises(ValueError):
        quantize_convrot_weight(np.zeros((3, 256), np.float32), group_size=128)


def _header_functions():
    text = (ROOT / "include" / "slimdit_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|uint64_t)\s+(slim_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_header_symbol():
    from slimdit import _native
    lib = _native.load()
    declared = _header_functions()
    assert declared, "no declarations parsed from include/slimdit_b200.h"
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_native.exported_symbols())
    assert lib.slim_version() == 1


def test_abi_validation_errors_need_no_device():
    """Argument checks run before any CUDA call: bad group / shape / null give codes, not crashes."""
    from slimdit import _native
    lib = _native.load()
    dummy = ctypes.c_void_p(16)
    assert lib.slim_rotate_quant_i8(dummy, 1, 4, 300, 256, 0, dummy, dummy, None, None) == _native.SLIM_ERR_GROUP
    assert lib.slim_rotate_quant_i8(dummy, 1, 4, 512, 128, 0, dummy, dummy, None, None) == _native.SLIM_ERR_GROUP
    assert lib.slim_rotate_quant_i8(dummy, 9, 4, 512, 256, 0, dummy, dummy, None, None) == _native.SLIM_ERR_DTYPE
    assert lib.slim_rotate_quant_i8(None, 1, 4, 512, 256, 0, dummy, dummy, None, None) == _native.SLIM_ERR_NULL
    assert lib.slim_rotate_quant_i8(ctypes.c_void_p(17), 1, 4, 512, 256, 0, dummy, dummy, None, None) == _native.SLIM_ERR_ALIGN
    assert lib.slim_rotate_quant_i8(dummy, 1, 4, 32768, 256, 1, dummy, dummy, None, None) == _native.SLIM_ERR_SHAPE
    assert lib.slim_gemm_i8(dummy, dummy, dummy, dummy, None, dummy, None, 8, 12, 64, 0, None) == _native.SLIM_ERR_SHAPE
    assert lib.slim_gemm_i8(dummy, dummy, dummy, dummy, None, dummy, None, 8, 16, 40, 0, None) == _native.SLIM_ERR_SHAPE
    assert lib.slim_gemm_i8(dummy, dummy, dummy, dummy, None, dummy, None, 8, 16, 64, 7, None) == _native.SLIM_ERR_DTYPE
    assert lib.slim_rotate_quant_i8(dummy, 1, 0, 512, 256, 0, dummy, dummy, None, None) == _native.SLIM_OK  # empty
    assert "group_size" in _native.last_error() or _native.last_error() != ""


def test_ffn_and_attention_entries_validate_before_any_device_work():
    """slim_ffn_i8 takes only an FFN activation and sane sizes; the attention entries take only
    head dim 128. Both reject the rest with a code and a message, with no CUDA call made."""
    from slimdit import _native
    lib = _native.load()
    d = ctypes.c_void_p(16)

    def ffn(act, m=4, k=512, f=1024):
        return lib.slim_ffn_i8(d, _native.BF16, d, d, None, d, d, None, d, d, d, d, d, d, m, k, f, act, None)

    assert ffn(_native.EPI_SCALE_BIAS) == _native.SLIM_ERR_DTYPE
    assert "activation" in _native.last_error()
    assert ffn(_native.EPI_GELU_TANH, f=0) == _native.SLIM_ERR_SHAPE
    assert ffn(_native.EPI_GELU_TANH, k=300) == _native.SLIM_ERR_GROUP
    assert ffn(_native.EPI_SWIGLU, m=0) == _native.SLIM_OK  # empty: nothing to do
    b = ctypes.c_uint64(0)
    assert lib.slim_attn_workspace_bytes(100, 2, 96, ctypes.byref(b)) != _native.SLIM_OK
    assert lib.slim_attn_workspace_bytes(100, 2, 128, None) == _native.SLIM_ERR_NULL
    assert lib.slim_attn_workspace_bytes(100, 2, 128, ctypes.byref(b)) == _native.SLIM_OK and b.value > 0
    assert lib.slim_attn_packed(d, 100, 2, 64, 1, d, d, b.value, None) != _native.SLIM_OK
    assert lib.slim_attn_packed(None, 100, 2, 128, 1, d, d, b.value, None) == _native.SLIM_ERR_NULL


def test_error_mapping_to_python_exceptions():
    from slimdit import _native
    lib = _native.load()
    dummy = ctypes.c_void_p(16)
    with pytest.raises(ValueError, match="not divisible"):
        _native.check(lib.slim_rotate_quant_i8(dummy, 1, 4, 300, 256, 0, dummy, dummy, None, None))
    with pytest.raises(TypeError):
        _native.check(lib.slim_rotate_quant_i8(dummy, 9, 4, 512, 256, 0, dummy, dummy, None, None))


# No TMA or bulk load in the library may use the cluster-multicast qualifier (the kernels
# run on 1-8 GPUs of a shared node): the sources must not contain it at all.
def test_library_source_uses_no_cluster_multicast_loads():
    needle = "." + "multi" + "cast" + "::" + "clu" + "ster"
    csrc = ROOT / "viggle-animate-workflow_b200" / "csrc"
    for p in csrc.glob("*"):
        assert needle not in p.read_text(), p
