"""The allocation-free linear entry point (slim_int8_linear_noalloc).

It serves callers that cannot allocate device memory themselves — for example a plugin that
runs inside a host framework owning the device memory pool and hands it only its input and
output buffers. Instead of caller workspaces it uses a fixed 32 MiB array compiled into the
library. These tests call it through the C ABI and compare its output with the workspace
entry point slim_int8_linear on the same inputs: both run the same kernels, so the outputs
must be identical (stricter than the 1-bf16-ulp tolerance of the GEMM tests). The file is
named to be collected last.
"""

import ctypes

import pytest
import torch

import synthetic

pytestmark = pytest.mark.gpu


def _weights(dev, n, k, seed):
    from slimdit import ops
    w = torch.from_numpy(synthetic.weight(n, k, seed=seed)).to(dev).to(torch.bfloat16)
    qw, sw = ops.rotate_quant(w, order="reference")
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(seed)) * 0.02).to(dev).to(torch.bfloat16)
    return qw, sw.reshape(-1).contiguous(), bias


def _with_workspaces(lib, nat, x, qw, sw, bias, stream):
    m, k = x.shape
    n = qw.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    xq = torch.empty((m, k), dtype=torch.int8, device=x.device)
    sx = torch.empty((m,), dtype=torch.float32, device=x.device)
    nat.check(lib.slim_int8_linear(x.data_ptr(), nat.BF16, qw.data_ptr(), sw.data_ptr(), bias.data_ptr(),
                                   out.data_ptr(), xq.data_ptr(), sx.data_ptr(), m, n, k, 256,
                                   nat.EPI_SCALE_BIAS, stream))
    return out


def _no_alloc(lib, nat, x, qw, sw, bias, stream):
    m, k = x.shape
    n = qw.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    nat.check(lib.slim_int8_linear_noalloc(x.data_ptr(), nat.BF16, qw.data_ptr(), sw.data_ptr(), bias.data_ptr(),
                                           out.data_ptr(), m, n, k, 256, nat.EPI_SCALE_BIAS, stream))
    return out


def test_no_alloc_linear_matches_workspace_linear_on_two_calls_in_a_row(cuda):
    from slimdit import _native as nat
    lib = nat.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    # Two calls in a row with different shapes: the second one runs on the scratch the first
    # one left behind, and the largest case (6400 x 5120) fills the 32 MiB scratch.
    for m, n, k, seed in [(1000, 768, 13824, 1), (6400, 512, 5120, 2)]:
        x = torch.from_numpy(synthetic.activations(m, k, seed=seed)).to(cuda).to(torch.bfloat16)
        qw, sw, bias = _weights(cuda, n, k, seed + 10)
        got = _no_alloc(lib, nat, x, qw, sw, bias, stream)
        want = _with_workspaces(lib, nat, x, qw, sw, bias, stream)
        torch.cuda.synchronize(cuda)
        assert got.shape == (m, n)
        assert torch.equal(got, want), f"no-alloc output differs for M={m} N={n} K={k}"
    assert nat.device_error() == 0


def test_no_alloc_linear_rejects_calls_beyond_its_scratch(cuda):
    from slimdit import _native as nat
    lib = nat.load()
    dummy = ctypes.c_void_p(256)
    # 8192 x 5120 codes + scales need 40 MiB of the 32 MiB scratch
    rc = lib.slim_int8_linear_noalloc(dummy, nat.BF16, dummy, dummy, None, dummy, 8192, 512, 5120, 256,
                                      nat.EPI_SCALE_BIAS, None)
    assert rc == nat.SLIM_ERR_SHAPE
    assert "scratch" in nat.last_error()
    # the empty problem is accepted and touches nothing
    assert lib.slim_int8_linear_noalloc(None, nat.BF16, None, None, None, None, 0, 512, 5120, 256,
                                        nat.EPI_SCALE_BIAS, None) == nat.SLIM_OK
