"""Parity at the benchmarked sizes, on sampled token rows.

The full outputs are too large for the oracle, but token rows are independent (rotation and
quantisation are per row), so 256 seeded rows of each full-size output are recomputed by the
oracle from the same bf16 inputs:
* the config-1 convrot linear, X [32768, 5120] x W [15360, 5120] -> [32768, 15360] bf16:
  every sampled output within 1 bf16 ulp of the fp64 dequant of the reference-order codes;
* the config-3 NVFP4 up-projection, X [115200, 5120] -> [115200, 13824] (rotated, per-token
  NVFP4): within 1 bf16 ulp plus the tensor cores' fp32 accumulation bound of the fp64 dequant.
Inputs are made on the device with the benchmark's distribution (Student-t(4) x 0.5, 16
outlier channels x30).
"""

import numpy as np
import pytest
import torch

import oracle
import synthetic
from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu

SAMPLE = 256
ACC_TOL = 2.0**-20  # tensor-core fp32 accumulation, relative to sum |a b| (tests/test_gpu_nvfp4.py)


def _activations(dev, m: int, k: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    z = torch.randn((m, k), generator=g, device=dev)
    chi2 = torch._standard_gamma(torch.full((m, k), 2.0, device=dev), generator=g) * 2.0
    x = z / torch.sqrt(chi2 / 4.0) * 0.5
    del z, chi2
    x[:, torch.randperm(k, generator=g, device=dev)[:16]] *= 30.0
    return x.to(torch.bfloat16)


def _rows(m: int, seed: int) -> np.ndarray:
    return np.sort(np.random.default_rng(seed).choice(m, size=SAMPLE, replace=False))


def test_config1_linear_sampled_rows(cuda):
    from slimdit import ops
    from test_gpu_gemm import check_bf16_within_one_ulp

    m, n, k = 32768, 15360, 5120
    x = _activations(cuda, m, k, seed=31)
    w = synthetic.weight(n, k, seed=32)
    qw, sw = ops.rotate_quant(torch.from_numpy(w).to(cuda).to(torch.bfloat16), order="reference")
    bias = synthetic.bf16_round_f32(np.random.default_rng(33).standard_normal(n).astype(np.float32) * 0.02)
    y = ops.int8_linear(x, qw, sw, bias=torch.from_numpy(bias).to(cuda).to(torch.bfloat16))
    idx = _rows(m, 34)
    ys = y[torch.from_numpy(idx).to(cuda)]
    xs = x[torch.from_numpy(idx).to(cuda)].float().cpu().numpy()
    del y, x
    qx, sx = oracle.quantize_activations(xs)
    acc = oracle.int8_gemm_i32(qx, qw.cpu().numpy())
    swn = sw.cpu().numpy().reshape(-1)
    check_bf16_within_one_ulp(ys, oracle.linear_reference_f64(acc, sx.reshape(-1), swn, bias), "config-1 rows",
                              term=oracle.linear_reference_f64(acc, sx.reshape(-1), swn, None))


def test_config3_nvfp4_up_projection_sampled_rows(cuda):
    from slimdit import ops

    m, n, k = 115200, 13824, 5120
    x = _activations(cuda, m, k, seed=41)
    w = oracle.rotate_reference(synthetic.weight(n, k, seed=42))
    qb, sfb, gb = ops.nvfp4_pack(torch.from_numpy(w).to(cuda).to(torch.bfloat16))
    y = ops.nvfp4_linear(x, qb, sfb, gb, rotate=True)
    idx = _rows(m, 43)
    ys = y[torch.from_numpy(idx).to(cuda)].float().cpu().numpy()
    xs = x[torch.from_numpy(idx).to(cuda)].float().cpu().numpy()
    del y, x
    qa, sfa, sa = onv.quantize_nvfp4_rows(xs, rotate=True)
    gbn = float(gb.reshape(-1)[0].item())
    exact, tsum = onv.gemm_reference_f64(qa, sfa, 1.0, qb.cpu().numpy(), sfb.cpu().numpy(), 1.0)
    ref = exact * sa.astype(np.float64).reshape(-1, 1) * np.float64(gbn)
    alpha = (sa.astype(np.float64) * gbn).reshape(-1, 1)
    bound = oracle.bf16_ulp(ref) + 2.0 * ACC_TOL * tsum * alpha
    bad = np.abs(ys - ref) > bound
    assert not bad.any(), f"{int(bad.sum())} sampled outputs beyond the bound"
