"""NVFP4 without a GPU: the host contract of slimdit/nvfp4.py (descriptor bytes, shape rules,
converter manifest) against outputs of the reference's own code (tests/golden/golden.json,
written by tests/golden/make_golden.py), and the oracle's NVFP4 restatement against
independent references: torch's FP8 E4M3 conversion for the block scales, a nearest-grid
search for the E2M1 codes, and a direct index formula for the tiled scale layout."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import synthetic
from oracle import nvfp4 as onv
from slimdit import mapping, nvfp4
from slimdit.convert import output_manifest
from slimdit.safetensors_io import ShardSet


# ------------------------------------------------------------------ reference host contract
def test_descriptor_and_constants_match_reference(golden_meta):
    g = golden_meta["nvfp4"]
    assert nvfp4.NVFP4_DESCRIPTOR == g["descriptor"]
    assert nvfp4.comfy_quant_blob().tolist() == g["blob"]
    assert nvfp4.NVFP4_BLOCK == g["block"]
    assert nvfp4.BLOB_LEN == g["blob_len"]
    assert nvfp4.descriptor_fields(nvfp4.comfy_quant_blob()) == {"format": "nvfp4"}
    # trailing NUL padding is ignored, as in the reference (slimdit/nvfp4.py:108-110)
    padded = np.concatenate([nvfp4.comfy_quant_blob(), np.zeros(5, np.uint8)])
    assert nvfp4.descriptor_fields(padded) == {"format": "nvfp4"}


def test_quantized_shapes_match_reference(golden_meta):
    for key, expect in golden_meta["nvfp4"]["shapes"].items():
        rows, cols = (int(v) for v in key.split("x"))
        if isinstance(expect, str):
            with pytest.raises(ValueError) as err:
                nvfp4.quantized_shapes(rows, cols)
            assert f"ValueError: {err.value}" == expect
        else:
            assert [list(s) for s in nvfp4.quantized_shapes(rows, cols)] == expect


def test_nvfp4_output_manifest_matches_reference(golden_meta, tmp_path):
    case = golden_meta["convert"]["case"]
    src_dir = synthetic.official_checkpoint(tmp_path / "official", **case)
    src = ShardSet(src_dir)
    ops = mapping.build_plan(src.manifest.keys())
    mine = output_manifest(ops, src, 8, 65, None, quant="nvfp4")
    assert [[n, d, list(s)] for n, d, s in mine] == golden_meta["nvfp4"]["output_manifest"]


def test_quantize_refuses_non_2d_and_bad_tiling_before_touching_a_device():
    with pytest.raises(ValueError):
        nvfp4.quantize_nvfp4_weight(np.zeros((4,), np.float32))
    with pytest.raises(ValueError):
        nvfp4.quantize_nvfp4_weight(np.zeros((100, 64), np.float32))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device refusal")
def test_unavailable_without_device_raises_comfy_kitchen_missing():
    assert nvfp4.nvfp4_available() is False
    with pytest.raises(nvfp4.ComfyKitchenMissing):
        nvfp4.quantize_nvfp4_weight(np.zeros((128, 64), np.float32))


# ------------------------------------------------------------------ oracle pins
def test_e4m3_encode_matches_torch_float8():
    rng = np.random.default_rng(3)
    codes = np.arange(0, 127, dtype=np.uint8)
    vals = onv.e4m3_decode(codes).astype(np.float64)
    mids = ((vals[:-1] + vals[1:]) / 2).astype(np.float32)  # exact ties
    x = np.concatenate([
        (rng.random(100_000) * 448).astype(np.float32),
        np.exp2(rng.uniform(-14, 8.8, 100_000)).astype(np.float32),
        mids, np.nextafter(mids, np.float32(0)), np.nextafter(mids, np.float32(1e9)), vals.astype(np.float32),
    ])
    x = np.minimum(x, np.float32(448)).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(onv.e4m3_encode(x), ref)
    dec = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(onv.e4m3_decode(codes), dec)


def test_e2m1_encode_is_round_half_even_on_the_grid():
    grid = onv.E2M1_VALUES.astype(np.float64)
    mids = (grid[:-1] + grid[1:]) / 2
    x = np.concatenate([np.linspace(-7, 7, 20001), mids, -mids, np.nextafter(mids, 0), np.nextafter(mids, 9)])
    x = x.astype(np.float32)
    codes = onv.e2m1_encode(x)
    for v, c in zip(x.tolist(), codes.tolist()):
        a = min(abs(v), 6.0)
        d = np.abs(grid - a)
        best = np.flatnonzero(d == d.min())
        want = best[0] if len(best) == 1 else [b for b in best if b % 2 == 0][0]  # tie: even code
        assert c & 7 == want, (v, c)
        assert (c >> 3) == (1 if np.signbit(np.float32(v)) else 0), (v, c)


def test_blocked_layout_index_formula_and_round_trip():
    rng = np.random.default_rng(5)
    r, c = 256, 12
    sf = rng.integers(0, 255, size=(r, c), dtype=np.uint8)
    blk = onv.to_blocked(sf).reshape(-1)
    for row in range(r):
        for col in range(c):
            off = ((row // 128) * (c // 4) + col // 4) * 512 + (row % 32) * 16 + ((row % 128) // 32) * 4 + col % 4
            assert blk[off] == sf[row, col]
    assert np.array_equal(onv.from_blocked(onv.to_blocked(sf), r, c), sf)


def test_pack_nibbles_high_nibble_first():
    """"two E2M1 values per byte, high nibble first" (slimdit/nvfp4.py:5, docs/DEV_NOTES.md:64)."""
    codes = np.array([[1, 2, 3, 4, 15, 8]], dtype=np.uint8)
    packed = onv.pack_nibbles(codes)
    assert packed.tolist() == [[0x12, 0x34, 0xF8]]
    assert np.array_equal(onv.unpack_nibbles(packed), codes)


def test_on_disk_bytes_of_a_known_block():
    """A 2 x 16 weight whose every element sits on the E2M1 grid: the packed bytes put element
    2i in the high nibble (E2M1 codes: 0.5 -> 1, 1 -> 2, 1.5 -> 3, 2 -> 4, 3 -> 5, 4 -> 6,
    6 -> 7, sign bit 8). With the global scale amax / 2688 a block whose maximum is 6 gets the
    block scale 448 (UE4M3 0x7E), so global x block scale = 1 and the values are their codes."""
    row = np.array([6, -6, 0.5, 1, 1.5, 2, 3, 4, -0.5, -1, -1.5, -2, -3, -4, 0, 6], np.float32)
    w = np.zeros((128, 64), np.float32)
    w[0, :16] = row
    w[1, :16] = row[::-1]
    q, sf, gs = onv.quantize_nvfp4_weight(w)
    assert gs == np.float32(np.float32(6.0) / np.float32(2688.0))
    assert q[0, :8].tolist() == [0x7F, 0x12, 0x34, 0x56, 0x9A, 0xBC, 0xDE, 0x07]
    assert q[1, :8].tolist() == [0x70, 0xED, 0xCB, 0xA9, 0x65, 0x43, 0x21, 0xF7]
    assert onv.from_blocked(sf, 128, 4)[0, 0] == 0x7E and onv.from_blocked(sf, 128, 4)[1, 0] == 0x7E


def test_oracle_weight_recipe_round_trip_error_is_nvfp4_sized():
    w = synthetic.weight(256, 512, seed=11)
    q, sf, gs = onv.quantize_nvfp4_weight(w)
    assert q.shape == (256, 256) and sf.shape == (256, 32) and gs.dtype == np.float32
    assert gs == np.float32(np.float32(np.abs(w).max()) / np.float32(2688))
    deq = onv.dequantize(q, sf, gs)
    err = np.linalg.norm(deq - w) / np.linalg.norm(w)
    assert 0.02 < err < 0.2  # NVFP4 level (the reference reports ~9.4 %, docs/DEV_NOTES.md:166)
    # every block's scaled maximum lands on the E2M1 top codes
    codes = onv.unpack_nibbles(q).reshape(256, 32, 16) & 7
    assert (codes.max(axis=2) >= 6).mean() > 0.99


def test_zero_blocks_and_zero_tensor_give_zero_codes_and_scales():
    w = synthetic.weight(128, 128, seed=12)
    w[:, :16] = 0.0
    q, sf, gs = onv.quantize_nvfp4_weight(w)
    assert np.all(onv.from_blocked(sf, 128, 8)[:, 0] == 0)
    assert np.all(onv.unpack_nibbles(q)[:, :16] == 0)
    q0, sf0, gs0 = onv.quantize_nvfp4_weight(np.zeros((128, 64), np.float32))
    assert gs0 == 0 and not q0.any() and not sf0.any()
