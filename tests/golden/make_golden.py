"""Generate the golden fixtures by running the REFERENCE's own slimdit code.

Run in a container where the reference tree is mounted (read-only), giving its path:

    python tests/golden/make_golden.py --reference <path to the reference tree>

It imports the reference's ``slimdit`` package by path and records, on seeded synthetic
inputs (tests/synthetic.py):
  * quantize_convrot_weight codes/scales and rotate() outputs for K = 256, 512, 1024, 1280,
    5120, 13824 (every OpenBLAS order the reference's rotation goes through);
  * dequantize_convrot_weight outputs;
  * per-token activation quantisation with the reference's own math (rotate + int8.py:49-51);
  * SHA-256 of the full weight conversion of W [5120, 5120];
  * SHA-256 of the reference's per-token codes and scales (rotate() + int8.py:49-51 per row) of
    8192 x 5120 activations and a 2048 x 13824 FFN hidden, with the number of codes and scales
    the butterfly order changes on them;
  * the descriptor blob, and the bytes (SHA-256 + header) of reference convert() runs on a
    2-block synthetic official checkpoint (full, and with block_limit=0);
  * the NVFP4 host contract of slimdit/nvfp4.py that needs no comfy_kitchen: descriptor
    bytes, quantized_shapes results and errors, and convert.output_manifest(quant="nvfp4")
    on the same checkpoint.
The GPU box has no reference tree: tests read only these fixtures.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import synthetic  # noqa: E402

WEIGHT_CASES = [  # name, rows, K, seed
    ("w_k256", 8, 256, 101),
    ("w_k512", 32, 512, 102),
    ("w_k768", 8, 768, 103),
    ("w_k1024", 16, 1024, 104),
    ("w_k1280", 16, 1280, 105),
    ("w_k5120", 16, 5120, 106),
    ("w_k13824", 8, 13824, 107),
]
ACT_CASES = [("x_k5120", 16, 5120, 201), ("x_k13824", 8, 13824, 202)]
SCALE_CASES = [  # name, synthetic generator, rows, K, seed
    ("act_8192x5120", "activations", 8192, 5120, 1),
    ("hidden_2048x13824", "ffn_hidden", 2048, 13824, 3),
]
CONVERT_CASE = {"n_blocks": 2, "hidden": 512, "ffn": 1024, "time_hidden": 64, "seed": 7, "n_shards": 2}


def sha256(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def nvfp4_contract(src_dir) -> dict:
    from slimdit import mapping, nvfp4
    from slimdit import convert as ref_convert
    from slimdit.safetensors_io import ShardSet

    shapes = {}
    for rows, cols in [(128, 64), (13824, 5120), (5120, 13824), (15360, 5120), (100, 64), (128, 48), (128, 80)]:
        try:
            shapes[f"{rows}x{cols}"] = [list(s) for s in nvfp4.quantized_shapes(rows, cols)]
        except ValueError as err:
            shapes[f"{rows}x{cols}"] = f"ValueError: {err}"
    src = ShardSet(src_dir)
    ops = mapping.build_plan(src.manifest.keys())
    manifest = ref_convert.output_manifest(ops, src, 8, 65, None, quant="nvfp4")
    return {
        "descriptor": nvfp4.NVFP4_DESCRIPTOR,
        "blob": [int(b) for b in nvfp4.comfy_quant_blob()],
        "block": nvfp4.NVFP4_BLOCK,
        "blob_len": nvfp4.BLOB_LEN,
        "shapes": shapes,
        "available_without_comfy_kitchen": bool(nvfp4.nvfp4_available()),
        "output_manifest": [[n, d, list(s)] for n, d, s in manifest],
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference tree (its slimdit package is imported)")
    ap.add_argument("--skip-config0", action="store_true")
    args = ap.parse_args(argv)
    sys.path.insert(0, args.reference)
    from slimdit import convert as ref_convert  # noqa: E402
    from slimdit.hadamard import build_hadamard, rotate  # noqa: E402
    from slimdit.int8 import comfy_quant_blob, dequantize_convrot_weight, quantize_convrot_weight  # noqa: E402

    h = build_hadamard(256)
    arrays: dict[str, np.ndarray] = {}
    meta: dict = {"numpy": np.__version__, "cases": {}}
    for name, rows, k, seed in WEIGHT_CASES:
        w = synthetic.weight(rows, k, seed=seed)
        q, s = quantize_convrot_weight(w)
        arrays[f"{name}_in_bf16"] = synthetic.f32_to_bf16_bits(w)
        arrays[f"{name}_rot"] = rotate(w, h, 256)
        arrays[f"{name}_q"] = q
        arrays[f"{name}_scale"] = s
        if k in (512, 5120):
            arrays[f"{name}_deq"] = dequantize_convrot_weight(q, s)
        meta["cases"][name] = {"rows": rows, "K": k, "seed": seed}
    for name, rows, k, seed in ACT_CASES:
        x = synthetic.activations(rows, k, seed=seed)
        rot = rotate(x, h, 256)
        abs_max = np.abs(rot).max(axis=1, keepdims=True)
        scale = np.clip(abs_max.astype(np.float32) / 127.0, 1e-30, None)
        q = np.rint(rot / scale).clip(-128.0, 127.0).astype(np.int8)
        arrays[f"{name}_in_bf16"] = synthetic.f32_to_bf16_bits(x)
        arrays[f"{name}_rot"] = rot
        arrays[f"{name}_q"] = q
        arrays[f"{name}_scale"] = scale.astype(np.float32)
        meta["cases"][name] = {"rows": rows, "K": k, "seed": seed}
    arrays["blob"] = comfy_quant_blob()
    np.savez_compressed(HERE / "rotation_quant.npz", **arrays)

    if not args.skip_config0:
        w0 = synthetic.weight(5120, 5120, seed=0)
        q0, s0 = quantize_convrot_weight(w0)
        meta["config0"] = {
            "rows": 5120, "K": 5120, "seed": 0,
            "sha256_input_bf16": sha256(synthetic.f32_to_bf16_bits(w0).tobytes()),
            "sha256_q": sha256(q0.tobytes()),
            "sha256_scale": sha256(s0.tobytes()),
            "q_min": int(q0.min()), "q_max": int(q0.max()),
        }

    # at-scale activation rows: the reference's own per-row math on token rows
    sys.path.insert(0, str(HERE.parent.parent))
    import oracle  # noqa: E402  (butterfly order, for the recorded mismatch counts only)

    meta["at_scale"] = {}
    for name, gen, rows, k, seed in SCALE_CASES:
        x = getattr(synthetic, gen)(rows, k, seed=seed)
        q, s = quantize_convrot_weight(x)
        qb, sb = oracle.quantize_activations(x, order="butterfly")
        meta["at_scale"][name] = {
            "generator": gen, "rows": rows, "K": k, "seed": seed,
            "sha256_input_bf16": sha256(synthetic.f32_to_bf16_bits(x).tobytes()),
            "sha256_q": sha256(q.tobytes()), "sha256_scale": sha256(s.tobytes()),
            "butterfly_codes_differ": int((q != qb).sum()),
            "butterfly_code_max_abs_diff": int(np.abs(q.astype(np.int32) - qb.astype(np.int32)).max()),
            "butterfly_scales_differ": int((s.view(np.uint32) != sb.view(np.uint32)).sum()),
        }

    with tempfile.TemporaryDirectory() as tmp:
        src = synthetic.official_checkpoint(Path(tmp) / "official", **CONVERT_CASE)
        out = Path(tmp) / "out.safetensors"
        report = ref_convert.convert(src, out, rank=8, grid=65)
        raw = out.read_bytes()
        (hlen,) = struct.unpack("<Q", raw[:8])
        meta["convert"] = {
            "case": CONVERT_CASE, "rank": 8, "grid": 65,
            "sha256_file": sha256(raw), "size": len(raw),
            "header": raw[8:8 + hlen].decode("utf-8"),
            "quant_errors": [float(e) for e in report.quant_errors],
            "src_sha256": {p.name: sha256(p.read_bytes()) for p in sorted(Path(src).glob("*.safetensors"))},
        }
        # block_limit=0: every host-side tensor (copies, concat, curves, table, rope) and no
        # quantised linear -- checkable without a GPU.
        out0 = Path(tmp) / "out_block0.safetensors"
        ref_convert.convert(src, out0, rank=8, grid=65, block_limit=0)
        raw0 = out0.read_bytes()
        meta["convert_block0"] = {"case": CONVERT_CASE, "rank": 8, "grid": 65, "block_limit": 0,
                                  "sha256_file": sha256(raw0), "size": len(raw0)}
        meta["nvfp4"] = nvfp4_contract(src)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    print("wrote", HERE / "rotation_quant.npz", HERE / "golden.json")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
