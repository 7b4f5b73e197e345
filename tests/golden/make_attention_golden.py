"""Golden vectors for the attention quantisers from the reference's own Triton kernels.

Runs comfyui/ComfyUI-SlimDiT/attention_triton.py's ``quant_int8_rows`` (without the
rotation) and ``tensor_amax`` under Triton's CPU interpreter (TRITON_INTERPRET=1; no GPU in
the container that holds the reference) on seeded packed bf16 buffers, and writes inputs and
outputs to attention_quant_golden.npz next to this script.

Only these two kernels are pinned. On this image's Triton 3.6 interpreter, ``tl.dot`` of
bf16 operands (the rotation in ``quant_int8_rows`` and the products in ``flash_int8``)
returns meaningless values and the fp32 -> float8e4nv cast mis-rounds when the mantissa
carries into the exponent (-126.54 -> -64), so the rotated quantiser, ``quant_fp8_global``
and ``flash_int8`` cannot be executed faithfully here. The unrotated quantiser and the amax
use only fp32 loads, max, division, floor and clamps, which the interpreter runs with numpy.

    python tests/golden/make_attention_golden.py <reference tree>/comfyui/ComfyUI-SlimDiT/attention_triton.py
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
CASES = [(100, 2, 11), (37, 3, 12), (200, 1, 13)]  # (tokens, heads, seed)
D = 128


def packed(seq: int, heads: int, seed: int) -> np.ndarray:
    """Seeded [seq, 3*heads*128] bf16 bits: Student-t(4) x 0.5 with six outlier columns x12."""
    rng = np.random.default_rng(seed)
    x = rng.standard_t(4, size=(seq, 3 * heads * D)).astype(np.float32) * np.float32(0.5)
    x[:, rng.choice(3 * heads * D, size=6, replace=False)] *= 12.0
    return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main(ref_path: str) -> None:
    spec = importlib.util.spec_from_file_location("reference_attention_triton", ref_path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    kernels = mod._kernels()
    out: dict[str, np.ndarray] = {}
    meta = {"cases": [], "source": "comfyui/ComfyUI-SlimDiT/attention_triton.py quant_int8_rows (ROT=False), tensor_amax",
            "triton": __import__("triton").__version__, "interpreter": True}
    for seq, heads, seed in CASES:
        bits = packed(seq, heads, seed)
        buf = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
        row = 3 * heads * D
        block = mod.QUANT_BLOCK
        grid = (-(-seq // block),)
        dummy_h = torch.zeros(1, dtype=torch.bfloat16)
        res = {}
        for name, off in (("q", 0), ("k", heads * D)):
            codes = torch.empty(seq, heads * D, dtype=torch.int8)
            scales = torch.empty(seq, heads, dtype=torch.float32)
            kernels["quant_int8_rows"][grid](buf, codes, scales, seq, row, D, off, dummy_h, H=heads, D=D, ROT=False,
                                             BLOCK=block)
            res[name + "_codes"] = codes.numpy()
            res[name + "_scales"] = scales.numpy()
        amax = torch.zeros(1, dtype=torch.float32)
        kernels["tensor_amax"][grid](buf, amax, seq, row, D, 2 * heads * D, H=heads, D=D, BLOCK=block)
        res["v_amax"] = amax.numpy()
        key = f"s{seq}_h{heads}"
        out[key + "_input_bf16"] = bits
        for k, v in res.items():
            out[f"{key}_{k}"] = v
        meta["cases"].append({"key": key, "seq": seq, "heads": heads, "seed": seed})
    np.savez_compressed(HERE / "attention_quant_golden.npz", **out)
    (HERE / "attention_quant_golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {len(CASES)} cases to {HERE / 'attention_quant_golden.npz'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_attention_golden.py <path to the reference's attention_triton.py>")
    main(sys.argv[1])
