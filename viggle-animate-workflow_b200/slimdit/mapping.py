"""Official MiniMax-H3 (Viggle-Animate) -> ComfyUI curve-format key plan.

Same tables and functions as the reference's slimdit/mapping.py:27-194, because the output
must be the layout ComfyUI's MiniMax loader reads: ``blocks.*`` instead of
``transformer_blocks.*``, fused ``qkv_proj`` (q, k, v concatenated along rows), ``fc1`` with
its two row halves swapped (the runtime's SwiGLU takes [up; gate], the official checkpoint
stores [gate; up]), adaLN linears replaced by rank-r curves, fp32 copies of the
patch/final/time-embedder projections, and a derived ``rope.inv_freq``.

Op kinds: ``quant`` (concat, rotate, INT8 -> weight + weight_scale + comfy_quant),
``copy`` (cast to the storage dtype), ``concat``, ``curve`` (W @ P), ``derived``.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

Kind = Literal["quant", "copy", "concat", "curve", "curve_table", "derived"]

# output suffix, official suffixes concatenated along dim 0 in this order, swap halves
QUANT_BLOCK_LAYERS: tuple[tuple[str, tuple[str, ...], bool], ...] = (
    ("attn.qkv_proj.weight", ("attn.to_q.weight", "attn.to_k.weight", "attn.to_v.weight"), False),
    ("attn.out_proj.weight", ("attn.to_out.0.weight",), False),
    ("mlp.fc1.weight", ("ff.net.0.proj.weight",), True),
    ("mlp.fc2.weight", ("ff.net.2.weight",), False),
)

COPY_BLOCK_LAYERS: tuple[tuple[str, str], ...] = (
    ("norm1.weight", "norm1.weight"),
    ("norm2.weight", "norm2.weight"),
    ("attn.q_norm.weight", "attn.norm_q.weight"),
    ("attn.k_norm.weight", "attn.norm_k.weight"),
)

REFINER_COPY_LAYERS: tuple[tuple[str, str, bool], ...] = (
    ("norm1.weight", "norm1.weight", False),
    ("norm2.weight", "norm2.weight", False),
    ("attn.q_norm.weight", "attn.norm_q.weight", False),
    ("attn.k_norm.weight", "attn.norm_k.weight", False),
    ("attn.out_proj.weight", "attn.to_out.0.weight", False),
    ("mlp.fc1.weight", "ff.net.0.proj.weight", True),
    ("mlp.fc2.weight", "ff.net.2.weight", False),
)

# The refiner stays bf16; its fused qkv_proj is assembled from the separate q/k/v weights.
REFINER_CONCAT_LAYERS: tuple[tuple[str, tuple[str, ...]], ...] = (
    ("attn.qkv_proj.weight", ("attn.to_q.weight", "attn.to_k.weight", "attn.to_v.weight")),
)

# output name, official name, storage dtype (the model builds these in fp32 except the
# condition projection and the final norm)
GLOBAL_COPY_LAYERS: tuple[tuple[str, str, str], ...] = (
    ("video_patch_proj.weight", "proj_in.weight", "f32"),
    ("video_patch_proj.bias", "proj_in.bias", "f32"),
    ("audio_patch_proj.weight", "audio_proj_in.weight", "f32"),
    ("audio_patch_proj.bias", "audio_proj_in.bias", "f32"),
    ("condition_proj.weight", "context_embedder.weight", "bf16"),
    ("condition_proj.bias", "context_embedder.bias", "bf16"),
    ("final_layer.video_out.weight", "proj_out.weight", "f32"),
    ("final_layer.video_out.bias", "proj_out.bias", "f32"),
    ("final_layer.audio_out.weight", "audio_proj_out.weight", "f32"),
    ("final_layer.audio_out.bias", "audio_proj_out.bias", "f32"),
    ("final_layer.norm.weight", "norm_out.norm.weight", "bf16"),
    ("time_embedder.proj_in.weight", "time_embedder.linear_1.weight", "f32"),
    ("time_embedder.proj_in.bias", "time_embedder.linear_1.bias", "f32"),
    ("time_embedder.proj_out.weight", "time_embedder.linear_2.weight", "f32"),
    ("time_embedder.proj_out.bias", "time_embedder.linear_2.bias", "f32"),
)

# Time-embedder tensors the shared curve basis is built from.
CURVE_SOURCES = (
    "time_embedder.linear_1.weight",
    "time_embedder.linear_1.bias",
    "time_embedder.linear_2.weight",
    "time_embedder.linear_2.bias",
)

FINAL_ADALN = ("final_layer.adaln_proj.linear", "norm_out.linear")
BLOCK_ADALN = ("blocks.{i}.adaln_proj.linear", "transformer_blocks.{i}.adaln_proj.linear")


@dataclass
class Op:
    """One unit of conversion work: read ``src`` tensors, write ``out`` tensors."""

    out: tuple[str, ...]
    kind: Kind
    src: tuple[str, ...] = ()
    dtype: str = "bf16"
    note: str = ""
    #: swap the two halves of the row dimension ([gate; up] -> [up; gate])
    swap_halves: bool = False
    extra: dict = field(default_factory=dict)


def block_count(keys) -> int:
    """Number of distinct ``transformer_blocks.<i>`` indices in ``keys``."""
    seen = set()
    for k in keys:
        parts = k.split(".")
        if parts[0] == "transformer_blocks" and len(parts) > 1 and parts[1].isdigit():
            seen.add(parts[1])
    return len(seen)


def build_plan(keys) -> list[Op]:
    """Ordered conversion plan for the official key set."""
    keys = set(keys)
    n_blocks = block_count(keys)
    if n_blocks == 0:
        raise ValueError("no transformer_blocks.* keys found -- wrong checkpoint?")

    plan: list[Op] = []
    for i in range(n_blocks):
        src_p, dst_p = f"transformer_blocks.{i}", f"blocks.{i}"
        for out_s, src_s, swap in QUANT_BLOCK_LAYERS:
            plan.append(Op(out=(f"{dst_p}.{out_s}",), kind="quant", src=tuple(f"{src_p}.{s}" for s in src_s),
                           swap_halves=swap))
        for out_s, src_s in COPY_BLOCK_LAYERS:
            plan.append(Op(out=(f"{dst_p}.{out_s}",), kind="copy", src=(f"{src_p}.{src_s}",)))
        plan.append(Op(out=(f"{dst_p}.adaln_proj.linear.weight",), kind="curve",
                       src=(f"{src_p}.adaln_proj.linear.weight",), dtype="f16"))
        plan.append(Op(out=(f"{dst_p}.adaln_proj.linear.bias",), kind="copy",
                       src=(f"{src_p}.adaln_proj.linear.bias",), dtype="f16"))

    refiner_ids = sorted({k.split(".")[2] for k in keys if k.startswith("token_refiner.refiner_blocks.")})
    for i in refiner_ids:
        src_p, dst_p = f"token_refiner.refiner_blocks.{i}", f"token_refiner.blocks.{i}"
        for out_s, src_s in REFINER_CONCAT_LAYERS:
            plan.append(Op(out=(f"{dst_p}.{out_s}",), kind="concat", src=tuple(f"{src_p}.{s}" for s in src_s)))
        for out_s, src_s, swap in REFINER_COPY_LAYERS:
            plan.append(Op(out=(f"{dst_p}.{out_s}",), kind="copy", src=(f"{src_p}.{src_s}",), swap_halves=swap))
    plan.append(Op(out=("token_refiner.final_norm.weight",), kind="copy", src=("token_refiner.final_norm.weight",)))

    for out_name, src_name, dt in GLOBAL_COPY_LAYERS:
        plan.append(Op(out=(out_name,), kind="copy", src=(src_name,), dtype=dt))

    plan.append(Op(out=(FINAL_ADALN[0] + ".weight",), kind="curve", src=(FINAL_ADALN[1] + ".weight",), dtype="f16"))
    plan.append(Op(out=(FINAL_ADALN[0] + ".bias",), kind="copy", src=(FINAL_ADALN[1] + ".bias",), dtype="f16"))
    # derived by the reference model, loaded by ComfyUI; not in the official checkpoint
    plan.append(Op(out=("rope.inv_freq",), kind="derived", dtype="f32", note="rope_inv_freq"))
    return plan


def quant_tensor_names(weight_name: str) -> tuple[str, str, str]:
    """The three tensors ComfyUI reads for one INT8 convrot linear."""
    base = weight_name[: -len(".weight")]
    return f"{base}.weight", f"{base}.weight_scale", f"{base}.comfy_quant"


def missing_sources(plan: list[Op], keys) -> list[str]:
    keys = set(keys)
    return sorted({s for op in plan for s in op.src if s not in keys})
