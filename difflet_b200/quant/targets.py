"""Which linears each DiT runs in MXFP8 (torch-free): regexes over diffusers module names.

The default sets follow the reference's per-model tables (difflet/quant/targets.py):
the per-token projections (q/k/v, MLP up/down, FLUX / HunyuanVideo single-block
MLP-up and the two halves of their fused ``proj_out``) are targets; everything that
conditions the blocks (adaLN modulation, embedders, ``norm_out``, ``proj_out``) and
the attention output projections stay bf16.  The patterns must name the same
checkpoint keys as the reference's, so quantized checkpoints and
``DIFFLET_QUANT_TARGETS`` overrides carry over unchanged.  HunyuanVideo-1.5 has no
default set: it needs explicit targets.
"""

from __future__ import annotations

import os

from difflet_b200.quant.spec import QuantSpec

DUAL = r"transformer_blocks\.\d+"
SINGLE = r"single_transformer_blocks\.\d+"
WAN_BLOCK = r"blocks\.\d+"
SINGLE_PROJ_OUT_SPLIT = (rf"{SINGLE}\.proj_out",)

TARGETS = {
    "flux": (
        rf"{DUAL}\.attn\.(to_q|to_k|to_v|add_q_proj|add_k_proj|add_v_proj)",
        rf"{DUAL}\.(ff|ff_context)\.net\.(0\.proj|2)",
        rf"{SINGLE}\.attn\.(to_q|to_k|to_v)",
        rf"{SINGLE}\.proj_mlp",
        rf"{SINGLE}\.proj_out_(attn|mlp)",
    ),
    "qwen_image": (
        rf"{DUAL}\.attn\.(to_q|to_k|to_v|add_q_proj|add_k_proj|add_v_proj)",
        rf"{DUAL}\.(img_mlp|txt_mlp)\.net\.(0\.proj|2)",
    ),
    "wan": (
        rf"{WAN_BLOCK}\.attn2\.(to_q|to_k|to_v)",
        rf"{WAN_BLOCK}\.ffn\.net\.(0\.proj|2)",
    ),
    "hunyuan_video": (
        rf"{DUAL}\.attn\.(add_q_proj|add_k_proj|add_v_proj)",
        rf"{DUAL}\.(ff|ff_context)\.net\.(0\.proj|2)",
        rf"{SINGLE}\.proj_mlp",
        rf"{SINGLE}\.proj_out_(attn|mlp)",
    ),
    "hunyuan_video_15": (),
    "ltx_2": (
        rf"{DUAL}\.(attn1|attn2)\.(to_q|to_k|to_v)",
        rf"{DUAL}\.audio_to_video_attn\.to_q",
        rf"{DUAL}\.video_to_audio_attn\.(to_k|to_v)",
        rf"{DUAL}\.ff\.net\.(0\.proj|2)",
    ),
}

ROW_PARALLEL = {
    "flux": (rf"{DUAL}\.attn\.(to_out\.0|to_add_out)", rf"{DUAL}\.(ff|ff_context)\.net\.2",
             rf"{SINGLE}\.proj_out_(attn|mlp)"),
    "qwen_image": (rf"{DUAL}\.attn\.(to_out\.0|to_add_out)", rf"{DUAL}\.(img_mlp|txt_mlp)\.net\.2"),
    "wan": (rf"{WAN_BLOCK}\.(attn1|attn2)\.to_out\.0", rf"{WAN_BLOCK}\.ffn\.net\.2"),
    "hunyuan_video": (rf"{DUAL}\.attn\.(to_out\.0|to_add_out)", rf"{DUAL}\.(ff|ff_context)\.net\.2",
                      rf"{SINGLE}\.proj_out_(attn|mlp)",
                      r"context_embedder\.token_refiner\.refiner_blocks\.\d+\.(attn\.to_out\.0|ff\.net\.2)"),
    "hunyuan_video_15": (rf"{DUAL}\.attn\.(to_out\.0|to_add_out)", rf"{DUAL}\.(ff|ff_context)\.net\.2",
                         r"context_embedder\.token_refiner\.refiner_blocks\.\d+\.(attn\.to_out\.0|ff\.net\.2)"),
    "ltx_2": (rf"{DUAL}\.(attn1|attn2|audio_attn1|audio_attn2|audio_to_video_attn|video_to_audio_attn)\.to_out\.0",
              rf"{DUAL}\.(ff|audio_ff)\.net\.2"),
}

SPLITS = {"flux": SINGLE_PROJ_OUT_SPLIT, "hunyuan_video": SINGLE_PROJ_OUT_SPLIT}

# HunyuanVideo-1.5 override groups (image / text q/k/v, image / text MLP)
HUNYUAN_VIDEO_15_GROUPS = {
    "G1": rf"{DUAL}\.attn\.(to_q|to_k|to_v)",
    "G2": rf"{DUAL}\.attn\.(add_q_proj|add_k_proj|add_v_proj)",
    "G3": rf"{DUAL}\.ff\.net\.(0\.proj|2)",
    "G4": rf"{DUAL}\.ff_context\.net\.(0\.proj|2)",
}


def targets_for(model: str) -> tuple[str, ...]:
    if model not in TARGETS:
        raise ValueError(f"no MXFP8 target layers are defined for {model!r}; models with MXFP8: {sorted(TARGETS)}")
    return TARGETS[model]


def env_targets() -> tuple[str, ...] | None:
    """``DIFFLET_QUANT_TARGETS``: comma-separated patterns, or HunyuanVideo-1.5 group names."""
    raw = os.environ.get("DIFFLET_QUANT_TARGETS", "").strip()
    if not raw:
        return None
    return tuple(HUNYUAN_VIDEO_15_GROUPS.get(p.strip(), p.strip()) for p in raw.split(",") if p.strip())


def default_spec(model: str, **overrides) -> QuantSpec:
    overrides.setdefault("row_parallel", ROW_PARALLEL.get(model, ()))
    if "targets" not in overrides:
        env = env_targets()
        overrides["targets"] = env if env is not None else targets_for(model)
        if not overrides["targets"]:
            raise ValueError(f"{model!r} has no default MXFP8 target set; name the layers with targets= "
                             f"(DIFFLET_QUANT_TARGETS on the CLI)")
    overrides.setdefault("split_linears", SPLITS.get(model, ()))
    return QuantSpec(**overrides)


__all__ = ["HUNYUAN_VIDEO_15_GROUPS", "ROW_PARALLEL", "SPLITS", "TARGETS", "default_spec", "env_targets",
           "targets_for"]
