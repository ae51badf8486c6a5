"""Apply an MXFP8 spec to a loaded model's fused weights.

The built-in models fuse several diffusers linears into one GEMM (q|k|v, FLUX's
single-block [q|mlp|k|v], the single-block ``proj_out`` over [attn|mlp]).  A fused
matrix runs in MXFP8 when every diffusers linear it holds is a target (for the split
``proj_out`` its ``_attn`` and ``_mlp`` halves); a fused matrix with only some of
its parts targeted stays bf16 and is reported in ``partial``.  Because OCP blocks
run along K, the fused matrix's scales equal its parts' scales, so a quantized
checkpoint (whose FP8 weights dequantize exactly to bf16 and re-quantize to the
same bits) loads through the same path.
"""

from __future__ import annotations

import torch

from difflet_b200.ops import fused as F
from difflet_b200.quant.spec import QuantSpec


def mmdit_fused_parts(cfg) -> dict[str, list[str]]:
    """Fused weight key -> the diffusers linears it holds (MMDiT families)."""
    from difflet_b200.models.mmdit.weights import _names

    nm = _names(cfg)
    parts = {}
    for i in range(cfg.double_blocks):
        p, q = f"transformer_blocks.{i}.", f"double.{i}."
        a = p + "attn."
        parts[q + "img_qkv.w"] = [a + n for n in ("to_q", "to_k", "to_v")]
        parts[q + "txt_qkv.w"] = [a + n for n in ("add_q_proj", "add_k_proj", "add_v_proj")]
        parts[q + "img_out.w"] = [a + "to_out.0"]
        parts[q + "txt_out.w"] = [a + "to_add_out"]
        for st in ("img", "txt"):
            parts[q + st + "_up.w"] = [p + nm[st + "_up"]]
            parts[q + st + "_down.w"] = [p + nm[st + "_down"]]
    for j in range(cfg.single_blocks):
        p, q = f"single_transformer_blocks.{j}.", f"single.{j}."
        parts[q + "fused.w"] = [p + "attn.to_q", p + "proj_mlp", p + "attn.to_k", p + "attn.to_v"]
        parts[q + "proj.w"] = [p + "proj_out_attn", p + "proj_out_mlp"]
    return parts


def wan_fused_parts(cfg) -> dict[str, list[str]]:
    parts = {}
    for i in range(cfg.layers):
        p, q = f"blocks.{i}.", f"blk.{i}."
        parts[q + "qkv.w"] = [p + "attn1." + n for n in ("to_q", "to_k", "to_v")]
        parts[q + "o.w"] = [p + "attn1.to_out.0"]
        parts[q + "cq.w"] = [p + "attn2.to_q"]
        parts[q + "ckv.w"] = [p + "attn2.to_k", p + "attn2.to_v"]
        parts[q + "co.w"] = [p + "attn2.to_out.0"]
        parts[q + "up.w"] = [p + "ffn.net.0.proj"]
        parts[q + "down.w"] = [p + "ffn.net.2"]
    return parts


def ltx2_fused_parts(cfg) -> dict[str, list[str]]:
    parts = {}
    for i in range(cfg.layers):
        p, q = f"transformer_blocks.{i}.", f"blk.{i}."
        for st, mod in (("v", "attn1"), ("a", "audio_attn1")):
            parts[q + st + "_qkv.w"] = [p + mod + "." + n for n in ("to_q", "to_k", "to_v")]
            parts[q + st + "_o.w"] = [p + mod + ".to_out.0"]
        for pre, mod in (("v_c", "attn2"), ("a_c", "audio_attn2"), ("a2v_", "audio_to_video_attn"),
                         ("v2a_", "video_to_audio_attn")):
            parts[q + pre + "q.w"] = [p + mod + ".to_q"]
            parts[q + pre + "kv.w"] = [p + mod + ".to_k", p + mod + ".to_v"]
            parts[q + pre + "o.w"] = [p + mod + ".to_out.0"]
        for st, ff in (("v", "ff"), ("a", "audio_ff")):
            parts[q + st + "_up.w"] = [p + ff + ".net.0.proj"]
            parts[q + st + "_down.w"] = [p + ff + ".net.2"]
    return parts


def apply_to_weights(w: dict, parts: dict[str, list[str]], spec: QuantSpec) -> dict[str, list[str]]:
    """Replace every fully targeted fused weight of ``w`` by an ``MXWeight`` (in place)."""
    done, partial = [], []
    for key, names in parts.items():
        hits = [spec.matches(n) for n in names]
        if all(hits):
            t = w[key]
            if t.shape[1] % 128:
                partial.append(key)
                continue
            w[key] = F.MXWeight.quantize(t, compute=spec.compute)
            done.append(key)
        elif any(hits):
            partial.append(key)
    return {"quantized": done, "partial": partial}


def apply_quant(model, spec: QuantSpec) -> dict[str, list[str]]:
    """Quantize the model's targeted fused weights (MMDiT families or Wan)."""
    cfg = model.cfg
    if hasattr(cfg, "double_blocks"):
        parts = mmdit_fused_parts(cfg)
    elif "blk.0.v_qkv.w" in model.w:
        parts = ltx2_fused_parts(cfg)
    elif hasattr(cfg, "layers") and "blk.0.qkv.w" in model.w:
        parts = wan_fused_parts(cfg)
    else:
        raise NotImplementedError(f"no MXFP8 mapping for {type(model).__name__}")
    res = apply_to_weights(model.w, parts, spec)
    if not res["quantized"]:
        raise ValueError(f"the spec quantizes no fused weight of this model (partial: {res['partial'][:4]})")
    model.quant_spec = spec
    return res


def dequantize_state_dict(sd: dict[str, torch.Tensor], dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """A quantized checkpoint's state dict back to ``dtype`` (exact for bf16); split
    ``proj_out_attn`` / ``proj_out_mlp`` halves are joined into ``proj_out``."""
    from difflet_b200.ops.mx import dequantize_mx

    out = {}
    for k, t in sd.items():
        if k.endswith(".weight_scale"):
            continue
        if k.endswith(".weight") and t.dtype == torch.float8_e4m3fn:
            out[k] = dequantize_mx(t, sd[k[:-7] + ".weight_scale"], output_dtype=dtype)
        else:
            out[k] = t.to(dtype) if t.is_floating_point() else t
    for k in [k for k in out if k.endswith("proj_out_attn.weight")]:
        base = k[: -len("_attn.weight")]
        out[base + ".weight"] = torch.cat([out.pop(k), out.pop(base + "_mlp.weight")], 1)
        if base + "_attn.bias" in out:
            out[base + ".bias"] = out.pop(base + "_attn.bias")
    return out


__all__ = ["apply_quant", "apply_to_weights", "dequantize_state_dict", "mmdit_fused_parts", "wan_fused_parts"]


def spec_from_kwargs(model_name: str, kw: dict) -> QuantSpec | None:
    """The spec an engine's application kwargs ask for (``quant="mxfp8"``,
    ``quant_compute`` "native" / "mx" / "dequant", optional ``quant_targets``)."""
    if not kw.get("quant"):
        return None
    if kw["quant"] != "mxfp8":
        raise ValueError(f"quant must be 'mxfp8', got {kw['quant']!r}")
    from difflet_b200.quant.targets import default_spec

    compute = {"native": "mx", "nki": "mx"}.get(kw.get("quant_compute", "mx"), kw.get("quant_compute", "mx"))
    over = {"compute": compute}
    if kw.get("quant_targets"):
        over["targets"] = tuple(kw["quant_targets"])
    return default_spec(model_name, **over)


def quantize_engine_model(dit, model_name: str, kw: dict):
    """Apply the engine's quant request to its DiT (no-op without one); returns the report."""
    spec = spec_from_kwargs(model_name, kw)
    if spec is None:
        return None
    return apply_quant(dit, spec)
