"""Qwen-Image engine (registry ``qwen_image``): 60 dual-stream blocks, true CFG 4.0.

Reference: ``difflet/models/qwen_image/*`` (true-CFG combine
``difflet/models/qwen_image/pipeline.py:450``).  The VAE is the Wan-style causal
decoder applied to one frame.  ``quant="mxfp8"`` routes the block linears
through the block-scaled MXFP8 GEMM (``difflet_b200/quant``).
"""

from __future__ import annotations

from difflet_b200.models.mmdit.entry import MMDiTEngine
from difflet_b200.models.vae.wan_vae import WanVAEConfig, WanVAEDecoder


class QwenImageEngine(MMDiTEngine):
    preset = "qwen-image"
    default_shape = {"height": 1328, "width": 1328}
    text_family = "qwen_image"

    def make_vae(self, dev):
        if self.kw.get("random_init") or not self.model_path:
            return WanVAEDecoder.random_init(WanVAEConfig(), device=dev, dtype=self.dtype, seed=7)
        from difflet_b200.utils.checkpoint import load_component

        return WanVAEDecoder(WanVAEConfig(), load_component(self.model_path, "vae", dtype=self.dtype, device=dev))

    def app_kwargs(self):
        return {"flow_shift": None, "text_len": 256, "true_cfg": True, "cfg_rescale": True}

    def generate(self, **kw):
        kw.setdefault("guidance_scale", 4.0)
        kw.setdefault("num_inference_steps", 50)
        return super().generate(**kw)


def create_application(**kw):
    return QwenImageEngine(**kw)
