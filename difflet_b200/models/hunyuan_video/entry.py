"""HunyuanVideo (registry ``hunyuan_video``) and HunyuanVideo 1.5 (``hunyuan_video_15``) engines.

Reference: ``difflet/models/hunyuan_video/*`` and
``difflet/backends/cuda/hunyuan_video{,_15}/*``.  HunyuanVideo is
guidance-distilled (embedded guidance 6.0, flow shift 7.0); 1.5 runs true CFG
(6.0) on token-refined Qwen2.5-VL text with 32-channel latents.
"""

from __future__ import annotations

from difflet_b200.models.mmdit.entry import MMDiTEngine
from difflet_b200.models.vae.hunyuan_vae import HunyuanVAEConfig, HunyuanVAEDecoder, HunyuanVAENative


def _vae_class(dev):
    """Channels-last native kernels on a GPU; the PyTorch decoder on the CPU."""
    return HunyuanVAENative if getattr(dev, "type", str(dev)) == "cuda" else HunyuanVAEDecoder


class HunyuanVideoEngine(MMDiTEngine):
    preset = "hunyuan-video"
    default_shape = {"height": 720, "width": 1280, "num_frames": 129}
    text_family = "hunyuan_video"

    def make_vae(self, dev):
        if self.kw.get("random_init") or not self.model_path:
            return _vae_class(dev).random_init(HunyuanVAEConfig(), device=dev, dtype=self.dtype, seed=5)
        from difflet_b200.utils.checkpoint import load_component

        return _vae_class(dev)(HunyuanVAEConfig(), load_component(self.model_path, "vae", dtype=self.dtype, device=dev))

    def app_kwargs(self):
        return {"flow_shift": float(self.kw.get("flow_shift", 7.0)), "text_len": 256}


class HunyuanVideo15Engine(HunyuanVideoEngine):
    preset = "hunyuan-video-1.5"
    default_shape = {"height": 480, "width": 848, "num_frames": 121}
    text_family = None  # Qwen2.5-VL + glyph byT5 encoders: synthetic embeddings of the DiT's text width

    def make_vae(self, dev):
        cfg = HunyuanVAEConfig(latent_channels=32, block_out_channels=(128, 256, 512, 1024, 1024))
        if self.kw.get("random_init") or not self.model_path:
            return _vae_class(dev).random_init(cfg, device=dev, dtype=self.dtype, seed=6)
        from difflet_b200.utils.checkpoint import load_component

        return _vae_class(dev)(cfg, load_component(self.model_path, "vae", dtype=self.dtype, device=dev))

    def app_kwargs(self):
        return {"flow_shift": float(self.kw.get("flow_shift", 5.0)), "text_len": 256, "true_cfg": True,
                "cond_channels": self.cfg.in_channels - self.cfg.latent_channels}


def create_application(**kw):
    return HunyuanVideoEngine(**kw)


def create_application_15(**kw):
    return HunyuanVideo15Engine(**kw)
