"""MiniMax-H3 engine (registry ``minimax_h3``): text / first-last keyframes -> video + audio.

Same lifecycle as the other engines (the reference's difflet/models/minimax_h3/
entry.py and application.py): ``compile()`` checks the native kernels, ``load()``
builds the DiT (checkpoint ``transformer`` component or seeded random init) and
the decoders, ``generate()`` runs the guidance-distilled loop.
"""

from __future__ import annotations

import torch

from difflet_b200.models.minimax_h3.model import MiniMaxH3Transformer, get_minimax_config
from difflet_b200.models.minimax_h3.pipeline import MiniMaxH3Application
from difflet_b200.models.minimax_h3.vae import TINY, MiniMaxDecoderConfig, MiniMaxDecoders


class MiniMaxH3Engine:
    default_shape = {"height": 480, "width": 832, "num_frames": 124}

    def __init__(self, *, entry, model_path, parallel, dtype, shape, backend, application_kwargs):
        self.entry, self.model_path, self.parallel, self.dtype = entry, model_path, parallel, dtype
        self.shape, self.backend = shape, backend
        self.kw = dict(application_kwargs or {})
        self.cfg = get_minimax_config(self.kw.get("preset") or "minimax-h3")
        self.app = None

    def compile(self, compiled_path):
        info = {"backend": self.backend, "layers": self.cfg.layers}
        if self.backend == "cuda":
            from difflet_b200 import _native

            _native.require()
            info["kernels"] = _native.source_hash()
        return info

    def load(self, compiled_path=None, skip_warmup=False):
        dev = torch.device("cuda", torch.cuda.current_device()) if self.backend == "cuda" else torch.device("cpu")
        if self.parallel.world_size > 1:
            raise NotImplementedError("MiniMax-H3 runs on one GPU here")
        from difflet_b200.utils.hbm import preload_check

        preload_check(MiniMaxH3Transformer.weight_shapes(self.cfg), self.dtype, dev, what="MiniMax-H3 DiT")
        if self.kw.get("random_init") or not self.model_path:
            dit = MiniMaxH3Transformer.random_init(self.cfg, device=dev, dtype=self.dtype,
                                                   seed=int(self.kw.get("seed", 0)))
        else:
            from difflet_b200.models.minimax_h3.weights import from_diffusers
            from difflet_b200.utils.checkpoint import load_component

            dit = MiniMaxH3Transformer(self.cfg, from_diffusers(self.cfg, load_component(self.model_path,
                                                                                          "transformer")))
            dit.to(dev, self.dtype)
        dcfg = TINY if self.cfg.in_channels != 24 else MiniMaxDecoderConfig()
        text_encoder = None
        if self.model_path and not self.kw.get("random_init") and self.kw.get("load_text_encoder", True):
            from difflet_b200.models.text_encoders import load_text_encoder

            # Qwen3-VL's language model read at hidden_states[50] (the released model's conditioning)
            text_encoder = load_text_encoder("minimax_h3", self.model_path, dev, self.dtype,
                                             text_len=self.kw.get("text_len", 128))
        self.app = MiniMaxH3Application(dit, MiniMaxDecoders.random_init(dcfg, device=dev, dtype=self.dtype),
                                        text_encoder=text_encoder)

    def generate(self, **kw):
        for k, v in self.default_shape.items():
            kw.setdefault(k, self.shape.get(k) or v)
        kw.setdefault("num_inference_steps", 30)
        return self.app.generate(**kw)

    def __call__(self, *args, **kw):
        if args and isinstance(args[0], str):
            kw["prompt"] = args[0]
        return self.generate(**kw)


def create_application(**kw):
    return MiniMaxH3Engine(**kw)
