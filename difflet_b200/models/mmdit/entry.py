"""Generic engine for MMDiT registry entries (HunyuanVideo, HunyuanVideo 1.5, Qwen-Image).

Lifecycle as the reference GPU flow (``difflet/backends/gpu/application.py:84-481``):
``compile()`` verifies the native kernels; ``load()`` builds the DiT and VAE on this
rank's GPU from the diffusers checkpoint components or seeded random init, sets up
Ulysses (cp axis) and CFG-parallel (cfg axis) contexts; ``generate()`` runs.
"""

from __future__ import annotations

import torch

from difflet_b200.models.mmdit.config import get_config
from difflet_b200.models.mmdit.model import MMDiT
from difflet_b200.models.mmdit.pipeline import MMDiTApplication


class MMDiTEngine:
    preset = "hunyuan-video"
    default_shape = {"height": 720, "width": 1280, "num_frames": 129}
    text_family = None  # prompt-encoder recipe of models/text_encoders.py (None: synthetic embeddings)

    def __init__(self, *, entry, model_path, parallel, dtype, shape, backend, application_kwargs):
        self.entry, self.model_path, self.parallel, self.dtype = entry, model_path, parallel, dtype
        self.shape, self.backend = shape, backend
        self.kw = dict(application_kwargs or {})
        self.cfg = get_config(self.kw.get("preset") or self.preset)
        self.app = None

    def compile(self, compiled_path):
        info = {"backend": self.backend, "family": self.cfg.family}
        if self.backend == "cuda":
            from difflet_b200 import _native

            _native.require()
            info["kernels"] = _native.source_hash()
        return info

    def make_vae(self, dev):
        raise NotImplementedError

    def app_kwargs(self):
        return {}

    def load(self, compiled_path=None, skip_warmup=False):
        dev = torch.device("cuda", torch.cuda.current_device()) if self.backend == "cuda" else torch.device("cpu")
        from difflet_b200.utils.hbm import preload_check

        preload_check(MMDiT.weight_shapes(self.cfg), self.dtype, dev, what=f"{self.entry.name} DiT")
        if self.kw.get("random_init") or not self.model_path:
            dit = MMDiT.random_init(self.cfg, device=dev, dtype=self.dtype, seed=int(self.kw.get("seed", 0)))
        else:
            from difflet_b200.utils.checkpoint import load_component

            dit = MMDiT.from_diffusers_state_dict(self.cfg, load_component(self.model_path, "transformer"),
                                                  device=dev, dtype=self.dtype)
        if self.parallel.tp_degree > 1:  # this rank's heads / MLP columns, before any quantization
            from difflet_b200.parallel.tp import make_tensor_parallel, shard_mmdit_weights

            dit.tp = make_tensor_parallel(self.parallel, dev)
            dit.w = shard_mmdit_weights(dit.cfg, dit.w, dit.tp.world, dit.tp.rank)
        from difflet_b200.quant.apply import quantize_engine_model

        self.quant_report = quantize_engine_model(dit, self.entry.name, self.kw)
        vae = self.make_vae(dev)
        cfg_par = None
        if self.parallel.world_size > 1:
            from difflet_b200.parallel.ulysses import make_cfg_parallel, make_sequence_parallel

            dit.par = make_sequence_parallel(self.parallel, dev)
            cfg_par = make_cfg_parallel(self.parallel, dev)
        kwargs = self.app_kwargs()
        if (self.text_family and self.model_path and not self.kw.get("random_init")
                and self.kw.get("load_text_encoder", True) and "text_encoder" not in kwargs):
            from difflet_b200.models.text_encoders import load_text_encoder

            te = load_text_encoder(self.text_family, self.model_path, dev, self.dtype, max_len=kwargs.get("text_len"))
            if te is not None:
                kwargs["text_encoder"] = te
        self.app = MMDiTApplication(dit, vae, cfg_par=cfg_par, **kwargs)

    def generate(self, **kw):
        for k, v in self.default_shape.items():
            kw.setdefault(k, self.shape.get(k) or v)
        return self.app.generate(**kw)

    def __call__(self, *args, **kw):
        if args and isinstance(args[0], str):
            kw["prompt"] = args[0]
        return self.generate(**kw)
