"""LTX-2 engine (registry ``ltx_2``): text -> video + audio.

Lifecycle of the other engines (difflet/models/ltx_2/entry.py, the reference's GPU
application ``difflet/backends/cuda/ltx_2/application.py``): ``compile()`` checks the
native kernels, ``load()`` builds the DiT (checkpoint ``transformer`` component or
seeded random init) and the decoders, CFG-parallel over the cfg axis, MXFP8 by
``quant="mxfp8"``; ``generate()`` returns frames, waveform, fps and sample rate.
"""

from __future__ import annotations

import torch

from difflet_b200.models.ltx_2.model import LTX2Transformer, get_ltx2_config
from difflet_b200.models.ltx_2.pipeline import LTX2Application
from difflet_b200.models.ltx_2.vae import TINY_DECODER, LTX2DecoderConfig, LTX2Decoders


class LTX2Engine:
    default_shape = {"height": 512, "width": 768, "num_frames": 121}

    def __init__(self, *, entry, model_path, parallel, dtype, shape, backend, application_kwargs):
        self.entry, self.model_path, self.parallel, self.dtype = entry, model_path, parallel, dtype
        self.shape, self.backend = shape, backend
        self.kw = dict(application_kwargs or {})
        self.cfg = get_ltx2_config(self.kw.get("preset") or "ltx-2")
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
        dcfg = TINY_DECODER if self.cfg.in_channels != 128 else LTX2DecoderConfig()
        from difflet_b200.utils.hbm import preload_check

        preload_check(LTX2Transformer.weight_shapes(self.cfg), self.dtype, dev, what="LTX-2 DiT")
        if self.kw.get("random_init") or not self.model_path:
            dit = LTX2Transformer.random_init(self.cfg, device=dev, dtype=self.dtype, seed=int(self.kw.get("seed", 0)))
        else:
            from difflet_b200.models.ltx_2.weights import from_diffusers
            from difflet_b200.utils.checkpoint import load_component

            dit = LTX2Transformer(self.cfg, from_diffusers(self.cfg, load_component(self.model_path, "transformer")))
            dit.to(dev, self.dtype)
        decoders = LTX2Decoders.random_init(dcfg, device=dev, dtype=self.dtype, seed=5)
        cfg_par = None
        if self.parallel.world_size > 1:
            if self.parallel.cp_degree > 1 or self.parallel.tp_degree > 1:
                raise NotImplementedError("LTX-2 runs single-GPU or CFG-parallel here")
            from difflet_b200.parallel.ulysses import make_cfg_parallel

            cfg_par = make_cfg_parallel(self.parallel, dev)
        from difflet_b200.quant.apply import quantize_engine_model

        self.quant_report = quantize_engine_model(dit, "ltx_2", self.kw)
        self.app = LTX2Application(dit, decoders, cfg_par=cfg_par)

    def generate(self, **kw):
        for k, v in self.default_shape.items():
            kw.setdefault(k, self.shape.get(k) or v)
        kw.setdefault("num_inference_steps", 40)
        kw.setdefault("guidance_scale", 4.0)
        return self.app.generate(**kw)

    def __call__(self, *args, **kw):
        if args and isinstance(args[0], str):
            kw["prompt"] = args[0]
        return self.generate(**kw)


def create_application(**kw):
    return LTX2Engine(**kw)
