"""Wan application factory (registry entry ``wan``): Wan 2.2 A14B (two experts) or 2.1 (one).

Lifecycle as the reference GPU flow (``difflet/backends/gpu/application.py:84-481``,
``difflet/backends/cuda/wan/application.py:52-336``): ``compile()`` verifies the
native kernels, ``load()`` materialises the expert(s) and the VAE on this rank's
GPU (checkpoint components ``transformer``, ``transformer_2``, ``vae`` or
seeded random init), sets up Ulysses (cp axis) and CFG-parallel (cfg axis)
contexts, and ``generate()`` runs text-to-video.
"""

from __future__ import annotations

import torch

from difflet_b200.models.vae.wan_vae import WanVAEConfig, WanVAEDecoder
from difflet_b200.models.wan.model import WanTransformer, get_wan_config
from difflet_b200.models.wan.pipeline import WanApplication


class WanEngine:
    def __init__(self, *, entry, model_path, parallel, dtype, shape, backend, application_kwargs):
        self.entry, self.model_path, self.parallel, self.dtype = entry, model_path, parallel, dtype
        self.shape, self.backend = shape, backend
        self.kw = dict(application_kwargs or {})
        mp = str(model_path or self.kw.get("preset", "")).lower()
        self.two_experts = "2.1" not in mp and not self.kw.get("single_expert")
        self.wcfg = get_wan_config(self.kw.get("preset") or ("wan2.2-t2v-a14b" if self.two_experts else "wan2.1-t2v-14b"))
        self.app: WanApplication | None = None

    def compile(self, compiled_path):
        info = {"backend": self.backend, "experts": 2 if self.two_experts else 1}
        if self.backend == "cuda":
            from difflet_b200 import _native

            _native.require()
            info["kernels"] = _native.source_hash()
        return info

    def load(self, compiled_path=None, skip_warmup=False):
        dev = torch.device("cuda", torch.cuda.current_device()) if self.backend == "cuda" else torch.device("cpu")
        n = 2 if self.two_experts else 1
        from difflet_b200.utils.hbm import preload_check

        preload_check(WanTransformer.weight_shapes(self.wcfg), self.dtype, dev, what="Wan experts", copies=n)
        if self.kw.get("random_init") or not self.model_path:
            experts = [WanTransformer.random_init(self.wcfg, device=dev, dtype=self.dtype, seed=10 + i) for i in range(n)]
            vae = WanVAEDecoder.random_init(WanVAEConfig(), device=dev, dtype=self.dtype, seed=3)
        else:
            from difflet_b200.utils.checkpoint import load_component

            comps = ["transformer", "transformer_2"][:n]
            experts = [WanTransformer.from_diffusers_state_dict(self.wcfg, load_component(self.model_path, c),
                                                               device=dev, dtype=self.dtype) for c in comps]
            vae = WanVAEDecoder(WanVAEConfig(), load_component(self.model_path, "vae", dtype=self.dtype, device=dev))
        if self.kw.get("host_vae"):  # decode on the host CPU in fp32 (frees the decoder's device memory)
            from difflet_b200.utils.host_vae import move_to_host

            move_to_host(vae)
        seq_par = cfg_par = None
        if self.parallel.world_size > 1:
            from difflet_b200.parallel.ulysses import make_cfg_parallel, make_sequence_parallel

            seq_par = make_sequence_parallel(self.parallel, dev)
            cfg_par = make_cfg_parallel(self.parallel, dev)
        if self.parallel.tp_degree > 1:  # heads / FFN columns over the tp axis (across-heads q/k RMS all-reduced)
            from difflet_b200.parallel.tp import make_tensor_parallel, shard_wan_weights

            tp = make_tensor_parallel(self.parallel, dev)
            for e in experts:
                e.tp = tp
                e.w = shard_wan_weights(e.cfg, e.w, tp.world, tp.rank)
        from difflet_b200.quant.apply import quantize_engine_model

        self.quant_report = [quantize_engine_model(e, "wan", self.kw) for e in experts]
        text_encoder = None
        if self.model_path and not self.kw.get("random_init") and self.kw.get("load_text_encoder", True):
            from difflet_b200.models.text_encoders import load_text_encoder

            text_encoder = load_text_encoder("wan", self.model_path, dev, self.dtype, text_len=experts[0].cfg.text_len)
        self.app = WanApplication(experts, vae, flow_shift=float(self.kw.get("flow_shift", 12.0 if n == 2 else 5.0)),
                                  text_encoder=text_encoder, cfg_par=cfg_par, seq_par=seq_par)

    def generate(self, **kw):
        kw.setdefault("height", self.shape.get("height") or 720)
        kw.setdefault("width", self.shape.get("width") or 1280)
        kw.setdefault("num_frames", self.shape.get("num_frames") or 81)
        return self.app.generate(**kw)

    def __call__(self, *args, **kw):
        if args and isinstance(args[0], str):
            kw["prompt"] = args[0]
        return self.generate(**kw)


def create_application(**kw):
    return WanEngine(**kw)
