"""FLUX application factory (registry entry ``flux``).

Lifecycle as in the reference GPU flow (``difflet/backends/gpu/application.py:84-481``):
``compile()`` builds / verifies the native kernels and records the kernel hash
in the manifest; ``load()`` materialises the weights on this rank's GPU
(checkpoint or seeded random init), sets up the sequence-parallel context,
and warms up (capturing the DiT step in a CUDA graph); ``generate()`` /
``__call__`` run text-to-image.
"""

from __future__ import annotations

import torch

from difflet_b200.models.flux.config import FluxConfig, get_config
from difflet_b200.models.flux.model import FluxTransformer
from difflet_b200.models.flux.pipeline import FluxApplication
from difflet_b200.models.vae.autoencoder_kl import KLDecoder, KLDecoderConfig


def _graph_default() -> bool:
    """``DIFFLET_EXEC_MODE``: "graph" (default) replays the denoise step as a CUDA graph,
    "eager" launches its kernels one by one (profiling, debugging)."""
    from difflet_b200 import envs

    mode = str(envs.DIFFLET_EXEC_MODE or "graph").lower()
    if mode not in ("graph", "eager"):
        raise ValueError(f"DIFFLET_EXEC_MODE must be graph or eager, got {mode!r}")
    return mode == "graph"


class FluxEngine:
    def __init__(self, *, entry, model_path, parallel, dtype, shape, backend, application_kwargs):
        self.entry = entry
        self.model_path = model_path
        self.parallel = parallel
        self.dtype = dtype
        self.shape = shape
        self.backend = backend
        self.kw = dict(application_kwargs or {})
        preset = self.kw.get("preset") or ("flux-schnell" if "schnell" in str(model_path).lower() else "flux-dev")
        self.cfg: FluxConfig = get_config(preset)
        self.app: FluxApplication | None = None

    def compile(self, compiled_path):
        info = {"backend": self.backend}
        if self.backend == "cuda":
            from difflet_b200 import _native

            _native.require()
            info["kernels"] = _native.source_hash()
        return info

    def _device(self):
        if self.backend == "cuda":
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device("cpu")

    def load(self, compiled_path=None, skip_warmup=False):
        dev = self._device()
        from difflet_b200.utils.hbm import preload_check

        preload_check(FluxTransformer.weight_shapes(self.cfg), self.dtype, dev, what="FLUX DiT")
        from difflet_b200.quant.apply import quantize_engine_model

        tp = None
        if self.parallel.tp_degree > 1:  # this rank's heads / MLP columns, before any quantization
            from difflet_b200.parallel.tp import make_tensor_parallel

            tp = make_tensor_parallel(self.parallel, dev)

        def device_weights(dit):
            """Checkpoint layout -> this rank's sharded (and quantized) engine weights."""
            if tp is not None:
                from difflet_b200.parallel.tp import shard_mmdit_weights

                dit.w = shard_mmdit_weights(dit.cfg, dit.w, tp.world, tp.rank)
            self.quant_report = quantize_engine_model(dit, "flux", self.kw)
            return dit.w

        if self.kw.get("random_init") or not self.model_path:
            dit = FluxTransformer.random_init(self.cfg, device=dev, dtype=self.dtype, seed=int(self.kw.get("seed", 0)))
            device_weights(dit)
            vae = KLDecoder.random_init(KLDecoderConfig(), device=dev, dtype=self.dtype, seed=1)
        else:
            from difflet_b200.utils import weight_store
            from difflet_b200.utils.checkpoint import load_component

            def build():
                sd = load_component(self.model_path, "transformer", dtype=self.dtype)
                return device_weights(FluxTransformer.from_diffusers_state_dict(self.cfg, sd, device=dev,
                                                                                dtype=self.dtype))

            layout = {"cfg": repr(self.cfg), "quant": self.kw.get("quant"), "compute": self.kw.get("quant_compute")}
            w, self.weight_store = weight_store.load_or_build(
                "flux", self.model_path, self.dtype, tp.world if tp else 1, tp.rank if tp else 0, layout, dev, build,
                compute="mx" if self.kw.get("quant_compute", "native") == "native" else "dequant")
            if self.weight_store == "hit":
                self.quant_report = {"weight_store": "hit"}
            dit = FluxTransformer(self.cfg, w)
            vsd = load_component(self.model_path, "vae", dtype=self.dtype, device=dev)
            vae = KLDecoder(KLDecoderConfig(), vsd)
        if self.kw.get("host_vae"):  # decode on the host CPU in fp32 (frees the decoder's device memory)
            from difflet_b200.utils.host_vae import move_to_host

            move_to_host(vae)
        dit.tp = tp
        if self.parallel.world_size > 1:
            from difflet_b200.parallel.ulysses import make_sequence_parallel

            dit.par = make_sequence_parallel(self.parallel, dev)
        text_encoder = None
        if self.model_path and not self.kw.get("random_init") and self.kw.get("load_text_encoder", True):
            from difflet_b200.models.text_encoders import load_text_encoder

            text_encoder = load_text_encoder("flux", self.model_path, dev, self.dtype,
                                             max_sequence_length=256 if "schnell" in str(self.model_path).lower() else 512)
        self.app = FluxApplication(dit, vae, text_encoder=text_encoder,
                                   use_cuda_graph=(self.backend == "cuda" and self.kw.get("cuda_graph", _graph_default())))
        if self.kw.get("teacache_speedup"):
            from difflet_b200.pipeline.teacache import build_controller

            self.app.teacache = build_controller(self.kw)
        if not skip_warmup and self.backend == "cuda":
            h = self.shape.get("height") or 1024
            w = self.shape.get("width") or 1024
            self.app.generate(prompt="warmup", height=h, width=w, num_inference_steps=2, output_type="latent")
            torch.cuda.synchronize()

    def generate(self, **kw):
        kw.setdefault("height", self.shape.get("height") or 1024)
        kw.setdefault("width", self.shape.get("width") or 1024)
        return self.app.generate(**kw)

    def __call__(self, *args, **kw):
        if args and isinstance(args[0], str):
            kw["prompt"] = args[0]
        return self.generate(**kw)


def create_application(**kw):
    return FluxEngine(**kw)
