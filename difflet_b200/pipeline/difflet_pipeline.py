"""``DiffletPipeline``: the diffusers-style entry point.

Same signature and flow as the reference (``difflet/pipeline/difflet_pipeline.py:16-223``):
resolve the registry entry -> prepare the runtime (bind the GPU, NCCL process
group under torchrun) -> resolve / download the checkpoint -> build the
``CacheSpec`` -> create the application -> ``compile()`` on a cache miss
(native-kernel build + manifest) -> ``load()`` (weights onto the device,
parallel buffers, warm-up / CUDA-graph capture).  ``pipe(prompt=...)`` then
generates.  Offline: ``random_init=True`` builds seeded weights of the named
architecture instead of downloading.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

from difflet_b200.pipeline.compile_cache import (CacheSpec, cache_path, canonicalize_shapes, has_valid_manifest,
                                                 write_manifest)
from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
from difflet_b200.pipeline.path_resolver import resolve_model_path
from difflet_b200.registry import ModelEntry, resolve_model


class DiffletPipeline:
    def __init__(self, *, app, model_id, model_path, model_entry: ModelEntry, compiled_path: Path,
                 cache_spec: CacheSpec, shape, parallel: DiffletParallelConfig, dtype, backend: str):
        self.app = app
        self.model_id = model_id
        self.model_path = model_path
        self.model_entry = model_entry
        self.compiled_path = compiled_path
        self.cache_spec = cache_spec
        self.shape = shape
        self.parallel = parallel
        self.dtype = dtype
        self.backend = backend

    @classmethod
    def from_pretrained(cls, model_id: str, *, parallel: DiffletParallelConfig | None = None, dtype=None,
                        compile_cache_dir: str | None = None, height: int | None = None, width: int | None = None,
                        num_frames: int | None = None, shapes=None, model_type: str | None = None,
                        revision: str | None = None, local_files_only: bool = False, force_compile: bool = False,
                        skip_compile: bool = False, load: bool = True, skip_warmup: bool = False,
                        backend: str | None = None, application_kwargs: dict | None = None,
                        teacache_speedup: float | None = None, teacache_calibration=None,
                        random_init: bool = False, **_ignored) -> "DiffletPipeline":
        import torch

        from difflet_b200.platforms import get_platform

        app_kwargs = dict(application_kwargs or {})
        if teacache_speedup is not None:
            app_kwargs["teacache_speedup"] = teacache_speedup
        if teacache_calibration is not None:
            app_kwargs["teacache_calibration"] = teacache_calibration
        if random_init:
            app_kwargs["random_init"] = True
        canon = None
        if shapes:
            canon = canonicalize_shapes(shapes)
            if height is None and width is None and num_frames is None:
                height, width, num_frames = canon[0]
            app_kwargs["shapes"] = [list(s) for s in canon]
        entry = resolve_model(model_id, model_type=model_type)
        platform = get_platform(backend)
        entry.require_backend(platform.name)
        par = parallel or entry.default_parallel
        if entry.capabilities is not None:
            entry.capabilities.check_parallel(par)
        bad = platform.unsupported_parallel_modes(par)
        if bad:
            raise ValueError(f"backend {platform.name} does not support parallel modes {bad}")
        platform.prepare_runtime(par)
        dtype = dtype if dtype is not None else (torch.bfloat16 if platform.name == "cuda" else torch.float32)
        shape = entry.resolve_shape(height=height, width=width, num_frames=num_frames)
        model_path = resolve_model_path(model_id, revision=revision, local_files_only=local_files_only,
                                        allow_patterns=entry.download_patterns,
                                        random_init=bool(app_kwargs.get("random_init")))
        spec = CacheSpec(model_id=model_id, model_path=model_path, model_name=entry.name, parallel=par,
                         dtype=dtype, height=shape.get("height"), width=shape.get("width"),
                         num_frames=shape.get("num_frames"), revision=revision, application_kwargs=app_kwargs,
                         shapes=tuple(canon) if canon else None, backend=platform.name)
        compiled_path = cache_path(compile_cache_dir, spec)
        app = entry.create_application(model_path=model_path, parallel=par, dtype=dtype, shape=shape,
                                       backend=platform.name, application_kwargs=app_kwargs)
        pipe = cls(app=app, model_id=model_id, model_path=model_path, model_entry=entry,
                   compiled_path=compiled_path, cache_spec=spec, shape=shape, parallel=par, dtype=dtype,
                   backend=platform.name)
        if not skip_compile:
            # one writer per node: local rank 0 builds and writes the manifest, the rest wait
            import torch.distributed as dist

            from difflet_b200 import envs

            if envs.LOCAL_RANK == 0 and (force_compile or not has_valid_manifest(compiled_path, spec)):
                pipe.compile(force=True)
            if dist.is_initialized():
                dist.barrier()
        if load:
            pipe.load(skip_warmup=skip_warmup)
        return pipe

    @classmethod
    def precompile(cls, model_id: str, **kwargs) -> "DiffletPipeline":
        kwargs.setdefault("load", False)
        return cls.from_pretrained(model_id, **kwargs)

    def compile(self, *, force: bool = False, debug: bool = False) -> None:
        if not force and has_valid_manifest(self.compiled_path, self.cache_spec):
            return
        self.compiled_path.mkdir(parents=True, exist_ok=True)
        extra = self.app.compile(self.compiled_path) or {}
        write_manifest(self.compiled_path, self.cache_spec, extra)

    def load(self, *, skip_warmup: bool = False, **_):
        self.app.load(self.compiled_path, skip_warmup=skip_warmup)

    def __call__(self, *args: Any, **kwargs: Any) -> Any:
        from difflet_b200.utils import telemetry

        self._requests = getattr(self, "_requests", 0) + 1
        req = f"r{self._requests:05d}"
        rec = telemetry.StepRecorder.maybe(req)
        if rec is not None:  # chain the per-step observer in front of a user callback
            user = kwargs.get("callback")
            kwargs["callback"] = (lambda i, x: (rec.callback(i, x), user(i, x))) if user else rec.callback
            rec.start()
        with telemetry.span("request", request=req, model=self.model_entry.name), \
                telemetry.nvtx_range(f"difflet.request.{req}"):
            out = self.app(*args, **kwargs)
        if rec is not None:
            rec.finish()
        return out
