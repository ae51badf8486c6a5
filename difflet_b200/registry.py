"""Model registry: ``@register_model``, ``ModelEntry``, ``ModelCapabilities``, built-in entries.

Same contract as the reference registry (``difflet/registry.py:20-235``): an
entry carries the HF ids that select it, a default parallel config and shape,
the parallel capabilities (head count for divisibility, distilled vs true-CFG,
CP/SP support and CP modes), the download allow-list, and a lazily imported
application factory.  The default parallel configs are the B200 ones (every
mode is native on this engine).
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from typing import Any, Callable

from difflet_b200.pipeline.parallel_config import CP_MODES, DiffletParallelConfig

_ALL_CP_MODES = frozenset(CP_MODES)


@dataclass(frozen=True)
class ModelCapabilities:
    num_attention_heads: int
    is_distilled: bool
    supports_cp: bool = True
    supports_sp: bool = True
    cp_modes: frozenset = _ALL_CP_MODES
    true_cfg_backends: frozenset = frozenset({"cuda"})

    def __post_init__(self):
        if self.num_attention_heads < 1:
            raise ValueError("num_attention_heads must be >= 1")
        unknown = set(self.cp_modes) - _ALL_CP_MODES
        if unknown:
            raise ValueError(f"unknown cp_modes: {sorted(unknown)}")
        if not self.supports_cp and self.cp_modes:
            raise ValueError("cp_modes must be empty when supports_cp is False")
        if self.supports_cp and not self.cp_modes:
            raise ValueError("supports_cp requires at least one cp_mode")

    @property
    def supports_cfg_parallel(self) -> bool:
        return not self.is_distilled

    def check_parallel(self, p: DiffletParallelConfig) -> None:
        H = self.num_attention_heads
        if H % p.tp_degree:
            raise ValueError(f"tp_degree={p.tp_degree} does not divide {H} heads")
        if p.cp_degree > 1:
            if not self.supports_cp:
                raise ValueError("model does not support context parallelism")
            if p.cp_mode not in self.cp_modes:
                raise ValueError(f"cp_mode {p.cp_mode!r} not supported (have {sorted(self.cp_modes)})")
            if p.cp_mode == "ulysses" and H % (p.tp_degree * p.cp_degree):
                raise ValueError(f"ulysses needs heads % (tp*cp) == 0: {H} % {p.tp_degree * p.cp_degree}")
        if p.sp_enabled and not self.supports_sp:
            raise ValueError("model does not support sequence parallelism")
        if p.cfg_parallel_enabled and not self.supports_cfg_parallel:
            raise ValueError("cfg-parallel needs a true-CFG model (this one is guidance-distilled)")


@dataclass(frozen=True)
class ModelEntry:
    name: str
    application_factory: Any  # callable or "module:function"
    hf_paths: tuple = ()
    detector: Callable[[str], bool] | None = None
    default_parallel: DiffletParallelConfig = field(default_factory=DiffletParallelConfig)
    default_shape: dict = field(default_factory=dict)
    capabilities: ModelCapabilities | None = None
    backends: tuple = ("cuda", "cpu")
    download_patterns: tuple | None = None
    output: str = "image"  # "image" | "video"

    def matches(self, model_id: str) -> bool:
        mid = model_id.rstrip("/")
        if mid in self.hf_paths or mid == self.name:
            return True
        return bool(self.detector(model_id)) if self.detector else False

    def resolve_shape(self, *, height=None, width=None, num_frames=None) -> dict:
        s = dict(self.default_shape)
        if height is not None:
            s["height"] = height
        if width is not None:
            s["width"] = width
        if num_frames is not None:
            s["num_frames"] = num_frames
        return s

    def require_backend(self, backend: str) -> None:
        if backend not in self.backends:
            raise ValueError(f"model {self.name!r} does not support backend {backend!r} (has {self.backends})")

    def create_application(self, **kwargs):
        fac = self.application_factory
        if isinstance(fac, str):
            mod, fn = fac.split(":")
            fac = getattr(importlib.import_module(mod), fn)
        return fac(entry=self, **kwargs)


_REGISTRY: dict[str, ModelEntry] = {}


def register_model(entry: ModelEntry | None = None, **kwargs):
    """Register an entry directly, or decorate an application factory:
    ``@register_model(name=..., hf_paths=...)``."""
    if entry is not None:
        _REGISTRY[entry.name] = entry
        return entry

    def deco(factory):
        _REGISTRY[kwargs["name"]] = ModelEntry(application_factory=factory, **kwargs)
        return factory

    return deco


def registered_models() -> dict[str, ModelEntry]:
    _ensure_builtins()
    return dict(_REGISTRY)


def resolve_model(model_id: str, model_type: str | None = None) -> ModelEntry:
    _ensure_builtins()
    if model_type is not None:
        if model_type not in _REGISTRY:
            raise ValueError(f"unknown model_type {model_type!r}; known: {sorted(_REGISTRY)}")
        return _REGISTRY[model_type]
    for e in _REGISTRY.values():
        if e.matches(model_id):
            return e
    raise ValueError(f"no registered model matches {model_id!r}; known: {sorted(_REGISTRY)}")


_BUILTINS_DONE = False


def _ensure_builtins():
    global _BUILTINS_DONE
    if _BUILTINS_DONE:
        return
    _BUILTINS_DONE = True
    P = DiffletParallelConfig
    register_model(ModelEntry(
        name="flux", application_factory="difflet_b200.models.flux.entry:create_application",
        hf_paths=("black-forest-labs/FLUX.1-dev", "black-forest-labs/FLUX.1-schnell", "flux-dev", "flux-schnell"),
        detector=lambda m: "flux" in m.lower() and "flux.2" not in m.lower(),
        default_parallel=P(), default_shape={"height": 1024, "width": 1024, "num_frames": None},
        capabilities=ModelCapabilities(num_attention_heads=24, is_distilled=True)))
    register_model(ModelEntry(
        name="wan", application_factory="difflet_b200.models.wan.entry:create_application",
        hf_paths=("Wan-AI/Wan2.2-T2V-A14B-Diffusers", "Wan-AI/Wan2.1-T2V-14B-Diffusers", "wan2.2-t2v-a14b", "wan2.1-t2v-14b"),
        detector=lambda m: "wan" in m.lower(),
        default_parallel=P(), default_shape={"height": 720, "width": 1280, "num_frames": 81},
        capabilities=ModelCapabilities(num_attention_heads=40, is_distilled=False), output="video"))
    register_model(ModelEntry(
        name="hunyuan_video", application_factory="difflet_b200.models.hunyuan_video.entry:create_application",
        hf_paths=("hunyuanvideo-community/HunyuanVideo", "tencent/HunyuanVideo", "hunyuan-video"),
        detector=lambda m: "hunyuanvideo" in m.lower().replace("-", "").replace("_", "") and "1.5" not in m,
        default_parallel=P(), default_shape={"height": 720, "width": 1280, "num_frames": 129},
        capabilities=ModelCapabilities(num_attention_heads=24, is_distilled=True), output="video"))
    register_model(ModelEntry(
        name="hunyuan_video_15", application_factory="difflet_b200.models.hunyuan_video.entry:create_application_15",
        hf_paths=("hunyuanvideo-community/HunyuanVideo-1.5-Diffusers-480p_t2v", "hunyuan-video-1.5"),
        detector=lambda m: "hunyuanvideo-1.5" in m.lower() or "hunyuan-video-1.5" in m.lower(),
        default_parallel=P(), default_shape={"height": 480, "width": 848, "num_frames": 121},
        capabilities=ModelCapabilities(num_attention_heads=16, is_distilled=False), output="video"))
    register_model(ModelEntry(
        name="qwen_image", application_factory="difflet_b200.models.qwen_image.entry:create_application",
        hf_paths=("Qwen/Qwen-Image", "qwen-image"), detector=lambda m: "qwen-image" in m.lower(),
        default_parallel=P(), default_shape={"height": 1328, "width": 1328, "num_frames": None},
        capabilities=ModelCapabilities(num_attention_heads=24, is_distilled=False)))
    register_model(ModelEntry(
        name="ltx_2", application_factory="difflet_b200.models.ltx_2.entry:create_application",
        hf_paths=("Lightricks/LTX-2", "ltx-2"), detector=lambda m: "ltx-2" in m.lower() or "ltx2" in m.lower(),
        default_parallel=P(), default_shape={"height": 512, "width": 768, "num_frames": 121},
        capabilities=ModelCapabilities(num_attention_heads=32, is_distilled=False), output="video"))
    register_model(ModelEntry(
        name="minimax_h3", application_factory="difflet_b200.models.minimax_h3.entry:create_application",
        hf_paths=("MiniMaxAI/MiniMax-H3", "minimax-h3"), detector=lambda m: "minimax" in m.lower(),
        default_parallel=P(), default_shape={"height": 480, "width": 832, "num_frames": 124},
        capabilities=ModelCapabilities(num_attention_heads=24, is_distilled=False), output="video"))
