"""DiffletPipeline public API over every registry entry (CPU backend, tiny random-init presets)."""

import json

import pytest
import torch

from difflet_b200 import DiffletParallelConfig, DiffletPipeline
from difflet_b200.pipeline.compile_cache import cache_key, read_manifest
from difflet_b200.registry import registered_models, resolve_model

CASES = [
    ("black-forest-labs/FLUX.1-dev", "tiny128", dict(height=64, width=64, num_inference_steps=2)),
    ("Wan-AI/Wan2.2-T2V-A14B-Diffusers", "tiny-wan", dict(height=32, width=32, num_frames=5, num_inference_steps=2)),
    ("hunyuanvideo-community/HunyuanVideo", "tiny-hunyuan", dict(height=32, width=32, num_frames=5,
                                                                  num_inference_steps=2)),
    ("Qwen/Qwen-Image", "tiny-qwen", dict(height=32, width=32, num_inference_steps=2)),
]


@pytest.mark.parametrize("model_id,preset,kw", CASES)
def test_from_pretrained_and_generate(tmp_path, monkeypatch, model_id, preset, kw):
    monkeypatch.setenv("DIFFLET_BACKEND", "cpu")
    pipe = DiffletPipeline.from_pretrained(model_id, random_init=True, compile_cache_dir=str(tmp_path),
                                           dtype=torch.float32, application_kwargs={"preset": preset})
    m = read_manifest(pipe.compiled_path)
    assert m is not None and m["key"] == cache_key(pipe.cache_spec)
    if preset == "tiny128":
        out = pipe(prompt="a photo", output_type="latent", **kw)
    else:
        out = pipe(prompt="a photo", output_type="latent", **kw)
    assert torch.isfinite(out).all()
    # second construction hits the cache (same key, no recompile needed)
    pipe2 = DiffletPipeline.from_pretrained(model_id, random_init=True, compile_cache_dir=str(tmp_path),
                                            dtype=torch.float32, application_kwargs={"preset": preset}, load=False)
    assert pipe2.compiled_path == pipe.compiled_path


def test_registry_resolution_and_capabilities():
    models = registered_models()
    for name in ("flux", "wan", "hunyuan_video", "hunyuan_video_15", "qwen_image", "ltx_2", "minimax_h3"):
        assert name in models
    assert resolve_model("black-forest-labs/FLUX.1-dev").name == "flux"
    assert resolve_model("Wan-AI/Wan2.2-T2V-A14B-Diffusers").name == "wan"
    caps = resolve_model("flux").capabilities
    with pytest.raises(ValueError):
        caps.check_parallel(DiffletParallelConfig(cfg_parallel_enabled=True))  # distilled: no CFG branches
    with pytest.raises(ValueError):
        caps.check_parallel(DiffletParallelConfig(cp_degree=5, cp_mode="ulysses"))  # 24 % 5 != 0
    caps.check_parallel(DiffletParallelConfig(cp_degree=8, cp_mode="ulysses"))


def test_parallel_config_rules():
    with pytest.raises(ValueError):
        DiffletParallelConfig(cp_mode="ring")
    with pytest.raises(ValueError):
        DiffletParallelConfig(sp_enabled=True, cp_degree=2, tp_degree=2)
    p = DiffletParallelConfig(tp_degree=2, cp_degree=2, cfg_parallel_enabled=True, cp_mode="ulysses")
    assert p.world_size == 8 and p.mesh_spec.rank_of(cfg=1, cp=1, tp=1) == 7
    assert p.to_cache_dict() == {"tp_degree": 2, "cp_degree": 2, "cfg_parallel_enabled": True, "cp_mode": "ulysses"}


def test_exec_mode_selects_graph_or_eager(monkeypatch):
    """``DIFFLET_EXEC_MODE`` decides whether the FLUX denoise step replays as a CUDA graph."""
    import pytest as _pytest

    from difflet_b200.models.flux.entry import _graph_default

    monkeypatch.delenv("DIFFLET_EXEC_MODE", raising=False)
    assert _graph_default() is True
    monkeypatch.setenv("DIFFLET_EXEC_MODE", "eager")
    assert _graph_default() is False
    monkeypatch.setenv("DIFFLET_EXEC_MODE", "sometimes")
    with _pytest.raises(ValueError):
        _graph_default()
