"""difflet_b200 — a Blackwell-native (sm_100a) diffusion-transformer inference engine.

Public API (same names as the reference's ``difflet`` package, ``difflet/__init__.py:16-46``):
    DiffletPipeline        unified entry point (``DiffletPipeline.from_pretrained(...)``)
    DiffletParallelConfig  TP / SP / CP / CFG-parallel / DP configuration
    CandidateConfig        candidate (N) axis, cache-key only
    current_backend        active backend name (``cuda`` on B200, ``cpu`` oracle)
    register_model         decorator for registering model entries
"""

__all__ = [
    "DiffletPipeline",
    "DiffletParallelConfig",
    "CandidateConfig",
    "current_backend",
    "register_model",
]

__version__ = "0.1.0"


def __getattr__(name: str):
    if name == "DiffletPipeline":
        from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline

        return DiffletPipeline
    if name == "DiffletParallelConfig":
        from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

        return DiffletParallelConfig
    if name == "CandidateConfig":
        from difflet_b200.pipeline.parallel_config import CandidateConfig

        return CandidateConfig
    if name == "current_backend":
        from difflet_b200.platforms import current_backend

        return current_backend
    if name == "register_model":
        from difflet_b200.registry import register_model

        return register_model
    raise AttributeError(f"module 'difflet_b200' has no attribute {name!r}")
