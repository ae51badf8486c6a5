"""Parallelism configuration (same public fields as the reference).

``DiffletParallelConfig(tp_degree, cp_degree, cfg_parallel_enabled, cp_mode,
sp_enabled, dp_degree)`` with the reference's validation rules
(``difflet/pipeline/parallel_config.py:30-117``).  On B200 every axis is a
separate mesh axis with its own peer-pointer table, so CP and CFG-parallel
compose (world = dp x cfg x cp x tp); SP (Megatron sequence parallelism) reuses
the TP group and adds no axis.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

from difflet_b200.parallel.mesh import MeshSpec

CP_MODES: tuple[str, ...] = ("gather_kv", "ring", "ulysses")


@dataclass(frozen=True)
class DiffletParallelConfig:
    tp_degree: int = 1
    cp_degree: int = 1
    cfg_parallel_enabled: bool = False
    cp_mode: str = "gather_kv"
    sp_enabled: bool = False
    dp_degree: int = 1

    def __post_init__(self) -> None:
        low = [n for n in ("tp_degree", "cp_degree", "dp_degree") if getattr(self, n) < 1]
        if low:
            raise ValueError(f"{low[0]} is {getattr(self, low[0])}; every parallel degree is at least 1")
        if self.cp_mode not in CP_MODES:
            raise ValueError(f"unknown cp_mode {self.cp_mode!r} (known: {', '.join(sorted(CP_MODES))})")
        if self.cp_mode != "gather_kv" and self.cp_degree <= 1:
            raise ValueError(f"cp_mode {self.cp_mode!r} only applies with a context-parallel degree above 1")
        if self.sp_enabled and self.cp_degree > 1:
            raise ValueError("Megatron sequence parallelism (sp) and context parallelism (cp > 1) cannot be combined")
        if self.sp_enabled and self.tp_degree <= 1:
            raise ValueError("sp_enabled shards over the tensor-parallel group: needs tp_degree > 1")

    @property
    def mesh_spec(self) -> MeshSpec:
        return MeshSpec(
            dp=self.dp_degree,
            cfg=2 if self.cfg_parallel_enabled else 1,
            cp=self.cp_degree,
            tp=self.tp_degree,
        )

    @property
    def world_size(self) -> int:
        return self.mesh_spec.world_size

    @property
    def model_world_size(self) -> int:
        """Ranks that hold one model replica (everything but dp)."""
        return self.world_size // self.dp_degree

    def to_cache_dict(self) -> dict[str, object]:
        d = asdict(self)
        if self.cp_mode == "gather_kv":
            d.pop("cp_mode")
        if not self.sp_enabled:
            d.pop("sp_enabled")
        if self.dp_degree == 1:
            d.pop("dp_degree")
        return d

    @classmethod
    def from_args(cls, *, tp=1, cp=1, cfg=False, cp_mode=None, sp=False, dp=1) -> "DiffletParallelConfig":
        return cls(tp_degree=tp, cp_degree=cp, cfg_parallel_enabled=bool(cfg),
                   cp_mode=cp_mode or ("ulysses" if cp > 1 else "gather_kv"), sp_enabled=sp,
                   dp_degree=dp)


@dataclass(frozen=True)
class CandidateConfig:
    """Candidate (``N``) axis: batch-like, never changes world size, cache-key only."""

    max_candidates: int = 1
    active_candidates: int | None = None

    def __post_init__(self) -> None:
        if self.max_candidates < 1:
            raise ValueError(f"max_candidates is {self.max_candidates}; at least one candidate is needed")
        if self.active_candidates is None:
            object.__setattr__(self, "active_candidates", self.max_candidates)
        if not 1 <= self.active_candidates <= self.max_candidates:
            raise ValueError(f"{self.active_candidates} active candidates do not fit the range 1.."
                             f"{self.max_candidates} set by max_candidates")

    @property
    def is_trivial(self) -> bool:
        return self.max_candidates == 1

    def world_size(self, parallel: DiffletParallelConfig) -> int:
        return parallel.world_size

    def to_cache_dict(self) -> dict[str, object]:
        return {"max_candidates": self.max_candidates}
