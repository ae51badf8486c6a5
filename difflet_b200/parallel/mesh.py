"""Orthogonal {dp, cfg, cp, tp} device-mesh math.

Rank layout (tp innermost, dp outermost), the same as the reference's
``MeshSpec`` (``difflet/pipeline/parallel_mesh.py:30-99``) so configs and
rank maps carry over unchanged::

    rank = tp + T * (cp + C * (cfg + G * dp))

An axis group is the set of ranks that differ only in that axis' coordinate.
On 8xB200 behind NVSwitch every pair of GPUs has the same bandwidth, so rank
placement needs no topology search.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import NamedTuple

AXES = ("dp", "cfg", "cp", "tp")


class MeshCoords(NamedTuple):
    dp: int
    cfg: int
    cp: int
    tp: int


@dataclass(frozen=True)
class MeshSpec:
    dp: int = 1
    cfg: int = 1
    cp: int = 1
    tp: int = 1

    def __post_init__(self) -> None:
        for axis in AXES:
            v = getattr(self, axis)
            if not isinstance(v, int) or isinstance(v, bool) or v < 1:
                raise ValueError(f"{axis} must be an int >= 1, got {v!r}")

    @property
    def world_size(self) -> int:
        return self.dp * self.cfg * self.cp * self.tp

    def axis_size(self, axis: str) -> int:
        if axis not in AXES:
            raise ValueError(f"unknown axis {axis!r}; expected one of {AXES}")
        return getattr(self, axis)

    def axis_stride(self, axis: str) -> int:
        self.axis_size(axis)
        return {"tp": 1, "cp": self.tp, "cfg": self.tp * self.cp, "dp": self.tp * self.cp * self.cfg}[axis]

    def coords_of(self, rank: int) -> MeshCoords:
        if not 0 <= rank < self.world_size:
            raise ValueError(f"rank {rank} out of range [0, {self.world_size})")
        return MeshCoords(
            dp=rank // (self.tp * self.cp * self.cfg),
            cfg=(rank // (self.tp * self.cp)) % self.cfg,
            cp=(rank // self.tp) % self.cp,
            tp=rank % self.tp,
        )

    def rank_of(self, *, dp: int = 0, cfg: int = 0, cp: int = 0, tp: int = 0) -> int:
        for axis, c in (("dp", dp), ("cfg", cfg), ("cp", cp), ("tp", tp)):
            if not 0 <= c < self.axis_size(axis):
                raise ValueError(f"{axis} coordinate {c} out of range [0, {self.axis_size(axis)})")
        return tp + self.tp * (cp + self.cp * (cfg + self.cfg * dp))

    def axis_rank(self, rank: int, axis: str) -> int:
        self.axis_size(axis)
        return getattr(self.coords_of(rank), axis)

    def axis_groups(self, axis: str) -> list[list[int]]:
        size, stride = self.axis_size(axis), self.axis_stride(axis)
        return [
            [base + i * stride for i in range(size)]
            for base in range(self.world_size)
            if (base // stride) % size == 0
        ]

    def group_of(self, rank: int, axis: str) -> list[int]:
        for g in self.axis_groups(axis):
            if rank in g:
                return g
        raise ValueError(rank)
