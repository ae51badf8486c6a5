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
        bad = [(a, getattr(self, a)) for a in AXES
               if isinstance(getattr(self, a), bool) or not isinstance(getattr(self, a), int) or getattr(self, a) < 1]
        if bad:
            axis, v = bad[0]
            raise ValueError(f"mesh axis {axis} needs a positive integer degree (got {v!r})")

    # Mixed-radix view: digits in AXES order (dp most significant, tp least).
    def _sizes(self) -> tuple[int, ...]:
        return tuple(getattr(self, a) for a in AXES)

    def _check_axis(self, axis: str) -> int:
        try:
            return AXES.index(axis)
        except ValueError:
            raise ValueError(f"{axis!r} is not a mesh axis (axes: {', '.join(AXES)})") from None

    @property
    def world_size(self) -> int:
        n = 1
        for size in self._sizes():
            n *= size
        return n

    def axis_size(self, axis: str) -> int:
        return self._sizes()[self._check_axis(axis)]

    def axis_stride(self, axis: str) -> int:
        """Rank distance between neighbours along ``axis``: the product of the faster axes."""
        stride = 1
        for size in self._sizes()[self._check_axis(axis) + 1:]:
            stride *= size
        return stride

    def coords_of(self, rank: int) -> MeshCoords:
        if rank < 0 or rank >= self.world_size:
            raise ValueError(f"rank {rank} is outside a mesh of {self.world_size} ranks")
        digits = []
        rest = rank
        for size in reversed(self._sizes()):  # least significant digit (tp) first
            rest, d = divmod(rest, size)
            digits.append(d)
        return MeshCoords(*reversed(digits))

    def rank_of(self, *, dp: int = 0, cfg: int = 0, cp: int = 0, tp: int = 0) -> int:
        coords = (dp, cfg, cp, tp)
        rank = 0
        for axis, c, size in zip(AXES, coords, self._sizes()):
            if c < 0 or c >= size:
                raise ValueError(f"coordinate {c} does not exist on mesh axis {axis} of degree {size}")
            rank = rank * size + c
        return rank

    def axis_rank(self, rank: int, axis: str) -> int:
        return self.coords_of(rank)[self._check_axis(axis)]

    def axis_groups(self, axis: str) -> list[list[int]]:
        """Every group of ranks that share all coordinates except ``axis``, each in axis order."""
        i = self._check_axis(axis)
        groups: dict[tuple, list[int]] = {}
        for r in range(self.world_size):
            c = self.coords_of(r)
            groups.setdefault(c[:i] + c[i + 1:], []).append(r)
        return list(groups.values())

    def group_of(self, rank: int, axis: str) -> list[int]:
        c = self.coords_of(rank)
        i = self._check_axis(axis)
        return [self.rank_of(**dict(zip(AXES, c[:i] + (j,) + c[i + 1:]))) for j in range(self.axis_size(axis))]
