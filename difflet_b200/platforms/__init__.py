"""Platform layer: detection, capabilities, runtime preparation.

Two platforms exist: ``cuda`` (B200 / sm_100a, native kernels, NCCL + peer
memory) and ``cpu`` (the fp32/fp64 oracle used by tests).  Code outside this
package asks the platform for capabilities instead of comparing names, as in
the reference (``difflet/platforms/base.py:22-91``, ``difflet/platforms/gpu.py:26-126``).
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

from difflet_b200 import envs

PARALLEL_MODES = ("tp", "sp", "cp", "cfg", "dp")


@dataclass(frozen=True)
class PlatformCapabilities:
    name: str
    requires_aot: bool = False
    flow: str = "gpu"
    parallel_modes: frozenset = field(default_factory=lambda: frozenset(PARALLEL_MODES))
    supports_cuda_graphs: bool = False
    supports_mx: bool = False
    device_type: str = "cpu"


class Platform:
    name = "base"
    capabilities: PlatformCapabilities

    def device(self, local_rank: int = 0):
        import torch

        return torch.device(self.capabilities.device_type, local_rank) if self.capabilities.device_type == "cuda" else torch.device("cpu")

    def unsupported_parallel_modes(self, parallel) -> list[str]:
        used = []
        if parallel.tp_degree > 1:
            used.append("tp")
        if parallel.sp_enabled:
            used.append("sp")
        if parallel.cp_degree > 1:
            used.append("cp")
        if parallel.cfg_parallel_enabled:
            used.append("cfg")
        if parallel.dp_degree > 1:
            used.append("dp")
        return [m for m in used if m not in self.capabilities.parallel_modes]

    def prepare_runtime(self, parallel=None) -> None:  # pragma: no cover - trivial
        pass

    def toolchain_versions(self) -> dict[str, str]:
        import torch

        return {"torch": torch.__version__}


class CpuPlatform(Platform):
    name = "cpu"
    capabilities = PlatformCapabilities(name="cpu", device_type="cpu")

    def prepare_runtime(self, parallel=None) -> None:
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world > 1:
            from difflet_b200.parallel.groups import init_distributed

            init_distributed(backend="gloo")


class CudaPlatform(Platform):
    """NVIDIA B200 (sm_100a): native kernels, NCCL bootstrap, symmetric peer memory."""

    name = "cuda"
    capabilities = PlatformCapabilities(
        name="cuda", device_type="cuda", supports_cuda_graphs=True, supports_mx=True
    )

    def prepare_runtime(self, parallel=None) -> None:
        import torch

        local = envs.LOCAL_RANK
        if torch.cuda.is_available():
            torch.cuda.set_device(local % max(1, torch.cuda.device_count()))
        world = envs.WORLD_SIZE
        if world > 1:
            from difflet_b200.parallel.groups import init_distributed

            init_distributed(backend="nccl")

    def toolchain_versions(self) -> dict[str, str]:
        import torch

        out = {"torch": torch.__version__, "cuda": str(torch.version.cuda)}
        try:
            from difflet_b200 import _native

            out["kernels"] = _native.source_hash()
        except Exception:
            pass
        if torch.cuda.is_available():
            out["gpu"] = torch.cuda.get_device_name(0)
            out["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
        return out


PLATFORM_FACTORIES = {"cuda": CudaPlatform, "cpu": CpuPlatform}
_DETECTION_ORDER = ("cuda", "cpu")
_current: Platform | None = None


def detect_platform_name() -> str:
    forced = envs.DIFFLET_BACKEND
    if forced:
        if forced not in PLATFORM_FACTORIES:
            raise ValueError(f"unknown DIFFLET_BACKEND {forced!r}; expected one of {sorted(PLATFORM_FACTORIES)}")
        return forced
    import torch

    return "cuda" if torch.cuda.is_available() else "cpu"


def get_platform(name: str | None = None) -> Platform:
    global _current
    name = name or detect_platform_name()
    if _current is None or _current.name != name:
        _current = PLATFORM_FACTORIES[name]()
    return _current


def current_backend() -> str:
    return get_platform().name
