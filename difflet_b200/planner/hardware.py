"""What the planner needs to know about this node, read (never set) through NVML.

Reference behaviour (``difflet/planner/hardware.py:113``): detect the accelerator count and kind
before enumerating layouts.  On an HGX B200 node the answer is small: how many GPUs, which SKU,
how much memory each has, and whether they reach each other over NVLink (behind NVSwitch every
pair has the same bandwidth, so placement needs no topology search).  Every NVML call is a query;
nothing here changes a GPU setting.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass


@dataclass(frozen=True)
class Hardware:
    gpus: int
    sku: str
    hbm_gb: float
    nvlink: bool          # at least one active NVLink on GPU 0
    nvlink_links: int     # active links on GPU 0 (18 on B200)
    source: str           # "nvml", or "none" when no GPU / NVML is reachable

    def to_dict(self) -> dict:
        return asdict(self)


def detect(nvml=None) -> Hardware:
    """Query NVML (``pynvml`` from nvidia-ml-py unless a module is given, e.g. a test fake)."""
    try:
        if nvml is None:
            import pynvml as nvml  # noqa: N813
        nvml.nvmlInit()
    except Exception:  # noqa: BLE001 - no driver / no GPU: the planner takes --gpus as given
        return Hardware(0, "none", 0.0, False, 0, "none")
    try:
        n = int(nvml.nvmlDeviceGetCount())
        if n == 0:
            return Hardware(0, "none", 0.0, False, 0, "nvml")
        h = nvml.nvmlDeviceGetHandleByIndex(0)
        name = nvml.nvmlDeviceGetName(h)
        name = name.decode() if isinstance(name, bytes) else str(name)
        mem = nvml.nvmlDeviceGetMemoryInfo(h)
        links = 0
        for link in range(getattr(nvml, "NVML_NVLINK_MAX_LINKS", 18)):
            try:
                if nvml.nvmlDeviceGetNvLinkState(h, link):
                    links += 1
            except Exception:  # noqa: BLE001 - link index not present on this part
                break
        return Hardware(n, name, round(mem.total / 2**30, 1), links > 0, links, "nvml")
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass


__all__ = ["Hardware", "detect"]
