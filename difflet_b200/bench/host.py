"""Idle check of a bench lane's GPUs before every measured launch.

Behaviour of the reference's lane check (difflet/bench/runner.py:7, :214-219, difflet/bench/host.py):
a launch whose devices are busy measures someone else's load, so the harness refuses it.  Here a
device is idle when no compute process holds it, its utilisation is at most ``util_max`` percent
and at most ``mem_max_mib`` of its memory is in use.  Read through NVML (``pynvml``, from the
``nvidia-ml-py`` package); tests pass a fake with the same four calls.  Nothing here changes a
device setting: the calls only read.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class DeviceState:
    index: int
    processes: int
    util_pct: int
    mem_used_mib: float


@dataclass
class IdleReport:
    devices: list[DeviceState] = field(default_factory=list)
    problems: list[str] = field(default_factory=list)

    @property
    def idle(self) -> bool:
        return not self.problems

    def reasons(self) -> list[str]:
        return list(self.problems)

    def to_dict(self) -> dict:
        return {"idle": self.idle, "problems": self.problems,
                "devices": [vars(d) for d in self.devices]}


def _nvml():
    import pynvml

    pynvml.nvmlInit()
    return pynvml


def check_idle(devices, nvml=None, *, util_max: int = 5, mem_max_mib: float = 2048.0) -> IdleReport:
    """State of each device index in ``devices`` and the reasons it is not idle."""
    nv = nvml or _nvml()
    rep = IdleReport()
    for i in devices:
        h = nv.nvmlDeviceGetHandleByIndex(int(i))
        procs = len(nv.nvmlDeviceGetComputeRunningProcesses(h) or [])
        util = int(nv.nvmlDeviceGetUtilizationRates(h).gpu)
        mem = float(nv.nvmlDeviceGetMemoryInfo(h).used) / (1 << 20)
        rep.devices.append(DeviceState(int(i), procs, util, round(mem, 1)))
        if procs:
            rep.problems.append(f"gpu{i}: {procs} compute process(es) running")
        if util > util_max:
            rep.problems.append(f"gpu{i}: utilisation {util} % > {util_max} %")
        if mem > mem_max_mib:
            rep.problems.append(f"gpu{i}: {mem:.0f} MiB in use > {mem_max_mib:.0f} MiB")
    return rep


__all__ = ["DeviceState", "IdleReport", "check_idle"]
