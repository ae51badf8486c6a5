"""Device memory per process and per GPU, sampled through NVML while a launch runs.

What the in-process ``torch.cuda.max_memory_allocated`` cannot see: memory that is not the caching
allocator's (the CUDA context, NCCL buffers, the symmetric peer-memory heap allocated with
``cudaMalloc``, cuBLAS workspaces) and the processes of the other ranks.  A background thread
reads, every ``interval_s``, each watched GPU's used memory and every compute process on it with
its own usage; ``summary`` gives each GPU's peak and each process's peak, with the sample count.
Short peaks between two samples are missed, so the in-process peak is recorded beside it as a
cross-check.  Only NVML queries run: nothing changes a device setting.  Reference behaviour:
``difflet/bench/memory.py`` (per-rank device memory sampled by a monitor during the launch).
"""

from __future__ import annotations

import threading
import time


def _nvml():
    import pynvml

    pynvml.nvmlInit()
    return pynvml


class DeviceMemorySampler:
    def __init__(self, devices, *, interval_s: float = 0.2, nvml=None):
        self.devices = [int(d) for d in devices]
        self.interval_s = float(interval_s)
        self._nv = nvml
        self.samples: list[dict] = []   # {"t", "gpu", "used", "procs": {pid: bytes}}
        self._stop = threading.Event()
        self._t: threading.Thread | None = None
        self.error: str | None = None

    def sample_once(self) -> None:
        nv = self._nv
        t = time.monotonic()
        for i in self.devices:
            h = nv.nvmlDeviceGetHandleByIndex(i)
            procs = {}
            for p in nv.nvmlDeviceGetComputeRunningProcesses(h) or []:
                used = getattr(p, "usedGpuMemory", None)
                if used is not None:
                    procs[int(p.pid)] = int(used)
            self.samples.append({"t": t, "gpu": i, "used": int(nv.nvmlDeviceGetMemoryInfo(h).used), "procs": procs})

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                self.sample_once()
            except Exception as exc:  # noqa: BLE001 - a sampler never fails the launch it watches
                self.error = repr(exc)
                return
            self._stop.wait(self.interval_s)

    def __enter__(self):
        try:
            self._nv = self._nv or _nvml()
        except Exception as exc:  # noqa: BLE001 - no NVML: the summary says so
            self.error = repr(exc)
            return self
        self._t = threading.Thread(target=self._loop, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=5)
        if self._nv is not None and self.error is None:
            try:
                self.sample_once()  # the state at the end of the launch
            except Exception as e:  # noqa: BLE001
                self.error = repr(e)

    def summary(self) -> dict:
        gpus: dict[int, int] = {}
        procs: dict[int, dict] = {}
        for s in self.samples:
            gpus[s["gpu"]] = max(gpus.get(s["gpu"], 0), s["used"])
            for pid, b in s["procs"].items():
                cur = procs.setdefault(pid, {"gpu": s["gpu"], "peak_bytes": 0})
                cur["peak_bytes"] = max(cur["peak_bytes"], b)
        gib = 1 << 30
        return {"samples": len(self.samples), "interval_s": self.interval_s, "error": self.error,
                "gpu_peak_gib": {str(g): round(b / gib, 3) for g, b in sorted(gpus.items())},
                "process_peak_gib": {str(p): {"gpu": v["gpu"], "peak_gib": round(v["peak_bytes"] / gib, 3)}
                                     for p, v in sorted(procs.items())}}


__all__ = ["DeviceMemorySampler"]
