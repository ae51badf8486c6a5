"""Opt-in run telemetry: structured timing events, per-step device times, latent dumps, NVTX.

* ``DIFFLET_BENCH_TIMING_DIR``: every process appends JSON lines to
  ``<dir>/<rank|proc><RANK>-<pid>.jsonl``.  The event schema is the reference's
  (difflet/utils/bench_timing.py:1-175) so its readers work unchanged: every record has
  ``event``, ``t_ns`` (``time.monotonic_ns()``, one clock per host), ``pid``, ``rank``,
  ``world``; kinds ``process`` (argv, role), ``args``, ``span`` (name, phase begin/end),
  ``step`` (index), ``forward`` (seconds), ``evidence``, ``output``.
* ``DIFFLET_STEP_TIMES_FILE``: one JSON line per denoise step with its device time (CUDA
  events recorded in the step callback, resolved once the request ends: no host sync inside
  the loop).
* ``DIFFLET_DUMP_LATENTS_DIR``: the latents after every step, ``<dir>/<request>/step_NNN.pt``.
* ``nvtx_range``: NVTX ranges around requests and DiT forwards for Nsight timelines.
Nothing here may fail a run: a write error disables the feature and is reported once.
"""

from __future__ import annotations

import contextlib
import json
import os
import sys
import time
from typing import Any, Iterator

TIMING_ENV = "DIFFLET_BENCH_TIMING_DIR"
STEP_TIMES_ENV = "DIFFLET_STEP_TIMES_FILE"
DUMP_ENV = "DIFFLET_DUMP_LATENTS_DIR"

_handle = None
_handle_pid = None
_failed = False
_step_index = 0


def enabled() -> bool:
    return bool(os.environ.get(TIMING_ENV))


def _rank_world() -> tuple[int, int]:
    dist = sys.modules.get("torch.distributed")
    try:
        if dist is not None and dist.is_available() and dist.is_initialized():
            return dist.get_rank(), dist.get_world_size()
    except Exception:  # noqa: BLE001 - a half-initialised process group
        pass
    try:
        return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    except ValueError:
        return 0, 1


def _jsonable(v: Any) -> Any:
    if v is None or isinstance(v, (bool, int, float, str)):
        return v
    if isinstance(v, dict):
        return {str(k): _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple, set)):
        return [_jsonable(x) for x in v]
    return str(v)


def _write(kind: str, fields: dict) -> None:
    rank, world = _rank_world()
    rec = {"event": kind, "t_ns": time.monotonic_ns(), "pid": os.getpid(), "rank": rank, "world": world}
    rec.update(_jsonable(fields))
    _handle.write(json.dumps(rec, ensure_ascii=False) + "\n")


def _open():
    global _handle, _handle_pid
    pid = os.getpid()
    if _handle is not None and _handle_pid == pid:
        return
    d = os.environ[TIMING_ENV]
    os.makedirs(d, exist_ok=True)
    role = "rank" if "LOCAL_RANK" in os.environ else "proc"
    name = f"{role}{os.environ.get('RANK', '0') if role == 'rank' else ''}-{pid}.jsonl"
    _handle = open(os.path.join(d, name), "a", encoding="utf-8", buffering=1)
    _handle_pid = pid
    _write("process", {"argv": list(sys.argv), "role": role})


def event(kind: str, /, **fields: Any) -> None:
    """Append one event (no-op unless ``DIFFLET_BENCH_TIMING_DIR`` is set)."""
    global _failed
    if _failed or not enabled():
        return
    try:
        _open()
        _write(kind, fields)
    except Exception as exc:  # noqa: BLE001 - telemetry never fails a run
        _failed = True
        print(f"[telemetry] timing events disabled after an error: {exc!r}", file=sys.stderr, flush=True)


@contextlib.contextmanager
def span(name: str, **fields: Any) -> Iterator[None]:
    """``span`` begin / end events around a block (the end is written on error too)."""
    if not enabled():
        yield
        return
    event("span", name=name, phase="begin", **fields)
    ok = False
    try:
        yield
        ok = True
    finally:
        event("span", name=name, phase="end", ok=ok, **fields)


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    """An NVTX range (visible in Nsight timelines; free when no tool is attached)."""
    rng = None
    try:
        import torch

        if torch.cuda.is_available():
            torch.cuda.nvtx.range_push(name)
            rng = torch.cuda.nvtx
    except Exception:  # noqa: BLE001
        rng = None
    try:
        yield
    finally:
        if rng is not None:
            rng.range_pop()


def new_request() -> None:
    global _step_index
    _step_index = 0


def device_memory() -> dict | None:
    try:
        import torch

        if not torch.cuda.is_available() or not torch.cuda.is_initialized():
            return None
        return {"max_allocated_mb": round(torch.cuda.max_memory_allocated() / 2**20, 1),
                "reserved_mb": round(torch.cuda.memory_reserved() / 2**20, 1)}
    except Exception:  # noqa: BLE001
        return None


class StepRecorder:
    """Per-request step observer: ``step`` events, device step times, latent dumps.

    Pass ``recorder.callback`` as a pipeline's ``callback(i, latents)``; call ``finish()``
    after the request.  Step times come from CUDA events recorded in the callback (on the
    current stream) and are read once at ``finish``."""

    def __init__(self, request: str, *, times_file: str | None = None, dump_dir: str | None = None):
        self.request = request
        self.times_file = times_file
        self.dump_dir = os.path.join(dump_dir, request) if dump_dir else None
        self._events = []
        self._t0 = None
        self._t0_host = time.perf_counter()
        new_request()

    @classmethod
    def maybe(cls, request: str) -> "StepRecorder | None":
        """A recorder when any per-step feature is switched on, else None."""
        times, dump = os.environ.get(STEP_TIMES_ENV), os.environ.get(DUMP_ENV)
        if not (times or dump or enabled()):
            return None
        return cls(request, times_file=times, dump_dir=dump)

    def _cuda_event(self):
        try:
            import torch

            if torch.cuda.is_available() and torch.cuda.is_initialized():
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                return e
        except Exception:  # noqa: BLE001
            pass
        return None

    def start(self) -> None:
        self._t0 = self._cuda_event()
        self._t0_host = time.perf_counter()

    def callback(self, i: int, latents) -> None:
        global _step_index
        event("step", index=_step_index, request=self.request)
        _step_index += 1
        if self.times_file:
            self._events.append((i, self._cuda_event(), time.perf_counter()))
        if self.dump_dir:
            try:
                import torch

                os.makedirs(self.dump_dir, exist_ok=True)
                torch.save(latents.detach().to("cpu"), os.path.join(self.dump_dir, f"step_{i:03d}.pt"))
            except Exception as exc:  # noqa: BLE001
                print(f"[telemetry] latent dump disabled: {exc!r}", file=sys.stderr, flush=True)
                self.dump_dir = None

    def step_times_ms(self) -> list:
        """Device milliseconds of every step (host wall time when CUDA events are absent)."""
        out, prev_e, prev_t = [], self._t0, self._t0_host
        for i, e, t in self._events:
            if e is not None and prev_e is not None:
                e.synchronize()
                out.append((i, prev_e.elapsed_time(e)))
            elif prev_t is not None:
                out.append((i, (t - prev_t) * 1e3))
            prev_e, prev_t = e, t
        return out

    def finish(self) -> None:
        if self.times_file:
            try:
                with open(self.times_file, "a", encoding="utf-8") as f:
                    for i, ms in self.step_times_ms():
                        f.write(json.dumps({"request": self.request, "step": i, "ms": round(ms, 4)}) + "\n")
            except Exception as exc:  # noqa: BLE001
                print(f"[telemetry] step times not written: {exc!r}", file=sys.stderr, flush=True)
        event("evidence", request=self.request, device_memory=device_memory())


__all__ = ["DUMP_ENV", "STEP_TIMES_ENV", "StepRecorder", "TIMING_ENV", "device_memory", "enabled", "event",
           "new_request", "nvtx_range", "span"]
