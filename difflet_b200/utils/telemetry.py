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

_step_index = 0


def enabled() -> bool:
    """True when a timing directory is configured (read on every call: tests flip it)."""
    return os.environ.get(TIMING_ENV, "") != ""


def _identity() -> tuple[int, int]:
    """(rank, world) of this process.  An initialised process group is authoritative; it is
    only consulted when ``torch.distributed`` was imported already (importing torch here would
    cost seconds inside whatever the caller is timing).  Otherwise torchrun's environment."""
    env_rank, env_world = os.environ.get("RANK", "0"), os.environ.get("WORLD_SIZE", "1")
    mod = sys.modules.get("torch.distributed")
    if mod is not None:
        try:
            if mod.is_initialized():
                return mod.get_rank(), mod.get_world_size()
        except (RuntimeError, ValueError, AttributeError):
            pass  # group being torn down: fall back to the environment
    try:
        return int(env_rank), int(env_world)
    except ValueError:
        return 0, 1


def _plain(v: Any) -> Any:
    """JSON-safe copy of ``v``: containers recursed, unknown objects as their ``str``."""
    if isinstance(v, dict):
        return {str(k): _plain(x) for k, x in v.items()}
    if isinstance(v, (list, tuple, set)):
        return [_plain(x) for x in v]
    return v if v is None or isinstance(v, (bool, int, float, str)) else str(v)


class _Sink:
    """One append-only JSONL file per process.  It is opened lazily and re-opened in a forked
    child (the pid is part of the name); the first record of a file describes the process.
    The first failure switches the sink off for the rest of the process."""

    def __init__(self) -> None:
        self.fh = None
        self.pid = -1
        self.dead = False

    def _filename(self) -> str:
        launched = "LOCAL_RANK" in os.environ
        tag = ("rank" + os.environ.get("RANK", "0")) if launched else "proc"
        return os.path.join(os.environ[TIMING_ENV], f"{tag}-{os.getpid()}.jsonl")

    def _record(self, kind: str, fields: dict) -> str:
        rank, world = _identity()
        body = {"event": kind, "t_ns": time.monotonic_ns(), "pid": os.getpid(), "rank": rank, "world": world}
        body.update(_plain(fields))
        return json.dumps(body, ensure_ascii=False)

    def write(self, kind: str, fields: dict) -> None:
        if self.dead:
            return
        try:
            if self.fh is None or self.pid != os.getpid():
                os.makedirs(os.environ[TIMING_ENV], exist_ok=True)
                self.fh = open(self._filename(), "a", encoding="utf-8", buffering=1)
                self.pid = os.getpid()
                role = "rank" if "LOCAL_RANK" in os.environ else "proc"
                self.fh.write(self._record("process", {"argv": list(sys.argv), "role": role}) + "\n")
            self.fh.write(self._record(kind, fields) + "\n")
        except OSError as exc:
            self.dead = True
            print(f"[telemetry] timing events disabled after an error: {exc!r}", file=sys.stderr, flush=True)


_SINK = _Sink()


def event(kind: str, /, **fields: Any) -> None:
    """Append one event (no-op unless ``DIFFLET_BENCH_TIMING_DIR`` is set)."""
    if enabled():
        _SINK.write(kind, fields)


class span(contextlib.AbstractContextManager):  # noqa: N801 - used like a function
    """``span`` begin / end events around a block; the end event carries ``ok`` (False when
    the block raised) and is written on error too."""

    def __init__(self, name: str, **fields: Any) -> None:
        self.name, self.fields = name, fields

    def __enter__(self):
        event("span", name=self.name, phase="begin", **self.fields)
        return self

    def __exit__(self, exc_type, exc, tb):
        event("span", name=self.name, phase="end", ok=exc_type is None, **self.fields)
        return False


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
