"""Read the run telemetry (``utils/telemetry.py``) back into spans, steps and per-process facts.

One launch writes one JSONL file per process (``DIFFLET_BENCH_TIMING_DIR``: the driver and every
rank).  Every record carries ``t_ns`` from ``time.monotonic_ns()``, so the files of one host line
up on one clock.  This module pairs each ``span`` begin with its end (per process, per name, in
nesting order), collects the ``step`` and ``forward`` records, and summarises a launch: wall time
of every named span over all processes, the steps' intervals, and the slowest rank of each span.
Reference behaviour: ``difflet/bench/timing.py`` over ``difflet/utils/bench_timing.py``.
"""

from __future__ import annotations

import json
import statistics
from dataclasses import dataclass, field
from pathlib import Path
from typing import Iterable


@dataclass
class Span:
    name: str
    rank: int
    pid: int
    begin_ns: int
    end_ns: int | None = None
    ok: bool | None = None
    fields: dict = field(default_factory=dict)

    @property
    def seconds(self) -> float | None:
        return None if self.end_ns is None else (self.end_ns - self.begin_ns) / 1e9


@dataclass
class ProcessLog:
    path: str
    pid: int | None = None
    rank: int = 0
    world: int = 1
    role: str | None = None
    argv: list | None = None
    spans: list = field(default_factory=list)
    steps: list = field(default_factory=list)      # (index, t_ns)
    forwards: list = field(default_factory=list)   # seconds
    evidence: list = field(default_factory=list)
    outputs: list = field(default_factory=list)
    bad_lines: int = 0


def read_events(path: str | Path) -> Iterable[dict]:
    """The records of one JSONL file; torn or foreign lines are skipped (and counted by
    ``read_process``)."""
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                rec = json.loads(line)
            except ValueError:
                yield {"event": "__bad__"}
                continue
            if isinstance(rec, dict) and "event" in rec and "t_ns" in rec:
                yield rec
            else:
                yield {"event": "__bad__"}


def read_process(path: str | Path) -> ProcessLog:
    log = ProcessLog(str(path))
    open_spans: dict[str, list[Span]] = {}
    for rec in read_events(path):
        kind = rec["event"]
        if kind == "__bad__":
            log.bad_lines += 1
            continue
        log.pid = rec.get("pid", log.pid)
        log.rank, log.world = int(rec.get("rank", log.rank)), int(rec.get("world", log.world))
        if kind == "process":
            log.role, log.argv = rec.get("role"), rec.get("argv")
        elif kind == "span":
            name = rec.get("name", "?")
            if rec.get("phase") == "begin":
                extra = {k: v for k, v in rec.items() if k not in ("event", "t_ns", "pid", "rank", "world", "name",
                                                                     "phase")}
                sp = Span(name, log.rank, log.pid or 0, rec["t_ns"], fields=extra)
                open_spans.setdefault(name, []).append(sp)
                log.spans.append(sp)
            elif rec.get("phase") == "end" and open_spans.get(name):
                sp = open_spans[name].pop()  # the innermost open span of that name
                sp.end_ns, sp.ok = rec["t_ns"], rec.get("ok")
        elif kind == "step":
            log.steps.append((rec.get("index"), rec["t_ns"]))
        elif kind == "forward":
            if rec.get("seconds") is not None:
                log.forwards.append(float(rec["seconds"]))
        elif kind == "evidence":
            log.evidence.append(rec)
        elif kind == "output":
            log.outputs.append(rec)
    return log


def read_launch(directory: str | Path) -> list[ProcessLog]:
    """Every process file of one launch, ordered by rank then pid."""
    logs = [read_process(p) for p in sorted(Path(directory).glob("*.jsonl"))]
    return sorted(logs, key=lambda lg: (lg.rank, lg.pid or 0))


def summarize(logs: list[ProcessLog]) -> dict:
    """Per span name: count, the slowest process's total seconds (the launch waits for it) and
    its rank, the median over processes; the step interval median over every process; unfinished
    spans (a crash or a kill) and unreadable lines."""
    per: dict[str, dict[int, float]] = {}
    unfinished = []
    for lg in logs:
        for sp in lg.spans:
            if sp.seconds is None:
                unfinished.append({"name": sp.name, "rank": sp.rank, "pid": sp.pid})
                continue
            per.setdefault(sp.name, {}).setdefault(lg.rank, 0.0)
            per[sp.name][lg.rank] += sp.seconds
    spans = {}
    for name, by_rank in per.items():
        slow_rank = max(by_rank, key=by_rank.get)
        spans[name] = {"processes": len(by_rank), "max_s": round(by_rank[slow_rank], 6), "max_rank": slow_rank,
                       "median_s": round(statistics.median(by_rank.values()), 6)}
    intervals = []
    for lg in logs:
        ts = [t for _, t in sorted(lg.steps, key=lambda s: s[1])]
        intervals += [(b - a) / 1e9 for a, b in zip(ts, ts[1:])]
    return {"processes": len(logs), "ranks": sorted({lg.rank for lg in logs}), "spans": spans,
            "step_interval_median_s": round(statistics.median(intervals), 6) if intervals else None,
            "steps": sum(len(lg.steps) for lg in logs), "unfinished_spans": unfinished,
            "bad_lines": sum(lg.bad_lines for lg in logs)}


__all__ = ["ProcessLog", "Span", "read_events", "read_launch", "read_process", "summarize"]
