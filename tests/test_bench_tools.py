"""Bench tooling on the CPU: result comparison, the Markdown report, telemetry reading and
page-cache control."""

import json
import os

import pytest


def _line(value, *, n=1, layout="single", e2e=None, gpu="NVIDIA B200", model="FLUX.1-dev", sha="abc",
          metric="FLUX step", reasons=("sw_power_cap",)):
    return {"metric": metric, "value": value, "unit": "ms/step", "n_gpus": n, "higher_is_better": False,
            "dtype": "bf16", "steps": 10, "warmup": 3,
            "config": {"model": model, "seq_len": 4608, "global_batch": 1, "parallelism": layout},
            "clocks": {"sm_mhz": 1900.0, "reasons": list(reasons)},
            "e2e": None if e2e is None else {"value": e2e, "unit": "s/image"},
            "provenance": {"device": {"gpu": gpu}, "git": {"sha": sha}}}


def _write(path, recs):
    path.write_text("\n".join(json.dumps(r) for r in recs) + "\n")
    return path


def test_compare_direction_differences_and_refusals(tmp_path):
    from difflet_b200.bench.compare import ComparisonRefused, compare, format_text, load, main

    a = _write(tmp_path / "a.json", [_line(66.0, e2e=1.9)])
    b = _write(tmp_path / "b.json", ["log line", _line(60.0, e2e=1.8, sha="def")])
    b.write_text("starting\n" + b.read_text())
    res = compare(load(a), load(b))
    assert res["metrics"]["value"]["ratio"] == pytest.approx(60 / 66, abs=1e-4)
    assert res["metrics"]["value"]["better"] and res["metrics"]["e2e"]["better"]  # lower is better
    assert res["differs"] == {"revision": ("abc", "def")} and not res["noisy"]
    assert "B/A" in format_text(res)
    # another workload: refused
    c = _write(tmp_path / "c.json", [_line(60.0, model="Wan2.2-T2V-A14B")])
    with pytest.raises(ComparisonRefused):
        compare(load(a), load(c))
    assert main([str(a), str(c)]) == 2
    # another GPU: only the per-step value is compared
    d = _write(tmp_path / "d.json", [_line(70.0, e2e=2.5, gpu="NVIDIA B300")])
    r2 = compare(load(a), load(d))
    assert r2["cross_machine"] and "e2e" not in r2["metrics"] and not r2["metrics"]["value"]["better"]
    # a control arm that spreads more than the difference: noisy
    ctrl = _write(tmp_path / "ctrl.jsonl", [{"suite": "s", "run": "flux/a", "result": _line(v)} for v in (60, 66, 63)])
    cand = _write(tmp_path / "cand.jsonl", [{"suite": "s", "run": "flux/b", "result": _line(v)} for v in (62, 62.5)])
    r3 = compare(load(ctrl), load(cand))
    assert r3["metrics"]["value"]["a"]["n"] == 3 and r3["noisy"]


def test_report_summarises_newest_results(tmp_path):
    from difflet_b200.bench.report import report

    _write(tmp_path / "old.json", [_line(70.0)])
    os.utime(tmp_path / "old.json", (1, 1))
    _write(tmp_path / "new.json", [_line(64.5, e2e=1.76)])
    _write(tmp_path / "n8.json", [_line(15.9, n=8, layout="ulysses8")])
    (tmp_path / "suite").mkdir()
    _write(tmp_path / "suite" / "s.jsonl", [{"suite": "s", "run": "flux/a", "error": "lane not idle"}])
    md = report(tmp_path).read_text()
    assert "## FLUX step" in md and "| 1 | single | 64.5 | 1.76 s/image |" in md
    assert "| 8 | ulysses8 | 15.9 |" in md and "| 1 | abc | new.json |" in md  # one older result
    assert "sw_power_cap" in md and "## Failed launches" in md and "lane not idle" in md


def test_timing_reader_pairs_spans_across_processes(tmp_path, monkeypatch):
    from difflet_b200.bench import timing
    from difflet_b200.utils import telemetry

    monkeypatch.setenv(telemetry.TIMING_ENV, str(tmp_path))
    recs = []
    t = 1_000_000_000
    for rank in (0, 1):
        lines = [{"event": "process", "t_ns": t, "pid": 10 + rank, "rank": rank, "world": 2, "role": "rank"}]
        lines.append({"event": "span", "t_ns": t, "pid": 10 + rank, "rank": rank, "world": 2, "name": "request",
                      "phase": "begin"})
        for i in range(3):
            lines.append({"event": "step", "t_ns": t + (i + 1) * 50_000_000, "pid": 10 + rank, "rank": rank,
                          "world": 2, "index": i})
        lines.append({"event": "span", "t_ns": t + (300 + 100 * rank) * 1_000_000, "pid": 10 + rank, "rank": rank,
                      "world": 2, "name": "request", "phase": "end", "ok": True})
        recs.append(lines)
        (tmp_path / f"rank{rank}-{10 + rank}.jsonl").write_text("\n".join(json.dumps(x) for x in lines) + "\n{torn")
    s = timing.summarize(timing.read_launch(tmp_path))
    assert s["processes"] == 2 and s["ranks"] == [0, 1] and s["steps"] == 6
    assert s["spans"]["request"]["max_s"] == pytest.approx(0.4) and s["spans"]["request"]["max_rank"] == 1
    assert s["step_interval_median_s"] == pytest.approx(0.05) and s["bad_lines"] == 2
    assert s["unfinished_spans"] == []


def test_page_cache_evict_warm_residency(tmp_path):
    from difflet_b200.bench import pagecache as pc

    f = tmp_path / "w.safetensors"
    f.write_bytes(os.urandom(4 << 20))
    (tmp_path / "notes.txt").write_text("x")
    files = pc.files_under([tmp_path])
    assert files == [f]
    assert pc.evict(files) == 4 << 20
    cold = pc.residency(files)
    assert pc.warm(files) == 4 << 20
    hot = pc.residency(files)
    assert hot["fraction"] == 1.0 and cold["fraction"] <= hot["fraction"] and hot["bytes"] == 4 << 20


def test_device_memory_sampler_with_a_fake_nvml():
    """Peaks per GPU and per process from NVML samples (a fake with the three queries used)."""
    import time
    from types import SimpleNamespace

    from difflet_b200.bench.memory import DeviceMemorySampler

    class FakeNVML:
        def __init__(self):
            self.tick = 0

        def nvmlDeviceGetHandleByIndex(self, i):
            return i

        def nvmlDeviceGetComputeRunningProcesses(self, h):
            self.tick += 1
            grow = min(self.tick, 5) << 30
            return [SimpleNamespace(pid=100 + h, usedGpuMemory=grow), SimpleNamespace(pid=999, usedGpuMemory=None)]

        def nvmlDeviceGetMemoryInfo(self, h):
            return SimpleNamespace(used=(min(self.tick, 5) + 1) << 30)

    with DeviceMemorySampler([0, 1], interval_s=0.01, nvml=FakeNVML()) as s:
        time.sleep(0.2)
    out = s.summary()
    assert out["error"] is None and out["samples"] >= 4
    assert out["gpu_peak_gib"] == {"0": 6.0, "1": 6.0}
    assert out["process_peak_gib"]["100"] == {"gpu": 0, "peak_gib": 5.0} and "999" not in out["process_peak_gib"]


def test_timing_reader_reads_what_the_engine_writes(tmp_path):
    """Round trip through the real writer, in a fresh process (its sink opens on first use)."""
    import subprocess
    import sys
    import textwrap
    from pathlib import Path

    from difflet_b200.bench import timing

    code = textwrap.dedent("""
        from difflet_b200.utils import telemetry as t
        t.event("process", role="driver")
        with t.span("request", request="r0"):
            for i in range(3):
                t.event("step", index=i)
            t.event("forward", seconds=0.25)
    """)
    repo = Path(__file__).resolve().parents[1]
    env = dict(os.environ, DIFFLET_BENCH_TIMING_DIR=str(tmp_path), PYTHONPATH=str(repo), RANK="0", WORLD_SIZE="1")
    subprocess.run([sys.executable, "-c", code], env=env, check=True, timeout=120)
    logs = timing.read_launch(tmp_path)
    assert len(logs) == 1 and logs[0].role == "driver" and logs[0].forwards == [0.25]
    sp = logs[0].spans[0]
    assert sp.name == "request" and sp.ok is True and sp.seconds >= 0 and sp.fields.get("request") == "r0"
    s = timing.summarize(logs)
    assert s["steps"] == 3 and s["bad_lines"] == 0 and s["unfinished_spans"] == []
