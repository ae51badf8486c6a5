"""Markdown summary of benchmark results, generated from the result files themselves.

``report(directory)`` reads every ``*.json`` / ``*.jsonl`` result under a directory (``bench.py``
lines and bench-suite records) and writes ``SUMMARY.md``: one section per metric, one row per
(GPU count, layout) with the newest valid result, how many older results exist for it, and the
settings that explain a number (clocks and their limit reasons, the device time per step against
the end-to-end value, the revision).  Failed launches are listed apart instead of dropped.
Reference behaviour: ``difflet/bench/report.py`` (results rendered from the records, no
hand-written tables).
"""

from __future__ import annotations

import json
from pathlib import Path


def _records(path: Path) -> tuple[list[dict], list[dict]]:
    ok, failed = [], []
    for line in path.read_text(errors="replace").splitlines():
        line = line.strip()
        if not line.startswith("{"):
            continue
        try:
            rec = json.loads(line)
        except ValueError:
            continue
        if "metric" in rec:
            ok.append(rec)
        elif "suite" in rec:
            if rec.get("error") or not isinstance(rec.get("result"), dict):
                failed.append({"file": path.name, "run": rec.get("run"), "error": str(rec.get("error"))[:200]})
            elif "metric" in rec["result"]:
                ok.append({**rec["result"], "provenance": rec.get("provenance")})
    return ok, failed


def collect(directory: str | Path) -> tuple[list[dict], list[dict]]:
    ok, failed = [], []
    paths = sorted(Path(directory).rglob("*.json*"), key=lambda p: p.stat().st_mtime)
    for p in paths:
        if p.suffix not in (".json", ".jsonl"):
            continue
        o, f = _records(p)
        for r in o:
            r.setdefault("_file", str(p.relative_to(directory)))
            r["_mtime"] = p.stat().st_mtime
        ok += o
        failed += f
    return ok, failed


def _fmt(v, digits=4):
    if v is None:
        return ""
    if isinstance(v, float):
        return f"{v:.{digits}g}"
    return str(v)


def render(ok: list[dict], failed: list[dict]) -> str:
    out = ["# Benchmark summary", "", "Generated from the result files; newest valid result per row.", ""]
    by_metric: dict[str, list[dict]] = {}
    for r in ok:
        by_metric.setdefault(r["metric"], []).append(r)
    for metric, recs in sorted(by_metric.items()):
        unit = recs[0].get("unit", "")
        hib = recs[0].get("higher_is_better")
        out += [f"## {metric}", "", f"unit: {unit} ({'higher' if hib else 'lower'} is better)", "",
                "| GPUs | layout | value | e2e | SM MHz (reasons) | launches | older | revision | file |",
                "|---|---|---|---|---|---|---|---|---|"]
        rows: dict[tuple, list[dict]] = {}
        for r in recs:
            key = (r.get("n_gpus"), (r.get("config") or {}).get("parallelism"))
            rows.setdefault(key, []).append(r)
        for key in sorted(rows, key=lambda k: (k[0] or 0, str(k[1]))):
            rs = sorted(rows[key], key=lambda r: r["_mtime"])
            r = rs[-1]
            clk = r.get("clocks") or {}
            e2e = r.get("e2e") or {}
            rev = (((r.get("provenance") or {}).get("git") or {}).get("sha") or "")[:10]
            out.append(f"| {_fmt(key[0])} | {_fmt(key[1])} | {_fmt(r.get('value'))} | "
                       f"{_fmt(e2e.get('value'))} {e2e.get('unit', '') if e2e else ''} | "
                       f"{_fmt(clk.get('sm_mhz'))} ({', '.join(clk.get('reasons') or []) or 'none'}) | "
                       f"{_fmt(r.get('gpu_launches'))} | {len(rs) - 1} | {rev} | {r['_file']} |")
        out.append("")
    if failed:
        out += ["## Failed launches", "", "| file | run | error |", "|---|---|---|"]
        out += [f"| {f['file']} | {f['run']} | {f['error'].replace('|', '/')} |" for f in failed]
        out.append("")
    return "\n".join(out)


def report(directory: str | Path, out: str | Path | None = None) -> Path:
    ok, failed = collect(directory)
    path = Path(out) if out else Path(directory) / "SUMMARY.md"
    path.write_text(render(ok, failed))
    return path


__all__ = ["collect", "render", "report"]
