"""Bench suites: recipes x variants, run in sequence or in ABBA order, with an idle check before
every launch and one JSON record per launch.

Behaviour of the reference's suites (difflet/bench/suite.py:1-50, runner.py): a suite file is ::

    description: bf16 against MXFP8
    recipes: [flux]
    variants:
      bf16: {}
      mxfp8: {args: {quant: mxfp8}}
    compare: {control: bf16, candidate: mxfp8}
    order: ABBA
    repeats: 2

Runs are ``<recipe>/<variant>``.  With ``order: ABBA`` the control and candidate launches of a recipe
alternate control, candidate, candidate, control for ``repeats`` rounds, so drift of the machine
shows up as a spread between one arm's launches instead of as a speed-up of the other.  Each launch
is one ``generate`` process (under ``torchrun`` when the recipe needs more than one GPU); its
wall time and the engine's own result line (output path, seconds) go into a JSONL record together
with the idle report, the recipe's argv and the provenance of the run.  ``summarize`` gives each
run's median seconds and the candidate / control ratio per recipe.
"""

from __future__ import annotations

import json
import os
import statistics
import subprocess
import sys
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable

from difflet_b200.bench.recipe import Recipe, RecipeError, load_recipes, validate

SUITES_DIR = Path(__file__).with_name("suites")
TOP_LEVEL = frozenset({"description", "recipes", "variants", "compare", "order", "repeats"})
ORDERS = ("sequential", "ABBA")


@dataclass
class Launch:
    run_key: str        # "<recipe>/<variant>"
    recipe: Recipe      # the variant's args merged in
    index: int          # launch number of this run (0 ..)


@dataclass
class Suite:
    name: str
    recipes: list[str]
    variants: dict[str, dict]
    compare: dict | None = None
    order: str = "sequential"
    repeats: int = 1
    description: str = ""


def load_suite(name_or_path: str) -> Suite:
    import yaml

    p = Path(name_or_path)
    if not p.exists():
        p = SUITES_DIR / f"{name_or_path}.yaml"
    doc = yaml.safe_load(p.read_text()) or {}
    bad = set(doc) - TOP_LEVEL
    if bad:
        raise RecipeError(f"suite {p.name}: unknown keys {sorted(bad)}")
    order = doc.get("order", "sequential")
    if order not in ORDERS:
        raise RecipeError(f"suite {p.name}: order must be one of {ORDERS}")
    variants = doc.get("variants") or {"default": {}}
    cmp_ = doc.get("compare")
    if order == "ABBA":
        if not cmp_ or set(cmp_) != {"control", "candidate"} or not {cmp_["control"], cmp_["candidate"]} <= set(variants):
            raise RecipeError(f"suite {p.name}: ABBA needs compare: {{control, candidate}} naming two variants")
    repeats = int(doc.get("repeats", 1))
    if repeats < 1:
        raise RecipeError(f"suite {p.name}: repeats must be >= 1")
    return Suite(p.stem, list(doc.get("recipes") or []), dict(variants), cmp_, order, repeats,
                 doc.get("description", ""))


def plan(suite: Suite, recipes: dict[str, Recipe] | None = None) -> list[Launch]:
    """The launches of a suite in execution order (every recipe validated first)."""
    table = recipes if recipes is not None else load_recipes()
    runs: dict[str, dict[str, Recipe]] = {}
    for rn in suite.recipes:
        if rn not in table:
            raise RecipeError(f"suite {suite.name}: unknown recipe {rn!r}")
        runs[rn] = {}
        for vn, vbody in suite.variants.items():
            r = table[rn].with_args((vbody or {}).get("args"), name=f"{rn}/{vn}")
            runs[rn][vn] = validate(r)
    out: list[Launch] = []
    count: dict[str, int] = {}

    def add(rn, vn):
        key = f"{rn}/{vn}"
        out.append(Launch(key, runs[rn][vn], count.get(key, 0)))
        count[key] = count.get(key, 0) + 1

    for rn in suite.recipes:
        if suite.order == "ABBA":
            a, b = suite.compare["control"], suite.compare["candidate"]
            for _ in range(suite.repeats):
                for vn in (a, b, b, a):
                    add(rn, vn)
        else:
            for vn in suite.variants:
                for _ in range(suite.repeats):
                    add(rn, vn)
    return out


def gpus_needed(recipe: Recipe) -> int:
    a = recipe.args
    n = int(a.get("tp-degree", 1) or 1) * int(a.get("cp-degree", 1) or 1)
    return n * (2 if a.get("cfg-parallel") else 1) * int(a.get("dp", 1) or 1)


def command(recipe: Recipe, output: str, master_port: int = 29611) -> list[str]:
    """``python -m difflet_b200 generate ...``, under ``torchrun`` (127.0.0.1) for more than one GPU."""
    gen = ["-m", "difflet_b200", "generate", *recipe.argv(), "--output", output]
    n = gpus_needed(recipe)
    if n > 1:
        return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                "--master-addr", "127.0.0.1", f"--master-port={master_port}", *gen]
    return [sys.executable, *gen]


def _result_line(stdout: str) -> dict | None:
    for line in reversed(stdout.strip().splitlines()):
        line = line.strip()
        if line.startswith("{"):
            try:
                return json.loads(line)
            except ValueError:
                continue
    return None


def run(suite: Suite, launches: list[Launch], out_dir: Path | str, *,
        launcher: Callable[..., Any] = subprocess.run, idle: Callable[[list[int]], Any] | None = None,
        dry_run: bool = False, timeout_s: float = 3600.0, memory_sampler: Callable[[list[int]], Any] | None = None
        ) -> list[dict]:
    """Execute ``launches``; one JSONL record per launch in ``<out_dir>/<suite>.jsonl``.
    ``memory_sampler(devices)``: a context manager with ``summary()`` (``bench/memory.py``) run
    around each launch; its per-GPU and per-process peaks go into the record."""
    from difflet_b200.bench import provenance

    out_dir = Path(out_dir)
    if not dry_run:
        out_dir.mkdir(parents=True, exist_ok=True)
    results_path = out_dir / f"{suite.name}.jsonl"
    prov = provenance.collect() if not dry_run else {}
    records = []
    for i, ln in enumerate(launches):
        output = str(out_dir / f"{ln.run_key.replace('/', '__')}_{ln.index}")
        cmd = command(ln.recipe, output, 29611 + (i % 50))
        rec: dict[str, Any] = {"suite": suite.name, "run": ln.run_key, "launch": ln.index, "argv": cmd}
        if dry_run:
            records.append(rec)
            continue
        devices = list(range(gpus_needed(ln.recipe)))
        report = idle(devices) if idle is not None else None
        if report is not None:
            rec["idle_check"] = report.to_dict()
            if not report.idle:
                rec["error"] = "lane not idle: " + "; ".join(report.reasons())
                records.append(rec)
                _append(results_path, rec)
                continue
        t0 = time.perf_counter()
        sampler = memory_sampler(devices) if memory_sampler is not None else None
        try:
            if sampler is not None:
                sampler.__enter__()
            proc = launcher(cmd, capture_output=True, text=True, timeout=timeout_s,
                            env=ln.recipe.env(os.environ))
            rec["wall_s"] = round(time.perf_counter() - t0, 3)
            rec["returncode"] = proc.returncode
            rec["result"] = _result_line(proc.stdout or "")
            if proc.returncode != 0:
                rec["error"] = (proc.stderr or "")[-2000:]
        except subprocess.TimeoutExpired:
            rec["error"] = f"timeout after {timeout_s} s"
        finally:
            if sampler is not None:
                sampler.__exit__(None, None, None)
                rec["device_memory"] = sampler.summary()
        rec["provenance"] = prov
        records.append(rec)
        _append(results_path, rec)
    return records


def _append(path: Path, rec: dict) -> None:
    with open(path, "a") as f:
        f.write(json.dumps(rec, default=str) + "\n")


def summarize(suite: Suite, records: list[dict]) -> dict:
    """Median seconds per run (engine-reported, else wall time) and candidate / control ratios."""
    per: dict[str, list[float]] = {}
    for r in records:
        if r.get("error"):
            continue
        sec = (r.get("result") or {}).get("seconds", r.get("wall_s"))
        if sec is not None:
            per.setdefault(r["run"], []).append(float(sec))
    out: dict[str, Any] = {"runs": {k: {"median_s": statistics.median(v), "n": len(v), "spread_s": max(v) - min(v)}
                                    for k, v in per.items()}}
    if suite.compare:
        ratios = {}
        for rn in suite.recipes:
            a = out["runs"].get(f"{rn}/{suite.compare['control']}")
            b = out["runs"].get(f"{rn}/{suite.compare['candidate']}")
            if a and b and a["median_s"] > 0:
                ratios[rn] = round(b["median_s"] / a["median_s"], 4)
        out["candidate_over_control"] = ratios
    return out


__all__ = ["Launch", "Suite", "command", "gpus_needed", "load_suite", "plan", "run", "summarize"]
