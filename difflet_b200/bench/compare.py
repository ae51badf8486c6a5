"""Compare two benchmark results (B against A), refusing comparisons that mean nothing.

Inputs are ``bench.py`` result lines (one JSON object per file, or the last JSON line of a log)
or bench-suite JSONL files (several launches of each arm).  Reference behaviour
(``difflet/bench/compare.py``):

* refused: a different metric, unit or workload (model, sequence length, batch, dtype) -- the
  two numbers do not measure the same thing;
* reported first: every setting that differs between the two (parallel layout, GPU count, GPU,
  clock-limit reasons, revision), since any of them can explain a difference;
* a control arm whose own repeated launches spread by more than ``noise`` (5 %) makes the
  comparison noisy: a difference below that spread is not a result;
* each metric keeps its direction (``higher_is_better``); the per-step value explains a
  difference and the end-to-end value decides it, and across different GPUs only the per-step
  value is compared.
"""

from __future__ import annotations

import json
import statistics
from pathlib import Path

WORKLOAD_KEYS = ("model", "seq_len", "global_batch", "height", "width", "frames")


class ComparisonRefused(ValueError):
    pass


def load(path: str | Path) -> list[dict]:
    """The result records in a file: every JSON object line that carries a ``metric`` (bench.py
    lines) or a ``result`` with one (suite records)."""
    out = []
    for line in Path(path).read_text().splitlines():
        line = line.strip()
        if not line.startswith("{"):
            continue
        try:
            rec = json.loads(line)
        except ValueError:
            continue
        if "metric" in rec:
            out.append(rec)
        elif isinstance(rec.get("result"), dict) and "metric" in rec["result"] and not rec.get("error"):
            out.append({**rec["result"], "provenance": rec.get("provenance", rec["result"].get("provenance"))})
    if not out:
        raise ComparisonRefused(f"{path}: no result records")
    return out


def _gpu(rec: dict) -> str | None:
    prov = rec.get("provenance") or {}
    dev = prov.get("device") if isinstance(prov, dict) else None
    return dev.get("gpu") if isinstance(dev, dict) else None


def _settings(rec: dict) -> dict:
    cfg = rec.get("config") or {}
    prov = rec.get("provenance") or {}
    return {"parallelism": cfg.get("parallelism"), "n_gpus": rec.get("n_gpus"), "gpu": _gpu(rec),
            "clock_reasons": tuple((rec.get("clocks") or {}).get("reasons") or ()),
            "revision": ((prov.get("git") or {}) if isinstance(prov, dict) else {}).get("sha"),
            "steps": rec.get("steps"), "warmup": rec.get("warmup"), "l2": cfg.get("l2")}


def _arm(recs: list[dict], key) -> dict | None:
    vals = [v for v in (key(r) for r in recs) if v is not None]
    if not vals:
        return None
    med = statistics.median(vals)
    return {"n": len(vals), "median": med, "spread": (max(vals) - min(vals)) / med if med else 0.0}


def compare(a: list[dict], b: list[dict], *, noise: float = 0.05) -> dict:
    ra, rb = a[0], b[0]
    for r in a + b:
        if (r.get("metric"), r.get("unit")) != (ra.get("metric"), ra.get("unit")):
            raise ComparisonRefused(f"different metrics: {ra.get('metric')!r} [{ra.get('unit')}] vs "
                                    f"{r.get('metric')!r} [{r.get('unit')}]")
    wa, wb = ({k: (r.get("config") or {}).get(k) for k in WORKLOAD_KEYS} for r in (ra, rb))
    if wa != wb or ra.get("dtype") != rb.get("dtype"):
        diff = {k: (wa[k], wb[k]) for k in WORKLOAD_KEYS if wa[k] != wb[k]}
        if ra.get("dtype") != rb.get("dtype"):
            diff["dtype"] = (ra.get("dtype"), rb.get("dtype"))
        raise ComparisonRefused(f"different workloads: {diff}")
    sa, sb = _settings(ra), _settings(rb)
    differs = {k: (sa[k], sb[k]) for k in sa if sa[k] != sb[k]}
    higher = bool(ra.get("higher_is_better", False))
    out = {"metric": ra["metric"], "unit": ra.get("unit"), "higher_is_better": higher, "differs": differs,
           "cross_machine": sa["gpu"] != sb["gpu"], "metrics": {}}

    def add(name, key, hib):
        xa, xb = _arm(a, key), _arm(b, key)
        if xa is None or xb is None or not xa["median"]:
            return
        ratio = xb["median"] / xa["median"]
        row = {"a": xa, "b": xb, "ratio": round(ratio, 4),
               "better": (ratio > 1) if hib else (ratio < 1)}
        row["noisy"] = xa["n"] > 1 and xa["spread"] > noise and abs(ratio - 1) <= xa["spread"]
        out["metrics"][name] = row

    add("value", lambda r: r.get("value"), higher)
    if not out["cross_machine"]:  # end-to-end numbers depend on the host as much as on the GPU
        e2e_hib = False if str(((ra.get("e2e") or {}).get("unit") or "")).startswith("s/") else higher
        add("e2e", lambda r: (r.get("e2e") or {}).get("value"), e2e_hib)
    out["noisy"] = any(m["noisy"] for m in out["metrics"].values())
    return out


def format_text(res: dict) -> str:
    lines = [f"{res['metric']} [{res['unit']}], {'higher' if res['higher_is_better'] else 'lower'} is better"]
    for k, (x, y) in res["differs"].items():
        lines.append(f"  differs: {k}: {x} -> {y}")
    if res["cross_machine"]:
        lines.append("  different GPUs: only the per-step value is compared")
    for name, m in res["metrics"].items():
        tag = "better" if m["better"] else "worse"
        if m["noisy"]:
            tag = "within the control's spread"
        lines.append(f"  {name}: {m['a']['median']:.6g} -> {m['b']['median']:.6g}  (B/A {m['ratio']:.4f}, {tag})")
    return "\n".join(lines)


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description="compare two benchmark results (B against A)")
    ap.add_argument("a")
    ap.add_argument("b")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--noise", type=float, default=0.05)
    args = ap.parse_args(argv)
    try:
        res = compare(load(args.a), load(args.b), noise=args.noise)
    except ComparisonRefused as exc:
        print(f"refused: {exc}")
        return 2
    print(json.dumps(res, default=str) if args.json else format_text(res))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
