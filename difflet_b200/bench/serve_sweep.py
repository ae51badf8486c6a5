"""``difflet serve`` throughput sweep: 1..8 concurrent image requests against one server.

The Qwen-Image serving benchmark is a sweep of 1-8 concurrent requests.  The reference
server answers one request per replica at a time and refuses with HTTP 429 once a request has
waited longer than the queue timeout (reference ``README.md:137-138``; ``--dp-degree N`` runs N replicas).
This tool measures the same thing here: for each concurrency level c it runs c client threads,
each sending ``rounds`` requests back to back to ``POST /v1/images/generations``, and reports the
completed requests per second, latency percentiles and the refusals.

Against a running server::

    python -m difflet_b200.bench.serve_sweep --url http://127.0.0.1:8000 --steps 10

or start one (random-init weights, its own port), sweep, and stop it::

    python -m difflet_b200.bench.serve_sweep --model-id Qwen/Qwen-Image --steps 10 [--dp-degree N]
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time


def _post(url: str, payload: dict, api_key: str | None, timeout: float):
    import requests

    headers = {"Authorization": f"Bearer {api_key}"} if api_key else {}
    t0 = time.perf_counter()
    try:
        r = requests.post(url, json=payload, headers=headers, timeout=timeout)
        return r.status_code, time.perf_counter() - t0
    except Exception:  # noqa: BLE001 - a dropped connection counts as a failure of this request
        return -1, time.perf_counter() - t0


def _pct(xs, q):
    if not xs:
        return None
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))]


def sweep(base_url: str, levels=(1, 2, 4, 8), rounds: int = 2, payload: dict | None = None,
          api_key: str | None = None, timeout: float = 900.0) -> list[dict]:
    """One row per concurrency level: completed / refused / failed counts, requests per second
    over the level's wall time, latency p50 / p95 / max of the completed requests."""
    url = base_url.rstrip("/") + "/v1/images/generations"
    payload = dict(payload or {"prompt": "a lighthouse at dusk", "size": "1024x1024", "num_inference_steps": 10})
    rows = []
    for c in levels:
        results = []
        lock = threading.Lock()

        def client():
            for _ in range(rounds):
                out = _post(url, payload, api_key, timeout)
                with lock:
                    results.append(out)

        threads = [threading.Thread(target=client) for _ in range(c)]
        t0 = time.perf_counter()
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        wall = time.perf_counter() - t0
        ok = [dt for code, dt in results if code == 200]
        rows.append({"concurrency": c, "requests": len(results), "completed": len(ok),
                     "refused_429": sum(1 for code, _ in results if code == 429),
                     "failed": sum(1 for code, _ in results if code not in (200, 429)),
                     "wall_s": round(wall, 3), "requests_per_s": round(len(ok) / wall, 4) if wall > 0 else None,
                     "latency_p50_s": _pct(ok, 0.5), "latency_p95_s": _pct(ok, 0.95),
                     "latency_max_s": max(ok) if ok else None})
    return rows


def wait_ready(base_url: str, timeout: float, proc=None) -> bool:
    import requests

    deadline = time.time() + timeout
    while time.time() < deadline:
        if proc is not None and proc.poll() is not None:
            return False
        try:
            if requests.get(base_url.rstrip("/") + "/ready", timeout=5).status_code == 200:
                return True
        except Exception:  # noqa: BLE001 - not listening yet
            pass
        time.sleep(2.0)
    return False


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--url", default=None, help="a running server; else start one for --model-id")
    ap.add_argument("--model-id", default="Qwen/Qwen-Image")
    ap.add_argument("--dp-degree", type=int, default=1)
    ap.add_argument("--quant", default=None, choices=[None, "mxfp8"])
    ap.add_argument("--size", default="1024x1024")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--levels", default="1,2,4,8")
    ap.add_argument("--rounds", type=int, default=2, help="requests per client thread per level")
    ap.add_argument("--start-timeout", type=float, default=900.0)
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    api_key = os.environ.get("DIFFLET_API_KEY")
    proc = None
    url = args.url
    if url is None:
        from difflet_b200.parallel.testing import free_port

        port = free_port()
        url = f"http://127.0.0.1:{port}"
        cmd = [sys.executable, "-m", "difflet_b200.cli.main", "serve", "--model-id", args.model_id, "--random-weights",
               "--host", "127.0.0.1", "--port", str(port), "--dp-degree", str(args.dp_degree),
               "--queue-timeout", "600"]
        if args.quant:
            cmd += ["--quant", args.quant]
        proc = subprocess.Popen(cmd)
        if not wait_ready(url, args.start_timeout, proc):
            proc.terminate()
            print(json.dumps({"error": "server did not become ready"}))
            return 1
    try:
        payload = {"prompt": "a lighthouse at dusk", "size": args.size, "num_inference_steps": args.steps}
        levels = tuple(int(x) for x in args.levels.split(",") if x)
        rows = sweep(url, levels, args.rounds, payload, api_key)
    finally:
        if proc is not None:
            proc.terminate()
            try:
                proc.wait(timeout=60)
            except subprocess.TimeoutExpired:
                proc.kill()
    result = {"metric": "serve throughput sweep", "model": args.model_id, "replicas": args.dp_degree,
              "size": args.size, "steps": args.steps, "rows": rows}
    print(json.dumps(result))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(result, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
