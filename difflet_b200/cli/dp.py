"""Data-parallel replicas for batch generation: a filesystem claim protocol.

Reference: ``difflet/cli/dp/router.py:28-248`` and ``difflet/cli/dp/claims.py:19-76``.
A JSONL file of requests is split across ``dp`` worker processes, each pinned to
its own GPU subset (``CUDA_VISIBLE_DEVICES``).  A worker claims request ``i`` by
creating ``<work>/<i>.claim`` with O_CREAT | O_EXCL; it writes ``<i>.done`` or
``<i>.failed`` when finished, so a rerun resumes where the last one stopped and
no request runs twice.  The dp axis carries no per-step collective.
"""

from __future__ import annotations

import json
import os
import signal
import subprocess
import sys
from pathlib import Path

from difflet_b200.cli.runner import die_with_parent


def _pid_alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    return True


def _stale(claim: Path) -> bool:
    """A claim whose worker no longer runs (a crashed or killed earlier batch)."""
    try:
        pid = int(claim.read_text().strip() or "0")
    except (OSError, ValueError):
        return False  # being written right now, or not ours to judge
    return pid > 0 and not _pid_alive(pid)


def try_claim(work: Path, i: int) -> bool:
    """Claim request ``i`` (an exclusive create).  A rerun after a crash takes over the claims
    whose worker is gone: the stale claim is renamed away first, so of several workers that
    find it at once exactly one takes it over."""
    if (work / f"{i}.done").exists():
        return False
    claim = work / f"{i}.claim"
    for _ in range(2):
        try:
            fd = os.open(str(claim), os.O_CREAT | os.O_EXCL | os.O_WRONLY, 0o644)
        except FileExistsError:
            if not _stale(claim):
                return False
            try:
                os.rename(claim, work / f"{i}.claim.stale.{os.getpid()}")
            except FileNotFoundError:
                return False  # another worker took it over first
            continue
        os.write(fd, str(os.getpid()).encode())
        os.close(fd)
        return True
    return False


def mark(work: Path, i: int, ok: bool, info: dict | None = None) -> None:
    (work / f"{i}.{'done' if ok else 'failed'}").write_text(json.dumps(info or {}))


def load_requests(path: str) -> list[dict]:
    return [json.loads(l) for l in Path(path).read_text().splitlines() if l.strip()]


def worker_loop(requests: list[dict], work: Path, generate_one, replica: tuple | None = None) -> int:
    """Run the requests this worker gets: by claim (first free worker takes the next request), or
    with ``replica`` = (r, dp) statically every dp-th request starting at r (still claimed, so
    a rerun skips what is done)."""
    failures = 0
    for i, req in enumerate(requests):
        if replica is not None and i % replica[1] != replica[0]:
            continue
        if not try_claim(work, i):
            continue
        try:
            out = generate_one(req, i)
            mark(work, i, True, {"output": out})
        except Exception as exc:  # noqa: BLE001 - recorded, not fatal to the other requests
            failures += 1
            mark(work, i, False, {"error": repr(exc)})
    return failures


def run_router(argv_worker: list[str], dp: int, gpus_per_replica: int, work: str, schedule: str = "claim") -> int:
    """Spawn ``dp`` worker processes of ``python -m difflet_b200 <argv_worker>`` on disjoint GPUs
    (``schedule``: claim or static, see ``worker_loop``)."""
    Path(work).mkdir(parents=True, exist_ok=True)
    procs = []
    for r in range(dp):
        env = dict(os.environ)
        env["CUDA_VISIBLE_DEVICES"] = ",".join(str(r * gpus_per_replica + k) for k in range(gpus_per_replica))
        env["DIFFLET_DP_RANK"] = str(r)
        # a worker owns its GPUs outright: SIGKILL it if the router dies, so no orphan keeps them
        procs.append(subprocess.Popen([sys.executable, "-m", "difflet_b200"] + argv_worker, env=env,
                                      preexec_fn=die_with_parent(signal.SIGKILL)))
    return max(p.wait() for p in procs)
