"""Spawn N CPU ranks (gloo) for multi-rank tests: per-rank tracebacks, bounded wall time.

Same role as the reference's ``run_ranks`` harness
(``tests/unit/backends/_neuron_gloo.py:59-126``).  Ranks rendezvous on
127.0.0.1 with a free port; a rank that raises reports its traceback and the
others are terminated when the deadline passes.
"""

from __future__ import annotations

import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, fn, args, q):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    try:
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        out = fn(rank, world, *args)
        q.put((rank, "ok", out))
    except BaseException:  # noqa: BLE001 - report everything to the parent
        q.put((rank, "err", traceback.format_exc()))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def run_ranks(fn, world: int, *args, timeout: float = 180.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results, errors = {}, {}
    import time

    deadline = time.time() + timeout
    while len(results) + len(errors) < world and time.time() < deadline:
        try:
            r, status, payload = q.get(timeout=max(0.1, deadline - time.time()))
        except Exception:
            break
        (results if status == "ok" else errors)[r] = payload
    for p in procs:
        p.join(timeout=5)
        if p.is_alive():
            p.terminate()
    if errors:
        raise RuntimeError("rank failures:\n" + "\n".join(f"[rank {r}]\n{tb}" for r, tb in sorted(errors.items())))
    if len(results) < world:
        raise TimeoutError(f"only {sorted(results)} of {world} ranks finished within {timeout}s")
    return [results[r] for r in range(world)]
