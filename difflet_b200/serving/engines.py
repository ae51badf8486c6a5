"""Serving engines: in-process, resident worker process (heartbeat + recovery), replicas.

Reference behaviour (``difflet/serving/engines/resident_worker.py:51-1404``,
``difflet/serving/engines/replicated.py:20-82``):
  * one request runs at a time per replica (a run lock); a request that cannot
    get the lock within ``queue_timeout`` is refused (HTTP 429)
  * the resident worker is a separate spawned process that loads the pipeline
    once, runs a smoke request, then reports ready; it sends a heartbeat
    (state, stage, request id) every ``heartbeat_s``
  * recovery never fails open: on a request timeout, a lost heartbeat or a dead
    worker the engine cancels, waits a grace period, terminates, restarts the
    worker and fences (the in-flight request fails; later ones run on the new
    worker)
  * ``ReplicatedEngine`` spreads requests over N replicas (least loaded first); each replica
    is pinned to its own GPUs (``CUDA_VISIBLE_DEVICES``), and a replica whose parallel world is
    larger than one GPU runs as a group of rank processes (rank 0 answers, the others follow
    every request; ``parallel/groups.py`` rendezvous on 127.0.0.1)
  * a running request can be cancelled: the worker checks a shared flag between denoise
    steps (rank 0 decides, every rank of a group learns the decision through a broadcast at
    the same step) and the request ends with ``RequestCancelled``
"""

from __future__ import annotations

import multiprocessing as mp
import queue
import threading
import time
import traceback
import uuid
from typing import Any, Callable


class QueueTimeout(Exception):
    """No replica became free within the queue timeout (HTTP 429)."""


class EngineError(RuntimeError):
    pass


class RequestCancelled(EngineError):
    """The request was cancelled while it ran."""


class _Admission:
    """One running request per replica; at most ``max_queued`` more wait for it (beyond that a
    request is refused at once), each for at most ``queue_timeout`` seconds."""

    def __init__(self, queue_timeout: float, max_queued: int | None):
        self.queue_timeout = queue_timeout
        self.max_queued = max_queued
        self._lock = threading.Lock()
        self._guard = threading.Lock()
        self.waiting = 0

    def acquire(self):
        with self._guard:
            if self.max_queued is not None and self.waiting >= self.max_queued and self._lock.locked():
                raise QueueTimeout("server busy: queue full")
            self.waiting += 1
        try:
            if not self._lock.acquire(timeout=self.queue_timeout):
                raise QueueTimeout("server busy")
        finally:
            with self._guard:
                self.waiting -= 1

    def release(self):
        self._lock.release()


class InProcessEngine:
    """Runs ``generate_fn(request) -> result`` in this process (tests, single-process serving)."""

    def __init__(self, generate_fn: Callable[[dict], Any], queue_timeout: float = 30.0, max_queued: int | None = None):
        self.fn = generate_fn
        self.queue_timeout = queue_timeout
        self._adm = _Admission(queue_timeout, max_queued)
        self.ready = True
        self.healthy = True
        self.inflight = 0
        self.completed = 0

    def generate(self, request: dict, timeout: float | None = None):
        self._adm.acquire()
        self.inflight += 1
        try:
            out = self.fn(request)
            self.completed += 1
            return out
        finally:
            self.inflight -= 1
            self._adm.release()

    def close(self):
        pass


def _apply_env(env: dict | None) -> None:
    """Process environment of a worker (GPU pinning, rendezvous), before CUDA is initialised."""
    import os

    if env:
        os.environ.update({k: str(v) for k, v in env.items()})


def _call_run(run, req, should_cancel, **extra):
    """run(req) with the keyword arguments it declares among should_cancel / on_stage / request_id."""
    import inspect

    try:
        params = inspect.signature(run).parameters
    except (TypeError, ValueError):
        params = {}
    kw = {k: v for k, v in dict(extra, should_cancel=should_cancel).items() if k in params}
    return run(req, **kw)


def _follower_main(rank, world, port, env, factory, factory_kwargs, feed, cancel_flag):
    """Rank > 0 of a multi-GPU replica: same pipeline, runs every request rank 0 forwards."""
    _apply_env(dict(env or {}, RANK=rank, LOCAL_RANK=rank, WORLD_SIZE=world, MASTER_ADDR="127.0.0.1",
                    MASTER_PORT=port))
    from difflet_b200.parallel.groups import init_distributed

    init_distributed()
    run = factory(**factory_kwargs)
    decide = _group_cancel(cancel_flag)
    run({"__smoke__": True})
    while True:
        req = feed.get()
        if req is None:
            break
        try:
            _call_run(run, req, decide)
        except Exception:  # noqa: BLE001 - rank 0 reports the request's outcome
            pass


def _group_cancel(cancel_flag):
    """should_cancel() for every rank of a group: rank 0 reads the shared flag, a broadcast makes
    the decision the same on every rank at the same step (no rank leaves a collective early)."""
    import torch.distributed as dist

    def decide() -> bool:
        import torch

        if not dist.is_initialized() or dist.get_world_size() == 1:
            return bool(cancel_flag.value)
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        t = torch.tensor([int(cancel_flag.value) if dist.get_rank() == 0 else 0], device=dev)
        dist.broadcast(t, 0)
        return bool(t.item())

    return decide


def _worker_main(conn_req, conn_resp, hb, factory, factory_kwargs, heartbeat_s, env=None, world=1,
                 cancel_flag=None):
    """Worker process (rank 0 of its replica): build the pipeline, smoke-test it, serve requests,
    beat.  With world > 1 it first starts the replica's other ranks and rendezvouses with them."""
    _apply_env(env)
    state = {"state": "loading", "stage": "", "request_id": None}
    stop = threading.Event()
    followers, feeds = [], []

    def beat():
        while not stop.is_set():
            try:
                hb.put(dict(state, t=time.time()))
            except Exception:
                pass
            stop.wait(heartbeat_s)

    threading.Thread(target=beat, daemon=True).start()
    try:
        if world > 1:
            from difflet_b200.parallel.testing import free_port

            port = free_port()
            ctx = mp.get_context("spawn")
            for r in range(1, world):
                q = ctx.Queue()
                p = ctx.Process(target=_follower_main, args=(r, world, port, env, factory, factory_kwargs, q,
                                                             cancel_flag), daemon=True)
                p.start()
                followers.append(p)
                feeds.append(q)
            _apply_env({"RANK": 0, "LOCAL_RANK": 0, "WORLD_SIZE": world, "MASTER_ADDR": "127.0.0.1",
                        "MASTER_PORT": port})
            from difflet_b200.parallel.groups import init_distributed

            init_distributed()
        run = factory(**factory_kwargs)
        decide = _group_cancel(cancel_flag) if cancel_flag is not None else (lambda: False)
        state["state"] = "smoke"
        run({"__smoke__": True})
        state["state"] = "ready"
        conn_resp.put(("ready", None, None))
    except Exception:
        conn_resp.put(("fatal", None, traceback.format_exc()))
        stop.set()
        return
    while True:
        msg = conn_req.get()
        if msg is None:
            break
        rid, req = msg
        state.update(state="running", request_id=rid, stage="generate")
        if cancel_flag is not None:
            cancel_flag.value = 0
        for q in feeds:
            q.put(req)
        try:
            out = _call_run(run, req, decide, on_stage=lambda st: state.update(stage=st), request_id=rid)
            conn_resp.put(("ok", rid, out))
        except Exception as exc:  # noqa: BLE001
            kind = "cancelled" if type(exc).__name__ == "RequestCancelled" else "error"
            conn_resp.put((kind, rid, traceback.format_exc()))
        state.update(state="ready", request_id=None, stage="")
    for q in feeds:
        q.put(None)
    for p in followers:
        p.join(timeout=30)
    stop.set()


class ResidentWorkerEngine:
    """A pipeline resident in a spawned worker process, with heartbeat-based recovery.

    ``factory(**factory_kwargs)`` runs in the worker and returns ``run(request) -> result``
    (picklable result).  It must be importable by name (spawn)."""

    def __init__(self, factory, factory_kwargs=None, *, queue_timeout=30.0, request_timeout=600.0,
                 heartbeat_s=5.0, heartbeat_timeout=None, start_timeout=1800.0, max_queued=None,
                 devices: list | None = None, world: int = 1, env: dict | None = None):
        self.factory = factory
        self.factory_kwargs = dict(factory_kwargs or {})
        self.devices = list(devices) if devices is not None else None
        self.world = int(world)
        self.env = dict(env or {})
        if self.devices is not None:  # this replica's GPUs only (replica i of dp: its own slice)
            self.env["CUDA_VISIBLE_DEVICES"] = ",".join(str(d) for d in self.devices)
        self._current = None
        self.queue_timeout = queue_timeout
        self._adm = _Admission(queue_timeout, max_queued)
        self.request_timeout = request_timeout
        self.heartbeat_s = heartbeat_s
        self.heartbeat_timeout = heartbeat_timeout or max(6 * heartbeat_s, 30.0)
        self.start_timeout = start_timeout
        self._ctx = mp.get_context("spawn")
        self._cancel = self._ctx.Value("b", 0)
        self.ready = False
        self.healthy = True
        self.inflight = 0
        self.restarts = 0
        self.last_heartbeat = None
        self._start()

    def _start(self):
        self._req = self._ctx.Queue()
        self._resp = self._ctx.Queue()
        self._hb = self._ctx.Queue()
        self.proc = self._ctx.Process(target=_worker_main, args=(self._req, self._resp, self._hb, self.factory,
                                                                self.factory_kwargs, self.heartbeat_s, self.env,
                                                                self.world, self._cancel),
                                      daemon=False)
        self.proc.start()
        deadline = time.time() + self.start_timeout
        while time.time() < deadline:
            try:
                kind, _, payload = self._resp.get(timeout=1.0)
            except queue.Empty:
                if not self.proc.is_alive():
                    break
                continue
            if kind == "ready":
                self.ready, self.healthy = True, True
                return
            if kind == "fatal":
                self.healthy = False
                raise EngineError(f"worker failed to start:\n{payload}")
        self.healthy = False
        raise EngineError("worker did not become ready")

    def _drain_heartbeats(self):
        while True:
            try:
                self.last_heartbeat = self._hb.get_nowait()
            except queue.Empty:
                return

    def _recover(self, reason: str):
        """Terminate -> restart -> fence.  The caller's request fails with ``reason``."""
        self.ready = False
        try:
            self._req.put(None)
            self.proc.join(timeout=5)
        except Exception:
            pass
        if self.proc.is_alive():
            self.proc.terminate()
            self.proc.join(timeout=10)
            if self.proc.is_alive():
                self.proc.kill()
        self.restarts += 1
        self._start()
        raise EngineError(f"request failed, worker restarted ({reason})")

    def cancel(self, request_id: str) -> bool:
        """Ask the worker to stop the running request ``request_id`` at its next denoise step."""
        if self._current != request_id:
            return False
        self._cancel.value = 1
        return True

    def generate(self, request: dict, timeout: float | None = None, request_id: str | None = None):
        self._adm.acquire()
        self.inflight += 1
        try:
            rid = request_id or str(uuid.uuid4())
            self._current = rid
            self._req.put((rid, request))
            deadline = time.time() + (timeout or self.request_timeout)
            last_beat = time.time()
            while True:
                try:
                    kind, r, payload = self._resp.get(timeout=0.5)
                except queue.Empty:
                    self._drain_heartbeats()
                    if self.last_heartbeat is not None:
                        last_beat = max(last_beat, self.last_heartbeat.get("t", 0))
                    now = time.time()
                    if not self.proc.is_alive():
                        self._recover("worker died")
                    if now > deadline:
                        self._recover("request timeout")
                    if now - last_beat > self.heartbeat_timeout:
                        self._recover("heartbeat lost")
                    continue
                if r != rid:
                    continue  # a late answer for a request fenced off by a restart
                if kind == "ok":
                    return payload
                if kind == "cancelled":
                    raise RequestCancelled(f"request {rid} cancelled")
                raise EngineError(payload)
        finally:
            self._current = None
            self.inflight -= 1
            self._adm.release()

    def close(self):
        try:
            self._req.put(None)
            self.proc.join(timeout=5)
        finally:
            if self.proc.is_alive():
                self.proc.terminate()


class ReplicatedEngine:
    """Least-loaded dispatch over N replicas (``serve --dp-degree N``)."""

    def __init__(self, replicas: list):
        self.replicas = replicas

    @property
    def ready(self):
        return any(r.ready for r in self.replicas)

    @property
    def healthy(self):
        return all(r.healthy for r in self.replicas)

    def generate(self, request, timeout=None, request_id=None):
        order = sorted(self.replicas, key=lambda r: r.inflight)
        last = None
        for r in order:
            try:
                if request_id is not None and hasattr(r, "cancel"):
                    return r.generate(request, timeout, request_id=request_id)
                return r.generate(request, timeout)
            except QueueTimeout as exc:
                last = exc
        raise last or QueueTimeout("server busy")

    def cancel(self, request_id: str) -> bool:
        return any(r.cancel(request_id) for r in self.replicas if hasattr(r, "cancel"))

    def close(self):
        for r in self.replicas:
            r.close()
