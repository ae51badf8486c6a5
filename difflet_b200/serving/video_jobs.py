"""Asynchronous video jobs: a persistent state machine, FIFO dispatch, cancellation, artifacts.

Reference behaviour (``difflet/serving/video_jobs.py:137-431``,
``difflet/serving/video_service.py:323-857``): a job moves ``queued -> in_progress ->
completed | failed``, or to ``cancelled`` from either non-terminal state; every transition is
a compare-and-set on the job's current status (a conflicting transition raises), and
terminal jobs never change again.  One dispatcher runs jobs in arrival order through the
engine, encodes the frames and publishes the file.

Here the repository is durable: each job is one JSON record written atomically (temporary
file + fsync + rename) in the job directory, so a restarted server lists the same jobs; jobs
that were running when the process stopped become ``failed`` ("interrupted"), queued ones are
dispatched again.  Finished videos are published as immutable content-addressed generations
(``artifact_manager.py``) and, when an S3-compatible store is configured, uploaded there and
served by presigned URL (``artifacts.py``).
"""

from __future__ import annotations

import json
import os
import queue
import tempfile
import threading
import time
import uuid
from dataclasses import asdict, dataclass, field

STATES = ("queued", "in_progress", "completed", "failed", "cancelled")
TERMINAL = frozenset({"completed", "failed", "cancelled"})
_ALLOWED = {"queued": {"in_progress", "cancelled", "failed"}, "in_progress": {"completed", "failed", "cancelled"}}


class VideoJobNotFound(KeyError):
    pass


class InvalidTransition(RuntimeError):
    """The job is not in the status the transition expects."""


@dataclass
class VideoJob:
    id: str
    request: dict
    status: str = "queued"
    created_at: float = field(default_factory=time.time)
    started_at: float | None = None
    completed_at: float | None = None
    error: str | None = None
    path: str | None = None
    digest: str | None = None
    url: str | None = None

    def public(self) -> dict:
        d = {"id": self.id, "object": "video", "status": self.status, "created_at": int(self.created_at),
             "prompt": self.request.get("prompt")}
        if self.completed_at:
            d["completed_at"] = int(self.completed_at)
        if self.error:
            d["error"] = {"message": self.error[-2000:]}
        if self.digest:
            d["sha256"] = self.digest
        if self.url:
            d["url"] = self.url
        return d


class VideoJobRepository:
    """Durable job records: ``<dir>/<id>.json``, replaced atomically on every transition."""

    def __init__(self, directory: str):
        self.dir = directory
        os.makedirs(directory, exist_ok=True)
        self._jobs: dict[str, VideoJob] = {}
        self._lock = threading.Lock()
        for name in sorted(os.listdir(directory)):
            if name.endswith(".json"):
                try:
                    with open(os.path.join(directory, name)) as f:
                        job = VideoJob(**json.load(f))
                except (OSError, ValueError, TypeError):
                    continue  # a torn or foreign file is not a job
                self._jobs[job.id] = job

    def _save(self, job: VideoJob) -> None:
        path = os.path.join(self.dir, job.id + ".json")
        tmp = path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(asdict(job), f)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)

    def create(self, request: dict) -> VideoJob:
        job = VideoJob(id="video_" + uuid.uuid4().hex[:24], request=dict(request))
        with self._lock:
            self._jobs[job.id] = job
            self._save(job)
        return job

    def get(self, vid: str) -> VideoJob | None:
        return self._jobs.get(vid)

    def require(self, vid: str) -> VideoJob:
        job = self._jobs.get(vid)
        if job is None:
            raise VideoJobNotFound(vid)
        return job

    def transition(self, vid: str, to: str, *, expect: str | tuple | None = None, **fields) -> VideoJob:
        """Compare-and-set: move job ``vid`` to ``to`` if its status is ``expect`` (any allowed
        predecessor when None) and the move is legal; returns the updated job."""
        if to not in STATES:
            raise ValueError(f"unknown job status {to!r}")
        with self._lock:
            job = self.require(vid)
            allowed = (expect,) if isinstance(expect, str) else (expect or tuple(_ALLOWED))
            if job.status not in allowed or to not in _ALLOWED.get(job.status, ()):
                raise InvalidTransition(f"{vid}: {job.status} -> {to}")
            job.status = to
            for k, v in fields.items():
                setattr(job, k, v)
            if to == "in_progress":
                job.started_at = time.time()
            if to in TERMINAL:
                job.completed_at = time.time()
            self._save(job)
            return job

    def list(self, *, after: str | None = None, limit: int = 20, status: str | None = None) -> list[VideoJob]:
        jobs = sorted(self._jobs.values(), key=lambda j: (j.created_at, j.id))
        if status:
            jobs = [j for j in jobs if j.status == status]
        if after:
            ids = [j.id for j in jobs]
            jobs = jobs[ids.index(after) + 1:] if after in ids else []
        return jobs[:limit]

    def delete(self, vid: str) -> None:
        with self._lock:
            job = self.require(vid)
            if job.status not in TERMINAL:
                raise InvalidTransition(f"{vid} is {job.status}; cancel it first")
            self._jobs.pop(vid)
            try:
                os.unlink(os.path.join(self.dir, vid + ".json"))
            except FileNotFoundError:
                pass

    def expired(self, ttl_s: float, now: float | None = None) -> list[VideoJob]:
        now = time.time() if now is None else now
        return [j for j in self._jobs.values() if j.status in TERMINAL and j.completed_at
                and now - j.completed_at > ttl_s]

    def recover(self) -> list[VideoJob]:
        """After a restart: running jobs failed (interrupted); returns the queued ones, oldest first."""
        for j in list(self._jobs.values()):
            if j.status == "in_progress":
                self.transition(j.id, "failed", expect="in_progress", error="interrupted by a server restart")
        return self.list(status="queued", limit=1 << 30)


class JobAdmissionError(RuntimeError):
    """A job the service cannot take now (its queue or its job table is full)."""


class VideoJobStore:
    """The video service: repository + dispatcher thread + artifact publication + cancellation.

    ``engine.generate(request)`` returns uint8 frames (or encoded bytes); ``engine.cancel(id)``,
    when the engine has it, stops a running request between denoise steps.

    Bounds, as in the reference service (``difflet/serving/video_service.py:165-260``): at most
    ``max_queued`` jobs wait behind the running one and at most ``max_jobs`` records exist (a
    new job beyond either is refused); a job that waited longer than ``queue_timeout_s`` fails
    without running, one that runs longer than ``request_timeout_s`` is cancelled and fails as
    timed out; finished jobs older than ``retention_s`` are deleted with their files by a sweep
    every ``sweep_interval_s``."""

    def __init__(self, engine, directory: str | None, encode_video, fps: int = 16, artifact_store=None, *,
                 max_queued: int = 64, max_jobs: int = 4096, queue_timeout_s: float | None = None,
                 request_timeout_s: float | None = None, retention_s: float = 25 * 3600.0,
                 sweep_interval_s: float = 300.0):
        from difflet_b200.serving.artifact_manager import ImmutableArtifacts

        if max_queued < 0 or max_jobs < 1 or retention_s <= 0 or sweep_interval_s <= 0:
            raise ValueError("max_queued >= 0, max_jobs >= 1 and positive retention / sweep interval required")
        self.max_queued, self.max_jobs = int(max_queued), int(max_jobs)
        self.queue_timeout_s, self.request_timeout_s = queue_timeout_s, request_timeout_s
        self.retention_s, self.sweep_interval_s = float(retention_s), float(sweep_interval_s)
        self._timed_out: set = set()
        self.engine = engine
        self.dir = directory or tempfile.mkdtemp(prefix="difflet_videos_")
        self.repo = VideoJobRepository(os.path.join(self.dir, "jobs"))
        self.artifacts = ImmutableArtifacts(os.path.join(self.dir, "artifacts"))
        self.remote = artifact_store
        self.encode = encode_video
        self.fps = fps
        self._q: queue.Queue = queue.Queue()
        self._running: str | None = None
        for job in self.repo.recover():
            self._q.put(job.id)
        # files whose job record is gone (a crash between the two deletions), and remote objects
        # whose deletion failed earlier
        self.artifacts.sweep(keep=list(self.repo._jobs))
        self._pending_path = os.path.join(self.dir, "pending_remote_deletes.json")
        self.retry_remote_deletes()
        self._t = threading.Thread(target=self._loop, daemon=True)
        self._t.start()
        self._stop = threading.Event()
        self._sweeper = threading.Thread(target=self._sweep_loop, daemon=True)
        self._sweeper.start()

    def close(self) -> None:
        self._stop.set()

    # ------------------------------------------------------------------ retention
    def sweep_expired(self, now: float | None = None) -> list:
        """Delete finished jobs older than the retention (record, local and remote files)."""
        now = time.time() if now is None else now
        gone = []
        for job in list(self.repo._jobs.values()):
            if job.status in TERMINAL and now - (job.completed_at or job.created_at) > self.retention_s:
                try:
                    self.delete(job.id)
                    gone.append(job.id)
                except (VideoJobNotFound, InvalidTransition):
                    pass
        return gone

    def _sweep_loop(self):
        while not self._stop.wait(self.sweep_interval_s):
            try:
                self.sweep_expired()
            except Exception:  # noqa: BLE001 - the next sweep tries again
                pass

    # ------------------------------------------------------------------ deletion
    def _pending(self) -> list:
        try:
            with open(self._pending_path) as f:
                return list(json.load(f))
        except (FileNotFoundError, ValueError):
            return []

    def _write_pending(self, keys: list) -> None:
        tmp = self._pending_path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(sorted(set(keys)), f)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, self._pending_path)

    def retry_remote_deletes(self) -> int:
        """Delete the remote objects whose deletion failed before; returns how many are left."""
        if self.remote is None or not hasattr(self.remote, "delete"):
            return len(self._pending())
        left = []
        for key in self._pending():
            try:
                self.remote.delete(key)
            except OSError:
                left.append(key)
        if left or os.path.exists(self._pending_path):
            self._write_pending(left)
        return len(left)

    def delete(self, vid: str) -> None:
        """Delete a finished job: its record, its local generations and its remote object.  A
        remote deletion that fails is recorded and retried on the next delete and at start-up."""
        self.repo.delete(vid)
        self.artifacts.delete(vid)
        if self.remote is not None and hasattr(self.remote, "delete"):
            key = f"videos/{vid}.avi"
            try:
                self.remote.delete(key)
            except OSError:
                self._write_pending(self._pending() + [key])
            self.retry_remote_deletes()

    @property
    def jobs(self) -> dict:
        return self.repo._jobs

    def queued(self) -> int:
        return sum(1 for j in self.repo._jobs.values() if j.status == "queued")

    def create(self, request: dict) -> VideoJob:
        if self.queued() >= self.max_queued:
            raise JobAdmissionError(f"{self.max_queued} video jobs are already waiting")
        if len(self.repo._jobs) >= self.max_jobs:
            self.sweep_expired()
            if len(self.repo._jobs) >= self.max_jobs:
                raise JobAdmissionError(f"the service holds {self.max_jobs} jobs; delete finished ones")
        job = self.repo.create(request)
        self._q.put(job.id)
        return job

    def get(self, vid: str) -> VideoJob | None:
        return self.repo.get(vid)

    def cancel(self, vid: str) -> VideoJob:
        """Cancel a queued job at once, or a running one between its denoise steps."""
        job = self.repo.require(vid)
        if job.status == "queued":
            try:
                return self.repo.transition(vid, "cancelled", expect="queued")
            except InvalidTransition:
                job = self.repo.require(vid)  # the dispatcher took it meanwhile
        if job.status == "in_progress" and hasattr(self.engine, "cancel"):
            self.engine.cancel(vid)
        return self.repo.require(vid)

    def _loop(self):
        while True:
            vid = self._q.get()
            job = self.repo.get(vid)
            if job is not None and job.status == "queued" and self.queue_timeout_s is not None \
                    and time.time() - job.created_at > self.queue_timeout_s:
                try:
                    self.repo.transition(vid, "failed", expect="queued",
                                         error=f"timed out after {self.queue_timeout_s:g} s in the queue")
                except InvalidTransition:
                    pass
                continue
            try:
                self.repo.transition(vid, "in_progress", expect="queued")
            except (InvalidTransition, VideoJobNotFound):
                continue  # cancelled while queued
            self._running = vid
            watch = None
            if self.request_timeout_s is not None and hasattr(self.engine, "cancel"):
                def _expire(v=vid):
                    self._timed_out.add(v)
                    self.engine.cancel(v)

                watch = threading.Timer(self.request_timeout_s, _expire)
                watch.daemon = True
                watch.start()
            try:
                req = dict(self.repo.require(vid).request)
                frames = self.engine.generate(req, request_id=vid) if _takes_request_id(self.engine) \
                    else self.engine.generate(req)
                data = frames if isinstance(frames, (bytes, bytearray)) else self.encode(frames, self.fps)
                gen = self.artifacts.publish(vid, {"video.avi": bytes(data)})
                url = None
                if self.remote is not None:
                    ref = self.remote.put_bytes(f"videos/{vid}.avi", bytes(data), "video/x-msvideo")
                    url = self.remote.get_url(ref)
                self.repo.transition(vid, "completed", expect="in_progress", path=str(gen.file("video.avi")),
                                     digest=gen.digest, url=url)
            except Exception as exc:  # noqa: BLE001
                cancelled = type(exc).__name__ in ("RequestCancelled",) or "cancelled" in str(exc).lower()
                timed_out = vid in self._timed_out
                to = "failed" if timed_out or not cancelled else "cancelled"
                if not (timed_out or cancelled):  # the detail stays in the server log
                    import logging

                    logging.getLogger("difflet_b200.serving.video").error("video %s failed: %r", vid, exc)
                err = (f"timed out after {self.request_timeout_s:g} s" if timed_out
                       else None if cancelled else f"generation failed: {type(exc).__name__}")
                try:
                    self.repo.transition(vid, to, expect="in_progress", error=err)
                except InvalidTransition:
                    pass
            finally:
                if watch is not None:
                    watch.cancel()
                self._timed_out.discard(vid)
                self._running = None

    def wait(self, vid: str, timeout: float = 60.0) -> VideoJob:
        t0 = time.time()
        while time.time() - t0 < timeout:
            j = self.repo.require(vid)
            if j.status in TERMINAL:
                return j
            time.sleep(0.02)
        return self.repo.require(vid)


def _takes_request_id(engine) -> bool:
    import inspect

    try:
        return "request_id" in inspect.signature(engine.generate).parameters
    except (TypeError, ValueError):
        return False


__all__ = ["InvalidTransition", "JobAdmissionError", "STATES", "VideoJob", "VideoJobNotFound", "VideoJobRepository", "VideoJobStore"]
