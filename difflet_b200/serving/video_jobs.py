"""Asynchronous video jobs: FIFO dispatch, state machine, local artefact storage.

Reference: ``difflet/serving/video_service.py:323-857`` and
``difflet/serving/video_jobs.py:137-431``: a job moves queued -> in_progress ->
completed | failed; one dispatcher thread runs jobs in arrival order through the
engine, encodes the frames and commits the file atomically (write to a temp
name, then rename).
"""

from __future__ import annotations

import os
import queue
import tempfile
import threading
import time
import uuid
from dataclasses import dataclass, field


@dataclass
class VideoJob:
    id: str
    request: dict
    status: str = "queued"
    created_at: float = field(default_factory=time.time)
    completed_at: float | None = None
    error: str | None = None
    path: str | None = None

    def public(self) -> dict:
        d = {"id": self.id, "object": "video", "status": self.status, "created_at": int(self.created_at),
             "prompt": self.request.get("prompt")}
        if self.completed_at:
            d["completed_at"] = int(self.completed_at)
        if self.error:
            d["error"] = {"message": self.error[-2000:]}
        return d


class VideoJobStore:
    def __init__(self, engine, directory: str | None, encode_video, fps: int = 16):
        self.engine = engine
        self.dir = directory or tempfile.mkdtemp(prefix="difflet_videos_")
        os.makedirs(self.dir, exist_ok=True)
        self.encode = encode_video
        self.fps = fps
        self.jobs: dict[str, VideoJob] = {}
        self._q: queue.Queue = queue.Queue()
        self._t = threading.Thread(target=self._loop, daemon=True)
        self._t.start()

    def create(self, request: dict) -> VideoJob:
        job = VideoJob(id="video_" + uuid.uuid4().hex[:24], request=request)
        self.jobs[job.id] = job
        self._q.put(job.id)
        return job

    def get(self, vid: str) -> VideoJob | None:
        return self.jobs.get(vid)

    def _loop(self):
        while True:
            vid = self._q.get()
            job = self.jobs[vid]
            job.status = "in_progress"
            try:
                frames = self.engine.generate(job.request)
                data = frames if isinstance(frames, (bytes, bytearray)) else self.encode(frames, self.fps)
                final = os.path.join(self.dir, vid + ".avi")
                tmp = final + ".tmp"
                with open(tmp, "wb") as f:
                    f.write(data)
                    f.flush()
                    os.fsync(f.fileno())
                os.replace(tmp, final)
                job.path = final
                job.status = "completed"
            except Exception as exc:  # noqa: BLE001
                job.status = "failed"
                job.error = repr(exc)
            job.completed_at = time.time()

    def wait(self, vid: str, timeout: float = 60.0) -> VideoJob:
        t0 = time.time()
        while time.time() - t0 < timeout:
            j = self.jobs[vid]
            if j.status in ("completed", "failed"):
                return j
            time.sleep(0.02)
        return self.jobs[vid]
