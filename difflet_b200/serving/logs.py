"""Serve log files: one file per size slice and per day, under ``<cwd>/logs``.

Reference behaviour (``difflet/cli/serve.py:26-150``): ``difflet serve`` writes every record of the
root, uvicorn and access loggers to ``logs/<project>-<YYYYmmdd_HHMMSS>.log`` (project = the name
of the working directory) besides the console; a new file starts when the next record would take
the current one past 5 MB or when the local date changes, and up to 1024 files are kept.

This handler opens the next file itself (a new timestamped name, never a renamed ``.1``), so
readers that tail one file never see it move, and it deletes the oldest files of the same project
beyond ``keep``.
"""

from __future__ import annotations

import logging
import os
import threading
from datetime import datetime
from pathlib import Path

FILE_FORMAT = "%(asctime)s.%(msecs)03d %(levelname)s %(name)s %(message)s"
DATE_FORMAT = "%Y-%m-%d %H:%M:%S"


def project_name(cwd: Path | None = None) -> str:
    name = (cwd or Path.cwd()).name
    return name.replace(" ", "_") if name else "difflet"


class ServeLogHandler(logging.Handler):
    def __init__(self, log_dir: str | os.PathLike | None = None, project: str | None = None,
                 max_bytes: int = 5 * 1024 * 1024, keep: int = 1024, clock=datetime.now):
        super().__init__()
        self.dir = Path(log_dir) if log_dir is not None else Path.cwd() / "logs"
        self.dir.mkdir(parents=True, exist_ok=True)
        self.project = project or project_name()
        self.max_bytes = int(max_bytes)
        self.keep = int(keep)
        self.clock = clock
        self._io = threading.Lock()
        self._stream = None
        self._day = None
        self._size = 0
        self.path: Path | None = None
        self.setFormatter(logging.Formatter(FILE_FORMAT, DATE_FORMAT))
        self._open(self.clock())

    def _open(self, now: datetime) -> None:
        if self._stream is not None:
            self._stream.close()
        stem = f"{self.project}-{now.strftime('%Y%m%d_%H%M%S')}"
        path, n = self.dir / f"{stem}.log", 1
        while path.exists():  # two files in one second: keep both
            path, n = self.dir / f"{stem}-{n}.log", n + 1
        self._stream = open(path, "a", encoding="utf-8")
        self.path = path
        self._day = now.date()
        self._size = 0
        self._prune()

    def _prune(self) -> None:
        mine = sorted(self.dir.glob(f"{self.project}-*.log"), key=lambda p: p.stat().st_mtime)
        for p in mine[: max(0, len(mine) - self.keep)]:
            if p != self.path:
                try:
                    p.unlink()
                except OSError:
                    pass

    def emit(self, record: logging.LogRecord) -> None:
        try:
            data = (self.format(record) + "\n").encode("utf-8")
            with self._io:
                now = self.clock()
                if (self._stream is None or now.date() != self._day
                        or (self.max_bytes > 0 and self._size and self._size + len(data) > self.max_bytes)):
                    self._open(now)
                self._stream.write(data.decode("utf-8"))
                self._stream.flush()
                self._size += len(data)
        except Exception:  # noqa: BLE001 - logging must never take the server down
            self.handleError(record)

    def close(self) -> None:
        with self._io:
            if self._stream is not None:
                self._stream.close()
                self._stream = None
        super().close()


def configure_serve_logging(log_dir=None, project=None, max_bytes: int = 5 * 1024 * 1024,
                            keep: int = 1024) -> ServeLogHandler:
    """Console + file logging for ``serve`` on the root logger; the uvicorn, uvicorn.error and
    uvicorn.access loggers propagate to it (run uvicorn with ``log_config=None`` so it does not
    install handlers of its own)."""
    handler = ServeLogHandler(log_dir, project, max_bytes, keep)
    root = logging.getLogger()
    root.setLevel(logging.INFO)
    if not any(type(h) is logging.StreamHandler for h in root.handlers):
        console = logging.StreamHandler()
        console.setFormatter(logging.Formatter(FILE_FORMAT, DATE_FORMAT))
        root.addHandler(console)
    root.addHandler(handler)
    for name in ("uvicorn", "uvicorn.error", "uvicorn.access"):
        lg = logging.getLogger(name)
        lg.setLevel(logging.INFO)
        lg.handlers.clear()
        lg.propagate = True
    return handler


__all__ = ["ServeLogHandler", "configure_serve_logging", "project_name"]
