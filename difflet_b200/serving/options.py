"""Options of ``difflet serve`` in one validated record.

Reference behaviour (difflet/serving/options.py:21-86): the server's model and parallel flags, the
HTTP endpoint, the API key (kept out of ``repr``), the number of replicas, the admission limits
(one running request per replica, ``max_queued_requests`` waiting, each for at most
``queue_timeout`` seconds, refused with HTTP 429 beyond either) and the worker's request timeout,
heartbeat interval and start timeout.  Values are checked once here so a bad flag fails at start,
not at the first request.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field


@dataclass
class ServeOptions:
    model_id: str
    host: str = "0.0.0.0"
    port: int = 8000
    api_key: str | None = field(default=None, repr=False)
    replicas: int = 1
    max_queued_requests: int = 8
    queue_timeout: float = 30.0
    request_timeout: float = 600.0
    heartbeat_interval: float = 5.0
    start_timeout: float = 1800.0

    def __post_init__(self):
        if not 0 < self.port < 65536:
            raise ValueError(f"port must be in 1..65535, got {self.port}")
        if self.replicas < 1:
            raise ValueError(f"replicas must be >= 1, got {self.replicas}")
        if self.max_queued_requests < 0:
            raise ValueError(f"max_queued_requests must be >= 0, got {self.max_queued_requests}")
        for name in ("queue_timeout", "request_timeout", "start_timeout"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be > 0, got {getattr(self, name)}")
        if not 0.05 <= self.heartbeat_interval <= self.request_timeout:
            raise ValueError(f"heartbeat_interval must be in [0.05, request_timeout], got {self.heartbeat_interval}")

    @classmethod
    def from_args(cls, a) -> "ServeOptions":
        from difflet_b200 import envs

        g = lambda name, default: default if getattr(a, name, None) is None else getattr(a, name)  # noqa: E731
        return cls(model_id=a.model_id, host=g("host", "0.0.0.0"), port=int(g("port", 8000)),
                   api_key=getattr(a, "api_key", None) or os.environ.get("DIFFLET_API_KEY"),
                   replicas=max(1, int(g("dp_degree", 1))), max_queued_requests=int(g("max_queued_requests", 8)),
                   queue_timeout=float(g("queue_timeout", envs.DIFFLET_SERVE_QUEUE_TIMEOUT_S)),
                   request_timeout=float(g("request_timeout", 600.0)),
                   heartbeat_interval=float(g("heartbeat_interval", envs.DIFFLET_HEARTBEAT_S)))

    def engine_kwargs(self) -> dict:
        return {"queue_timeout": self.queue_timeout, "request_timeout": self.request_timeout,
                "heartbeat_s": self.heartbeat_interval, "start_timeout": self.start_timeout,
                "max_queued": self.max_queued_requests}


__all__ = ["ServeOptions"]
