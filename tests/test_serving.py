"""Serving: OpenAI routes, auth, 429 admission, video jobs, resident-worker recovery (fake adapters)."""

import base64
import threading
import time

import pytest
import torch
from fastapi.testclient import TestClient

from difflet_b200.serving.api import create_app, normalize_chat_request
from difflet_b200.serving.engines import EngineError, InProcessEngine, ResidentWorkerEngine


def _img(req):
    h, w = req.get("height", 16), req.get("width", 16)
    return torch.full((h, w, 3), 7, dtype=torch.uint8)


def test_chat_completion_image_and_auth():
    app = create_app(InProcessEngine(_img), "flux", api_key="k")
    c = TestClient(app)
    assert c.get("/health").json()["status"] == "ok"
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "a cat"}]})
    assert r.status_code == 401
    r = c.post("/v1/chat/completions", headers={"Authorization": "Bearer k"},
               json={"messages": [{"role": "user", "content": "a cat"}], "extra_body": {"size": "32x24"}})
    assert r.status_code == 200
    url = r.json()["choices"][0]["message"]["content"][0]["image_url"]["url"]
    png = base64.b64decode(url.split(",", 1)[1])
    assert png[:4] == b"\x89PNG"
    r = c.post("/v1/images/generations", headers={"Authorization": "Bearer k"}, json={"prompt": "x", "size": "8x8"})
    assert r.status_code == 200 and r.json()["data"][0]["b64_json"]


def test_normalize_chat_request():
    req = normalize_chat_request({"messages": [{"role": "user", "content": [{"type": "text", "text": "hi"}]}],
                                  "extra_body": {"num_inference_steps": 4, "seed": 3, "size": "64x32"}})
    assert req == {"prompt": "hi", "width": 64, "height": 32, "num_inference_steps": 4, "seed": 3}


def test_busy_returns_429():
    gate = threading.Event()

    def slow(req):
        gate.wait(5)
        return _img(req)

    eng = InProcessEngine(slow, queue_timeout=0.2)
    c = TestClient(create_app(eng, "flux"))
    t = threading.Thread(target=lambda: c.post("/v1/chat/completions",
                                               json={"messages": [{"role": "user", "content": "a"}]}))
    t.start()
    time.sleep(0.2)
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "b"}]})
    gate.set()
    t.join()
    assert r.status_code == 429


def test_video_job_lifecycle(tmp_path):
    eng = InProcessEngine(lambda req: torch.zeros(5, 16, 16, 3, dtype=torch.uint8))
    c = TestClient(create_app(eng, "wan", output="video", video_dir=str(tmp_path)))
    r = c.post("/v1/videos", json={"prompt": "waves", "size": "16x16"})
    vid = r.json()["id"]
    job = c.app.state.jobs.wait(vid, 10)
    assert job.status == "completed"
    assert c.get(f"/v1/videos/{vid}").json()["status"] == "completed"
    data = c.get(f"/v1/videos/{vid}/content").content
    assert data[:4] == b"RIFF" and data[8:12] == b"AVI "


# --- resident worker (spawned process) with fake runners ---------------------------------

def fake_runner(mode="ok", delay=0.0):
    def run(req):
        if req.get("__smoke__"):
            return None
        if mode == "crash" and req.get("crash"):
            import os

            os._exit(3)
        if req.get("sleep"):
            time.sleep(req["sleep"])
        return {"echo": req.get("prompt")}

    return run


@pytest.mark.slow
def test_resident_worker_recovers_from_crash_and_timeout():
    eng = ResidentWorkerEngine(fake_runner, {"mode": "crash"}, heartbeat_s=0.2, request_timeout=3.0,
                               start_timeout=60)
    try:
        assert eng.ready and eng.generate({"prompt": "a"}) == {"echo": "a"}
        with pytest.raises(EngineError):
            eng.generate({"prompt": "b", "crash": True})
        assert eng.restarts == 1 and eng.ready
        assert eng.generate({"prompt": "c"}) == {"echo": "c"}  # fenced: the new worker serves
        with pytest.raises(EngineError):
            eng.generate({"prompt": "d", "sleep": 10}, timeout=1.0)
        assert eng.restarts == 2 and eng.generate({"prompt": "e"}) == {"echo": "e"}
    finally:
        eng.close()


def test_queue_full_refused_at_once_and_options():
    """One request runs, ``max_queued`` wait; the next is refused without waiting."""
    from difflet_b200.serving.engines import QueueTimeout
    from difflet_b200.serving.options import ServeOptions

    gate = threading.Event()
    eng = InProcessEngine(lambda req: (gate.wait(5), req)[1], queue_timeout=5.0, max_queued=1)
    running = threading.Thread(target=lambda: eng.generate({"i": 0}))
    running.start()
    time.sleep(0.1)
    waiting = threading.Thread(target=lambda: eng.generate({"i": 1}))
    waiting.start()
    time.sleep(0.1)
    t0 = time.time()
    try:
        eng.generate({"i": 2})
        refused = False
    except QueueTimeout as exc:
        refused = "queue full" in str(exc)
    assert refused and time.time() - t0 < 1.0
    gate.set()
    running.join()
    waiting.join()
    assert eng.completed == 2

    o = ServeOptions(model_id="flux", api_key="secret", max_queued_requests=3)
    assert "secret" not in repr(o) and o.engine_kwargs()["max_queued"] == 3
    for bad in ({"port": 0}, {"replicas": 0}, {"queue_timeout": 0}, {"heartbeat_interval": 0.0}):
        with pytest.raises(ValueError):
            ServeOptions(model_id="flux", **bad)
