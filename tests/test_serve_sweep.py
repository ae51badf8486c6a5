"""The serve throughput sweep against a live HTTP server (uvicorn in a thread, CPU engine)."""

import threading
import time

import torch


def test_sweep_counts_completions_and_refusals():
    import uvicorn

    from difflet_b200.bench.serve_sweep import sweep, wait_ready
    from difflet_b200.parallel.testing import free_port
    from difflet_b200.serving.api import create_app
    from difflet_b200.serving.engines import InProcessEngine

    def gen(req):
        time.sleep(0.05)
        return torch.zeros(8, 8, 3, dtype=torch.uint8)

    # one request at a time, at most one waiting for at most 0.5 s: a burst of 8 gets refusals
    eng = InProcessEngine(gen, queue_timeout=0.5, max_queued=1)
    app = create_app(eng, "flux")
    port = free_port()
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    try:
        url = f"http://127.0.0.1:{port}"
        assert wait_ready(url, 30)
        rows = sweep(url, levels=(1, 8), rounds=2, payload={"prompt": "x", "size": "16x16"}, timeout=30)
    finally:
        server.should_exit = True
        th.join(timeout=10)
    one, eight = rows
    assert one["concurrency"] == 1 and one["requests"] == 2 and one["completed"] == 2 and one["failed"] == 0
    assert one["requests_per_s"] > 0 and one["latency_p50_s"] >= 0.05
    assert eight["requests"] == 16
    assert eight["completed"] + eight["refused_429"] == 16 and eight["refused_429"] > 0
