"""Run telemetry through the public pipeline API: JSONL timing events (reference schema),
per-step times, latent dumps; and the event writer never failing a run."""

import json

import torch

from difflet_b200 import DiffletPipeline
from difflet_b200.utils import telemetry


def test_pipeline_telemetry(tmp_path, monkeypatch):
    monkeypatch.setenv("DIFFLET_BACKEND", "cpu")
    monkeypatch.setenv("DIFFLET_BENCH_TIMING_DIR", str(tmp_path / "timing"))
    monkeypatch.setenv("DIFFLET_STEP_TIMES_FILE", str(tmp_path / "steps.jsonl"))
    monkeypatch.setenv("DIFFLET_DUMP_LATENTS_DIR", str(tmp_path / "latents"))
    pipe = DiffletPipeline.from_pretrained("black-forest-labs/FLUX.1-dev", random_init=True,
                                           compile_cache_dir=str(tmp_path / "cache"), dtype=torch.float32,
                                           application_kwargs={"preset": "tiny128"})
    seen = []
    out = pipe(prompt="a photo", output_type="latent", height=64, width=64, num_inference_steps=3,
               callback=lambda i, x: seen.append(i))
    assert torch.isfinite(out).all() and seen == [0, 1, 2]  # the user's callback still runs
    files = list((tmp_path / "timing").glob("*.jsonl"))
    assert len(files) == 1
    ev = [json.loads(line) for line in files[0].read_text().splitlines()]
    kinds = [e["event"] for e in ev]
    assert kinds[0] == "process" and kinds.count("step") == 3 and "evidence" in kinds
    spans = [e for e in ev if e["event"] == "span" and e["name"] == "request"]
    assert [s["phase"] for s in spans] == ["begin", "end"] and spans[1]["ok"] is True
    assert all({"t_ns", "pid", "rank", "world"} <= set(e) for e in ev)
    assert [e["index"] for e in ev if e["event"] == "step"] == [0, 1, 2]
    steps = [json.loads(line) for line in (tmp_path / "steps.jsonl").read_text().splitlines()]
    assert [s["step"] for s in steps] == [0, 1, 2] and all(s["ms"] >= 0 for s in steps)
    dumps = sorted((tmp_path / "latents").rglob("step_*.pt"))
    assert len(dumps) == 3 and all(torch.isfinite(torch.load(d)).all() for d in dumps)


def test_event_writer_never_fails(tmp_path, monkeypatch):
    blocker = tmp_path / "file"
    blocker.write_text("x")
    monkeypatch.setenv("DIFFLET_BENCH_TIMING_DIR", str(blocker / "sub"))  # cannot be created
    monkeypatch.setattr(telemetry, "_SINK", telemetry._Sink())
    telemetry.event("args", a=1)  # swallowed, then disabled
    assert telemetry._SINK.dead
    with telemetry.span("x"):
        pass
