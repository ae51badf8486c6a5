"""Stage pipeline of a serving request and the serve log files (CPU)."""

import logging
from datetime import datetime, timedelta
from types import SimpleNamespace

import pytest
import torch

from difflet_b200.serving.engines import RequestCancelled
from difflet_b200.serving.logs import ServeLogHandler
from difflet_b200.serving.stages import (DecodedPayload, OutputPayload, RequestPayload, Stage, StageContext,
                                         StagePayloadTypeError, StagePipeline, StageShutdownError,
                                         pipeline_stages)


def _two_stage(fn_gen=None):
    gen = fn_gen or (lambda p, ctx: DecodedPayload(p.request, torch.ones(2)))
    return StagePipeline([Stage("generate", RequestPayload, DecodedPayload, gen),
                          Stage("output", DecodedPayload, OutputPayload, lambda p, c: OutputPayload(p.output),
                                final=True)])


def test_pipeline_checks_its_definition():
    out = Stage("output", DecodedPayload, OutputPayload, lambda p, c: OutputPayload(None), final=True)
    with pytest.raises(StagePayloadTypeError):  # the chain of types is broken
        StagePipeline([Stage("a", RequestPayload, RequestPayload, lambda p, c: p), out])
    with pytest.raises(StagePayloadTypeError):  # final stage not last
        StagePipeline([Stage("a", RequestPayload, DecodedPayload, lambda p, c: p, final=True), out])
    with pytest.raises(StagePayloadTypeError):  # duplicate ids
        StagePipeline([Stage("output", RequestPayload, DecodedPayload, lambda p, c: p), out])


def test_run_records_events_and_reports_stages():
    seen = []
    pipe = _two_stage()
    ctx = StageContext("rid-1", on_stage=seen.append)
    out = pipe.run({"prompt": "x"}, ctx)
    assert torch.equal(out, torch.ones(2))  # _two_stage's own output stage passes it through
    assert seen == ["generate", "output"]
    kinds = [(e.stage, e.kind) for e in ctx.events]
    assert kinds == [("generate", "start"), ("generate", "complete"), ("output", "start"), ("output", "complete")]
    assert all(e.request_id == "rid-1" for e in ctx.events)
    assert all(e.duration is not None and e.duration >= 0 for e in ctx.events if e.kind == "complete")


def test_wrong_payload_type_is_refused():
    pipe = _two_stage(lambda p, ctx: OutputPayload(None))
    with pytest.raises(StagePayloadTypeError):
        pipe.run({}, StageContext("r"))


def test_cancel_before_and_during_stages():
    calls = []
    pipe = _two_stage(lambda p, ctx: calls.append(1) or DecodedPayload(p.request, None))
    with pytest.raises(RequestCancelled):
        pipe.run({}, StageContext("r", should_cancel=lambda: True))
    assert calls == []  # never started

    state = {"n": 0}

    def should_cancel():
        state["n"] += 1
        return state["n"] > 1  # passes the check before the first stage only

    ctx = StageContext("r", should_cancel=should_cancel)
    with pytest.raises(RequestCancelled):
        pipe.run({}, ctx)
    assert calls == [1] and ctx.events[-1].kind == "complete"  # stopped after the generate stage


def test_shutdown_runs_every_cleanup_and_raises_together():
    order = []

    def bad():
        order.append("b")
        raise RuntimeError("b failed")

    pipe = StagePipeline([
        Stage("a", RequestPayload, DecodedPayload, lambda p, c: DecodedPayload({}, None), cleanup=lambda: order.append("a")),
        Stage("b", DecodedPayload, OutputPayload, lambda p, c: OutputPayload(None), final=True, cleanup=bad)])
    with pytest.raises(StageShutdownError) as ei:
        pipe.shutdown()
    assert order == ["b", "a"] and len(ei.value.errors) == 1
    with pytest.raises(RuntimeError):
        pipe.run({}, StageContext("r"))


class _FakeRun:
    def __init__(self, steps):
        self.steps = steps
        self.x32 = torch.zeros(3)
        self.done = []

    def step(self, i):
        self.done.append(i)
        self.x32 += 1

    def latents(self):
        return self.x32.clone()


class _FakeApp:
    def __init__(self):
        self.runs = []

    def prepare(self, *, prompt=None, num_inference_steps=4, height=64, width=64):
        r = _FakeRun(num_inference_steps)
        self.runs.append(r)
        return r

    def decode(self, lat):
        return lat.view(1, 3, 1, 1, 1).expand(1, 3, 2, 2, 2) * 0.0


def test_phase_pipeline_of_an_application():
    app = _FakeApp()
    pipe = SimpleNamespace(app=SimpleNamespace(app=app))
    stages = pipeline_stages(pipe)
    assert stages.stage_ids == ("prepare", "denoise", "decode", "output")
    ctx = StageContext("r")
    video = stages.run({"prompt": "p", "num_inference_steps": 3, "unused": 1}, ctx)
    assert app.runs[0].done == [0, 1, 2]
    assert video.dtype == torch.uint8 and video.shape == (2, 2, 2, 3)  # the first video of the batch
    assert (video == 128).all()  # 0 in [-1, 1] -> 127.5 -> 128
    lat = stages.run({"prompt": "p", "num_inference_steps": 2, "output_type": "latent"}, StageContext("r2"))
    assert torch.equal(lat, torch.tensor(2.0))  # first element of the latent batch
    # cancellation polled between denoise steps
    n = {"k": 0}

    def cancel_at_step_2():
        n["k"] += 1
        return len(app.runs[-1].done) >= 2 if n["k"] > 2 else False

    with pytest.raises(RequestCancelled):
        stages.run({"prompt": "p", "num_inference_steps": 5}, StageContext("r3", should_cancel=cancel_at_step_2))
    assert app.runs[-1].done == [0, 1]


def test_generic_pipeline_wraps_the_call():
    seen = {}

    def call(**kw):
        seen.update(kw)
        kw["callback"](0, None)
        return torch.ones(1, 2)  # a batch of one

    stages = pipeline_stages(call)
    assert stages.stage_ids == ("generate", "output")
    out = stages.run({"prompt": "p"}, StageContext("r"))
    assert torch.equal(out, torch.ones(2)) and seen["prompt"] == "p"
    answers = iter([False, True])  # the check before the stage passes; the step callback cancels
    with pytest.raises(RequestCancelled):
        stages.run({"prompt": "p"}, StageContext("r", should_cancel=lambda: next(answers)))


def _record(msg):
    return logging.LogRecord("t", logging.INFO, __file__, 1, msg, None, None)


def test_serve_log_files_roll_by_size_and_day(tmp_path):
    now = {"t": datetime(2026, 3, 1, 23, 59, 58)}
    h = ServeLogHandler(tmp_path, project="proj", max_bytes=200, keep=3, clock=lambda: now["t"])
    first = h.path
    assert first.name.startswith("proj-20260301_235958")
    for i in range(3):
        h.emit(_record("x" * 60 + str(i)))
    assert h.path != first  # the third record would pass 200 bytes
    now["t"] += timedelta(seconds=3)  # next day
    h.emit(_record("after midnight"))
    assert "20260302_000001" in h.path.name
    for i in range(6):
        now["t"] += timedelta(seconds=1)
        h.emit(_record("y" * 150))
    h.close()
    files = sorted(tmp_path.glob("proj-*.log"))
    assert len(files) == 3  # oldest pruned
    assert all(f.stat().st_size <= 200 for f in files)
