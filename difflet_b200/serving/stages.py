"""Typed stage pipeline of one serving request, with per-request stage events.

Reference behaviour (``difflet/serving/engines/stage_pipeline.py:38-311``): a request runs through
an ordered list of stages; each stage declares the exact payload type it takes and returns and the
executor refuses anything else; cancellation is checked before and after every stage; the worker's
heartbeat reports the running stage; every stage start / completion is logged with the request id
and its duration; the last stage is the only one marked final; shutdown runs every stage's cleanup
in reverse order and reports all failures together.

Here a stage is a plain callable on a dataclass payload, run in the rank process that owns the
GPU(s) of the replica.  ``pipeline_stages`` splits a loaded ``DiffletPipeline`` into
prepare -> denoise -> decode -> output where the application exposes those phases (Wan: ``prepare``,
``WanRun.step``, ``decode``), and into generate -> output otherwise; the denoise loop polls the
cancellation between steps, so a multi-GPU replica stops at the same step on every rank.
"""

from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field
from typing import Any, Callable

logger = logging.getLogger("difflet_b200.serving.engine")


class StagePayloadTypeError(TypeError):
    """A stage got or returned a payload other than the exact type it declares."""


class StageShutdownError(RuntimeError):
    def __init__(self, errors: list[BaseException]):
        self.errors = tuple(errors)
        super().__init__(f"{len(errors)} stage cleanup(s) failed: " + "; ".join(repr(e) for e in errors))


# ------------------------------------------------------------------ payloads
@dataclass
class StagePayload:
    pass


@dataclass
class RequestPayload(StagePayload):
    request: dict


@dataclass
class PreparedPayload(StagePayload):
    request: dict
    run: Any  # the application's per-generation state (e.g. ``WanRun``)


@dataclass
class LatentPayload(StagePayload):
    request: dict
    latents: Any


@dataclass
class DecodedPayload(StagePayload):
    request: dict
    output: Any  # pixels on the device (None on ranks that do not hold the result)


@dataclass
class OutputPayload(StagePayload):
    output: Any  # what the engine returns to the caller (host tensor or None)


# ------------------------------------------------------------------ stages
@dataclass(frozen=True)
class Stage:
    stage_id: str
    input_type: type
    output_type: type
    fn: Callable[[StagePayload, "StageContext"], StagePayload]
    final: bool = False
    cleanup: Callable[[], None] | None = None


@dataclass
class StageEvent:
    request_id: str
    stage: str
    kind: str  # start | complete | error | cancelled
    t: float   # time.monotonic()
    duration: float | None = None
    detail: str = ""


@dataclass
class StageContext:
    request_id: str
    should_cancel: Callable[[], bool] = lambda: False
    on_stage: Callable[[str], None] | None = None  # heartbeat: the running stage
    events: list = field(default_factory=list)

    def check_cancel(self, where: str = "") -> None:
        if self.should_cancel():
            from difflet_b200.serving.engines import RequestCancelled

            raise RequestCancelled(f"cancelled {where}".strip())


def _exact(value, typ, what) -> None:
    if type(value) is not typ:
        raise StagePayloadTypeError(f"{what} must be exactly {typ.__name__}, got {type(value).__name__}")


class StagePipeline:
    """An ordered, type-checked list of stages (checked once, at construction)."""

    def __init__(self, stages: list[Stage], *, reset: Callable[[str], None] | None = None):
        if not stages:
            raise StagePayloadTypeError("a pipeline needs at least one stage")
        ids = [s.stage_id for s in stages]
        if len(set(ids)) != len(ids):
            raise StagePayloadTypeError(f"stage ids must be unique: {ids}")
        finals = [i for i, s in enumerate(stages) if s.final]
        if finals != [len(stages) - 1]:
            raise StagePayloadTypeError("exactly one final stage, and it must be the last")
        for a, b in zip(stages, stages[1:]):
            if a.output_type is not b.input_type:
                raise StagePayloadTypeError(f"stage {a.stage_id!r} returns {a.output_type.__name__} but "
                                            f"{b.stage_id!r} takes {b.input_type.__name__}")
        if stages[0].input_type is not RequestPayload:
            raise StagePayloadTypeError("the first stage must take RequestPayload")
        self.stages = list(stages)
        self.reset = reset
        self._closed = False

    @property
    def stage_ids(self) -> tuple[str, ...]:
        return tuple(s.stage_id for s in self.stages)

    def _event(self, ctx: StageContext, stage: str, kind: str, t0: float | None = None, detail: str = "") -> None:
        now = time.monotonic()
        ev = StageEvent(ctx.request_id, stage, kind, now, None if t0 is None else now - t0, detail)
        ctx.events.append(ev)
        if kind == "start":
            logger.info("stage.start request_id=%s stage=%s", ctx.request_id, stage)
        else:
            logger.info("stage.%s request_id=%s stage=%s duration=%.3f%s", kind, ctx.request_id, stage,
                        ev.duration or 0.0, f" detail={detail}" if detail else "")

    def run(self, request: dict, ctx: StageContext) -> Any:
        if self._closed:
            raise RuntimeError("stage pipeline is shut down")
        if self.reset is not None:
            self.reset("before_request")
        payload: StagePayload = RequestPayload(dict(request))
        try:
            for st in self.stages:
                ctx.check_cancel(f"before stage {st.stage_id}")
                _exact(payload, st.input_type, f"input of stage {st.stage_id!r}")
                if ctx.on_stage is not None:
                    ctx.on_stage(st.stage_id)
                t0 = time.monotonic()
                self._event(ctx, st.stage_id, "start")
                try:
                    out = st.fn(payload, ctx)
                except BaseException as exc:
                    kind = "cancelled" if type(exc).__name__ == "RequestCancelled" else "error"
                    self._event(ctx, st.stage_id, kind, t0, detail=type(exc).__name__)
                    raise
                _exact(out, st.output_type, f"output of stage {st.stage_id!r}")
                self._event(ctx, st.stage_id, "complete", t0)
                payload = out
                if not st.final:
                    ctx.check_cancel(f"after stage {st.stage_id}")
            if self.reset is not None:
                self.reset("completed")
            return payload.output
        except BaseException:
            if self.reset is not None:
                self.reset("error")
            raise

    def shutdown(self) -> None:
        if self._closed:
            return
        self._closed = True
        errors = []
        for st in reversed(self.stages):
            if st.cleanup is None:
                continue
            try:
                st.cleanup()
            except BaseException as exc:  # noqa: BLE001 - collected and raised together
                errors.append(exc)
        if errors:
            raise StageShutdownError(errors)


# ------------------------------------------------------------------ stages of a DiffletPipeline
def _to_host(p: DecodedPayload, ctx: StageContext) -> OutputPayload:
    """The request's result on the host: the first item of the batch (the serving API answers
    one image / video per request)."""
    out = p.output
    if out is None:
        return OutputPayload(None)
    out = out[0]
    return OutputPayload(out.cpu() if hasattr(out, "cpu") else out)


def _phase_app(pipe):
    """The application object with prepare / decode phases, or None."""
    app = getattr(getattr(pipe, "app", None), "app", None)
    if app is not None and all(hasattr(app, n) for n in ("prepare", "decode")):
        return app
    return None


def pipeline_stages(pipe) -> StagePipeline:
    app = _phase_app(pipe)
    if app is None:
        def generate(p: RequestPayload, ctx: StageContext) -> DecodedPayload:
            req = dict(p.request)
            user_cb = req.pop("callback", None)

            def callback(i, latents):
                ctx.check_cancel(f"at step {i}")
                if user_cb is not None:
                    user_cb(i, latents)

            req["callback"] = callback
            return DecodedPayload(p.request, pipe(**req))

        return StagePipeline([Stage("generate", RequestPayload, DecodedPayload, generate),
                              Stage("output", DecodedPayload, OutputPayload, _to_host, final=True)])

    import inspect

    prep_args = set(inspect.signature(app.prepare).parameters)

    def prepare(p: RequestPayload, ctx: StageContext) -> PreparedPayload:
        req = dict(p.request)
        if isinstance(req.get("prompt"), str) and "prompt" not in prep_args:
            raise StagePayloadTypeError("the application takes no prompt")
        kw = {k: v for k, v in req.items() if k in prep_args}
        return PreparedPayload(req, app.prepare(**kw))

    def denoise(p: PreparedPayload, ctx: StageContext) -> LatentPayload:
        import torch

        run = p.run
        user_cb = p.request.get("callback")
        with torch.no_grad():
            for i in range(run.steps):
                ctx.check_cancel(f"at step {i}")
                run.step(i)
                if user_cb is not None:
                    user_cb(i, run.x32)
            return LatentPayload(p.request, run.latents())

    def decode(p: LatentPayload, ctx: StageContext) -> DecodedPayload:
        import torch

        kind = p.request.get("output_type", "uint8")
        if kind == "latent":
            return DecodedPayload(p.request, p.latents)
        with torch.no_grad():
            video = app.decode(p.latents)
        if video is None or kind == "float":
            return DecodedPayload(p.request, video)
        return DecodedPayload(p.request, ((video.float() * 0.5 + 0.5).clamp(0, 1) * 255).round()
                              .to(torch.uint8).permute(0, 2, 3, 4, 1))

    return StagePipeline([Stage("prepare", RequestPayload, PreparedPayload, prepare),
                          Stage("denoise", PreparedPayload, LatentPayload, denoise),
                          Stage("decode", LatentPayload, DecodedPayload, decode),
                          Stage("output", DecodedPayload, OutputPayload, _to_host, final=True)])


__all__ = ["DecodedPayload", "LatentPayload", "OutputPayload", "PreparedPayload", "RequestPayload", "Stage",
           "StageContext", "StageEvent", "StagePayload", "StagePayloadTypeError", "StagePipeline",
           "StageShutdownError", "pipeline_stages"]
