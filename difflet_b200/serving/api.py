"""OpenAI-compatible HTTP API for image and video generation (FastAPI).

Routes as in the reference (``difflet/serving/openai/api_server.py:96-515``):
  GET  /health, /ready, /v1/models
  POST /v1/chat/completions   image models: the last user message is the prompt;
                              generation options in the body or ``extra_body``
                              (size, height, width, num_inference_steps, seed,
                              guidance_scale, negative_prompt, response_format);
                              the answer carries the PNG as a data URL
  POST /v1/images/generations image models: OpenAI Images API (b64_json)
  POST /v1/videos             video models: create an asynchronous job
  GET  /v1/videos/{id}        job status (queued / in_progress / completed / failed)
  GET  /v1/videos/{id}/content  the encoded video
  POST /v1/videos/sync        video models: generate in the request and answer with the
                              encoded video itself (``X-Request-Id``, ``X-Model``,
                              ``X-Inference-Time-S`` headers); a client that disconnects
                              cancels its generation (reference ``api_server.py:405-457``)
An API key (``--api-key`` or ``DIFFLET_API_KEY``) is enforced as a Bearer token
on every /v1 route.  A busy server answers 429.

Errors use the OpenAI envelope ``{"error": {"message", "type", "code"}}`` with a stable
``code`` per status (reference ``difflet/serving/errors.py:9-64``); chat-completion fields that
ask for something an image generator does not do (streaming, tools, n > 1, sampling
parameters) are refused with ``feature_not_supported``.
"""

from __future__ import annotations

import base64
import time
import uuid
from typing import Any

from fastapi import Body, FastAPI, HTTPException, Request
from fastapi.responses import FileResponse, JSONResponse

from difflet_b200.serving.engines import EngineError, QueueTimeout, RequestCancelled
from difflet_b200.serving.video_jobs import VideoJobStore

_GEN_KEYS = ("height", "width", "num_inference_steps", "seed", "guidance_scale", "guidance_scale_2",
             "true_cfg_scale", "negative_prompt", "num_frames")


# status -> (OpenAI error type, stable code)
_ERROR_CODES = {400: ("invalid_request_error", "invalid_request"), 401: ("invalid_request_error", "invalid_api_key"),
                404: ("invalid_request_error", "not_found"), 409: ("invalid_request_error", "conflict"),
                422: ("invalid_request_error", "invalid_request"), 429: ("server_error", "server_busy"),
                410: ("invalid_request_error", "gone"), 499: ("server_error", "request_cancelled"), 500: ("server_error", "internal_error"),
                503: ("server_error", "unavailable")}
# chat-completion fields an image generator cannot honour
_CHAT_UNSUPPORTED = ("stream", "tools", "tool_choice", "functions", "function_call", "temperature", "top_p", "stop",
                     "max_tokens", "logprobs")


class ServingError(HTTPException):
    """An HTTP error with an explicit machine-readable ``code`` (else derived from the status)."""

    def __init__(self, status_code: int, message: str, code: str | None = None):
        super().__init__(status_code, message)
        self.code = code


def error_payload(status: int, message: str, code: str | None = None) -> dict:
    etype, default = _ERROR_CODES.get(status, ("server_error" if status >= 500 else "invalid_request_error",
                                               "error"))
    return {"error": {"message": message, "type": etype, "code": code or default}}


MAX_PROMPT_CHARS = 10000


def _parse_size(size: str | None):
    if not size:
        return {}
    try:
        w, h = str(size).lower().split("x")
        return {"width": int(w), "height": int(h)}
    except ValueError:
        raise ServingError(400, f"size must be WIDTHxHEIGHT, got {size!r}", "invalid_request") from None


def _int_field(req, key, lo, hi, multiple=1):
    v = req.get(key)
    if v is None:
        return
    if isinstance(v, bool) or not isinstance(v, int) or not lo <= v <= hi or v % multiple:
        extra = f", a multiple of {multiple}" if multiple > 1 else ""
        raise ServingError(400, f"{key} must be an integer in [{lo}, {hi}]{extra}, got {v!r}", "invalid_request")


def check_request_fields(req: dict) -> None:
    """Types and ranges of the generation fields, checked before a request is queued (a bad value
    answers 400 instead of failing inside the engine)."""
    import math

    prompt = req.get("prompt")
    if not isinstance(prompt, str) or not prompt.strip():
        raise ServingError(400, "prompt must be a non-empty string", "invalid_prompt")
    if len(prompt) > MAX_PROMPT_CHARS:
        raise ServingError(400, f"prompt has {len(prompt)} characters (at most {MAX_PROMPT_CHARS})",
                           "prompt_too_long")
    neg = req.get("negative_prompt")
    if neg is not None and not isinstance(neg, str):
        raise ServingError(400, "negative_prompt must be a string", "invalid_prompt")
    _int_field(req, "height", 16, 8192, 16)
    _int_field(req, "width", 16, 8192, 16)
    _int_field(req, "num_inference_steps", 1, 1000)
    _int_field(req, "num_frames", 1, 1024)
    _int_field(req, "seed", 0, (1 << 63) - 1)
    for key in ("guidance_scale", "guidance_scale_2", "true_cfg_scale"):
        v = req.get(key)
        if v is None:
            continue
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v) or not 0 <= v <= 100:
            raise ServingError(400, f"{key} must be a number in [0, 100], got {v!r}", "invalid_request")


def normalize_chat_request(payload: dict) -> dict:
    if not isinstance(payload, dict):
        raise ServingError(400, "request body must be a JSON object", "invalid_request")
    for k in _CHAT_UNSUPPORTED:
        if payload.get(k) not in (None, False):
            raise ServingError(400, f"{k} is not supported by an image generation model", "feature_not_supported")
    if payload.get("n") not in (None, 1):
        raise ServingError(400, "one image per request (n = 1)", "feature_not_supported")
    msgs = payload.get("messages") or []
    if not isinstance(msgs, list) or not all(isinstance(m, dict) for m in msgs):
        raise ServingError(400, "messages must be a list of message objects", "invalid_request")
    if payload.get("extra_body") is not None and not isinstance(payload["extra_body"], dict):
        raise ServingError(400, "extra_body must be an object", "invalid_extra_body")
    prompt = None
    for m in reversed(msgs):
        if m.get("role") == "user":
            c = m.get("content")
            if isinstance(c, list):
                c = " ".join(p.get("text", "") for p in c if isinstance(p, dict) and p.get("type") == "text")
            prompt = c
            break
    if not prompt:
        raise ServingError(400, "no user message with text content", "invalid_prompt")
    opts = dict(payload.get("extra_body") or {})
    for k in _GEN_KEYS + ("size", "n"):
        if k in payload:
            opts.setdefault(k, payload[k])
    req = {"prompt": prompt}
    req.update(_parse_size(opts.pop("size", None)))
    for k in _GEN_KEYS:
        if k in opts and opts[k] is not None:
            req[k] = opts[k]
    return req


def create_app(engine, model_id: str, *, output: str = "image", api_key: str | None = None,
               request_timeout: float = 600.0, video_dir: str | None = None, encode_image=None,
               encode_video=None, artifact_store=None, video_limits: dict | None = None) -> FastAPI:
    from difflet_b200.utils.media import encode_mjpeg_avi, encode_png

    encode_image = encode_image or encode_png
    encode_video = encode_video or encode_mjpeg_avi
    app = FastAPI(title="difflet_b200", version="0.1.0")
    jobs = (VideoJobStore(engine, video_dir, encode_video, artifact_store=artifact_store, **(video_limits or {}))
            if output == "video" else None)

    from fastapi.exceptions import RequestValidationError

    @app.exception_handler(HTTPException)
    async def http_error(request: Request, exc: HTTPException):
        return JSONResponse(status_code=exc.status_code,
                            content=error_payload(exc.status_code, str(exc.detail), getattr(exc, "code", None)))

    @app.exception_handler(RequestValidationError)
    async def validation_error(request: Request, exc: RequestValidationError):
        return JSONResponse(status_code=400, content=error_payload(400, str(exc.errors())[:2000]))

    import hashlib
    import hmac

    key_digest = hashlib.sha256(api_key.encode()).digest() if api_key else None

    @app.middleware("http")
    async def auth(request: Request, call_next):
        """Bearer-token check on the versioned routes (health and readiness stay open for
        probes; CORS preflights pass).  The token is compared by digest in constant time."""
        path = request.url.path
        if key_digest is not None and request.method != "OPTIONS" and (path == "/v1" or path.startswith("/v1/")):
            scheme, _, token = request.headers.get("authorization", "").partition(" ")
            ok = scheme.lower() == "bearer" and hmac.compare_digest(
                hashlib.sha256(token.strip().encode()).digest(), key_digest)
            if not ok:
                return JSONResponse(status_code=401, content=error_payload(401, "invalid api key"))
        return await call_next(request)

    @app.get("/health")
    async def health():
        if not engine.healthy:
            return JSONResponse(status_code=503, content={"status": "unhealthy"})
        return {"status": "ok"}

    @app.get("/ready")
    async def ready():
        if not engine.ready:
            return JSONResponse(status_code=503, content={"status": "not_ready", "model": model_id})
        return {"status": "ready", "model": model_id}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_id, "object": "model", "owned_by": "difflet_b200",
                                            "output": output}]}

    from difflet_b200.models.spec import SpecRefusal, check_generate_kwargs, spec_for_model_id

    spec = spec_for_model_id(model_id)

    def _validate(req):
        """Bad values and options the model does not take answer 400 before the request is queued."""
        check_request_fields(req)
        if spec is None:
            return
        try:
            check_generate_kwargs(spec, req)
        except SpecRefusal as exc:
            raise ServingError(400, str(exc), "feature_not_supported")
        for field, why in spec.refused_video_fields:
            if req.get(field) is not None:
                raise ServingError(400, f"{field}: {why}", "feature_not_supported")

    def _run(req, request_id=None):
        _validate(req)
        try:
            if request_id is not None and hasattr(engine, "cancel"):
                return engine.generate(req, timeout=request_timeout, request_id=request_id)
            return engine.generate(req, timeout=request_timeout)
        except QueueTimeout:
            raise HTTPException(429, "server busy, retry later")
        except RequestCancelled as exc:
            raise HTTPException(499, str(exc))
        except EngineError as exc:
            # the engine's message can hold paths and tracebacks: logged here, not sent to clients
            import logging

            logging.getLogger("difflet_b200.serving.api").error("request %s failed: %s", request_id, str(exc)[-4000:])
            raise ServingError(500, "internal model execution error"
                               + (f" (request {request_id})" if request_id else ""), "internal_error")

    @app.post("/v1/requests/{rid}/cancel")
    async def cancel_request(rid: str):
        """Cancel a running request started with an ``X-Request-Id`` header (or a video job id)."""
        if jobs is not None and jobs.get(rid) is not None:
            return jobs.cancel(rid).public()
        ok = bool(hasattr(engine, "cancel") and engine.cancel(rid))
        if not ok:
            raise HTTPException(404, "no running request with that id")
        return {"id": rid, "status": "cancelling"}

    if output == "image":
        import asyncio

        @app.post("/v1/chat/completions")
        async def chat(request: Request, payload: Any = Body(default=None)):
            req = normalize_chat_request(payload)
            t0 = time.perf_counter()
            rid = request.headers.get("x-request-id")
            img = await asyncio.get_running_loop().run_in_executor(None, _run, req, rid)
            png = encode_image(img) if not isinstance(img, (bytes, bytearray)) else bytes(img)
            url = "data:image/png;base64," + base64.b64encode(png).decode()
            return {"id": "chatcmpl-" + uuid.uuid4().hex, "object": "chat.completion", "created": int(time.time()),
                    "model": model_id,
                    "choices": [{"index": 0, "finish_reason": "stop",
                                 "message": {"role": "assistant", "content": [{"type": "image_url",
                                                                               "image_url": {"url": url}}]}}],
                    "usage": {"generation_seconds": round(time.perf_counter() - t0, 3)}}

        @app.post("/v1/images/generations")
        async def images(request: Request, payload: Any = Body(default=None)):
            if not isinstance(payload, dict) or not payload.get("prompt"):
                raise ServingError(400, "prompt is required", "invalid_prompt")
            req = {"prompt": payload["prompt"], **_parse_size(payload.get("size"))}
            for k in _GEN_KEYS:
                if k in payload:
                    req[k] = payload[k]
            img = await asyncio.get_running_loop().run_in_executor(None, _run, req, request.headers.get("x-request-id"))
            png = encode_image(img) if not isinstance(img, (bytes, bytearray)) else bytes(img)
            return {"created": int(time.time()), "data": [{"b64_json": base64.b64encode(png).decode()}]}

    else:
        import asyncio

        def _video_request(payload) -> dict:
            if not isinstance(payload, dict) or not payload.get("prompt"):
                raise ServingError(400, "prompt is required", "invalid_prompt")
            req = {"prompt": payload["prompt"], **_parse_size(payload.get("size"))}
            for k in _GEN_KEYS:
                if k in payload:
                    req[k] = payload[k]
            if "seconds" in payload and "num_frames" not in req:
                sec = payload["seconds"]
                try:
                    sec = float(sec)
                except (TypeError, ValueError):
                    raise ServingError(400, f"seconds must be a number, got {sec!r}", "invalid_request") from None
                if not 0 < sec <= 60:
                    raise ServingError(400, f"seconds must be in (0, 60], got {sec}", "invalid_request")
                req["num_frames"] = int(sec * 16) // 4 * 4 + 1
            _validate(req)
            return req

        @app.post("/v1/videos")
        async def create_video(payload: Any = Body(default=None)):
            from difflet_b200.serving.video_jobs import JobAdmissionError

            try:
                job = jobs.create(_video_request(payload))
            except JobAdmissionError as exc:
                raise ServingError(429, str(exc), "server_busy")
            return job.public()

        @app.post("/v1/videos/sync")
        async def create_video_sync(request: Request, payload: Any = Body(default=None)):
            """Generate while the client waits and answer with the encoded video.  The generation
            runs on a worker thread; the connection is polled meanwhile, and a client that goes
            away cancels its request (the engine stops between denoise steps)."""
            from fastapi.responses import Response

            req = _video_request(payload)
            rid = request.headers.get("x-request-id") or f"video_sync_{uuid.uuid4().hex}"
            loop = asyncio.get_running_loop()
            t0 = time.perf_counter()
            fut = loop.run_in_executor(None, _run, req, rid)
            while True:
                done, _ = await asyncio.wait({fut}, timeout=0.25)
                if done:
                    break
                if await request.is_disconnected():
                    if hasattr(engine, "cancel"):
                        engine.cancel(rid)
                    try:
                        await fut
                    except Exception:  # noqa: BLE001 - the client is gone; nothing to answer
                        pass
                    return Response(status_code=499)
            frames = fut.result()  # HTTP errors of the engine propagate from here
            infer_s = time.perf_counter() - t0
            data = frames if isinstance(frames, (bytes, bytearray)) else encode_video(frames, jobs.fps)
            return Response(content=bytes(data), media_type="video/x-msvideo",
                            headers={"X-Request-Id": rid, "X-Model": model_id,
                                     "X-Inference-Time-S": f"{infer_s:.6f}"})

        @app.get("/v1/videos/{vid}")
        async def get_video(vid: str):
            job = jobs.get(vid)
            if job is None:
                raise HTTPException(404, "no such video")
            return job.public()

        @app.get("/v1/videos")
        async def list_videos(after: str | None = None, limit: int = 20):
            page = jobs.repo.list(after=after, limit=max(1, min(100, limit)))
            return {"object": "list", "data": [j.public() for j in page],
                    "has_more": len(jobs.repo.list(after=page[-1].id, limit=1)) > 0 if page else False}

        @app.get("/v1/videos/{vid}/content")
        async def video_content(vid: str):
            job = jobs.get(vid)
            if job is None:
                raise HTTPException(404, "no such video")
            if job.status != "completed":
                raise HTTPException(409, f"video is {job.status}")
            if job.url and not job.url.startswith("file://"):
                from fastapi.responses import RedirectResponse

                return RedirectResponse(job.url, status_code=307)
            import os

            if not job.path or not os.path.isfile(job.path):
                raise ServingError(410, "the video file is no longer available", "gone")
            return FileResponse(job.path, media_type="video/x-msvideo")

        @app.post("/v1/videos/{vid}/cancel")
        async def cancel_video(vid: str):
            if jobs.get(vid) is None:
                raise HTTPException(404, "no such video")
            return jobs.cancel(vid).public()

        @app.delete("/v1/videos/{vid}")
        async def delete_video(vid: str):
            """Delete a finished job's record (a queued or running one is cancelled first)."""
            from difflet_b200.serving.video_jobs import TERMINAL

            job = jobs.get(vid)
            if job is None:
                raise HTTPException(404, "no such video")
            if job.status not in TERMINAL:
                job = jobs.cancel(vid)
                if job.status not in TERMINAL:
                    return {"id": vid, "object": "video.deleted", "deleted": False, "status": job.status}
            from difflet_b200.serving.video_jobs import VideoJobNotFound

            try:
                jobs.delete(vid)
            except VideoJobNotFound:  # deleted meanwhile (the retention sweep or another client)
                raise HTTPException(404, "no such video")
            return {"id": vid, "object": "video.deleted", "deleted": True}

    app.state.jobs = jobs
    return app
