"""``difflet serve``: build the engine stack and run the HTTP server (uvicorn).

Reference: ``difflet/cli/serve.py:153-216`` and ``difflet/serving/factory.py:39-106``.
The worker factory builds ``DiffletPipeline.from_pretrained(...)`` inside the
resident worker process and returns a ``run(request)`` that produces uint8
images / frames (moved to the host) for the API layer to encode.
"""

from __future__ import annotations

import logging


def pipeline_runner(model_id: str, pipeline_kwargs: dict):
    """Runs inside every rank process of a replica: load once, return run(request, ...).

    A request runs through the pipeline's stages (``serving/stages.py``: prepare -> denoise ->
    decode -> output, or generate -> output), each logged with its duration; ``on_stage`` feeds
    the worker's heartbeat.  ``should_cancel()`` is polled between denoise steps (every rank of a
    multi-GPU replica polls at the same step and gets the same answer); a cancelled request
    raises RequestCancelled."""
    from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline
    from difflet_b200.serving.stages import StageContext, pipeline_stages

    pipe = DiffletPipeline.from_pretrained(model_id, **pipeline_kwargs)
    video = pipe.model_entry.output == "video"
    stages = pipeline_stages(pipe)

    def run(req: dict, should_cancel=None, on_stage=None, request_id=None):
        smoke = bool(req.get("__smoke__"))
        if smoke:
            req = {"prompt": "smoke", "num_inference_steps": 2, "height": 256, "width": 256}
            if video:
                req["num_frames"] = 5
        ctx = StageContext(request_id or ("smoke" if smoke else "-"), should_cancel or (lambda: False), on_stage)
        out = stages.run(req, ctx)
        return None if smoke else out

    run.stages = stages
    return run


def replica_devices(replicas: int, model_world: int, visible: list | None = None) -> list[list[int]]:
    """GPU indices of each replica: consecutive slices of ``model_world`` GPUs (replica i of a
    dp group never shares a GPU with another replica)."""
    import torch

    gpus = visible if visible is not None else list(range(torch.cuda.device_count()))
    need = replicas * model_world
    if gpus and len(gpus) < need:
        raise ValueError(f"{replicas} replicas x {model_world} GPUs each need {need} GPUs, {len(gpus)} visible")
    if not gpus:
        return [[] for _ in range(replicas)]
    return [gpus[i * model_world:(i + 1) * model_world] for i in range(replicas)]


def serve_main(a) -> int:
    import uvicorn

    from difflet_b200.cli.main import _app_kwargs, parallel_from_args
    from difflet_b200.registry import resolve_model
    from difflet_b200.serving.api import create_app
    from difflet_b200.serving.engines import ReplicatedEngine, ResidentWorkerEngine

    from difflet_b200.serving.logs import configure_serve_logging

    log_file = configure_serve_logging(getattr(a, "log_dir", None))
    logging.getLogger(__name__).info("serve log: %s", log_file.path)
    entry = resolve_model(a.model_id)
    kw = {"parallel": parallel_from_args(a), "backend": a.backend, "height": a.height, "width": a.width,
          "num_frames": a.num_frames, "compile_cache_dir": a.cache_dir, "random_init": a.random_weights,
          "application_kwargs": _app_kwargs(a)}
    from difflet_b200.serving.options import ServeOptions

    opts = ServeOptions.from_args(a)
    world = kw["parallel"].model_world_size
    import os

    visible = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip().isdigit()] or None
    devices = replica_devices(opts.replicas, world, visible) if a.backend != "cpu" else [None] * opts.replicas
    replicas = [ResidentWorkerEngine(pipeline_runner, {"model_id": a.model_id, "pipeline_kwargs": kw},
                                     devices=dev or None, world=world, **opts.engine_kwargs())
                for dev in devices]
    engine = replicas[0] if len(replicas) == 1 else ReplicatedEngine(replicas)
    from difflet_b200.serving.artifacts import make_artifact_store

    store = make_artifact_store() if entry.output == "video" and any(k.startswith("DIFFLET_S3_") for k in os.environ) \
        else None
    app = create_app(engine, a.model_id, output=entry.output, api_key=opts.api_key, artifact_store=store,
                     video_limits={"max_queued": opts.max_queued_requests, "request_timeout_s": opts.request_timeout,
                                   "retention_s": 3600.0 * getattr(a, "video_retention_hours", 25.0),
                                   "max_jobs": getattr(a, "max_video_jobs", 4096)})
    uvicorn.run(app, host=opts.host, port=opts.port, log_level="info", log_config=None)
    engine.close()
    return 0
