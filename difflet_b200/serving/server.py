"""``difflet serve``: build the engine stack and run the HTTP server (uvicorn).

Reference: ``difflet/cli/serve.py:153-216`` and ``difflet/serving/factory.py:39-106``.
The worker factory builds ``DiffletPipeline.from_pretrained(...)`` inside the
resident worker process and returns a ``run(request)`` that produces uint8
images / frames (moved to the host) for the API layer to encode.
"""

from __future__ import annotations

import logging


def pipeline_runner(model_id: str, pipeline_kwargs: dict):
    """Runs inside the worker process: load once, return run(request)."""
    from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline

    pipe = DiffletPipeline.from_pretrained(model_id, **pipeline_kwargs)
    video = pipe.model_entry.output == "video"

    def run(req: dict):
        if req.get("__smoke__"):
            kw = {"prompt": "smoke", "num_inference_steps": 2}
            if video:
                kw["num_frames"] = 5
            kw["height"], kw["width"] = 256, 256
            pipe(**kw)
            return None
        out = pipe(**req)
        if out is None:
            return None
        return out[0].cpu()

    return run


def serve_main(a) -> int:
    import uvicorn

    from difflet_b200.cli.main import _app_kwargs, parallel_from_args
    from difflet_b200.registry import resolve_model
    from difflet_b200.serving.api import create_app
    from difflet_b200.serving.engines import ReplicatedEngine, ResidentWorkerEngine

    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
    entry = resolve_model(a.model_id)
    kw = {"parallel": parallel_from_args(a), "backend": a.backend, "height": a.height, "width": a.width,
          "num_frames": a.num_frames, "compile_cache_dir": a.cache_dir, "random_init": a.random_weights,
          "application_kwargs": _app_kwargs(a)}
    from difflet_b200.serving.options import ServeOptions

    opts = ServeOptions.from_args(a)
    replicas = [ResidentWorkerEngine(pipeline_runner, {"model_id": a.model_id, "pipeline_kwargs": kw},
                                     **opts.engine_kwargs())
                for _ in range(opts.replicas)]
    engine = replicas[0] if len(replicas) == 1 else ReplicatedEngine(replicas)
    app = create_app(engine, a.model_id, output=entry.output, api_key=opts.api_key)
    uvicorn.run(app, host=opts.host, port=opts.port, log_level="info")
    engine.close()
    return 0
