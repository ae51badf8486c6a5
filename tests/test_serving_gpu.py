"""A serving request end to end on a B200: the resident runner's stage pipeline around a real
(random-init) FLUX.1-dev engine, as ``difflet serve`` runs it in its worker process."""

import pytest
import torch


@pytest.mark.gpu
def test_pipeline_runner_serves_an_image_gpu(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
    from difflet_b200.serving.server import pipeline_runner
    from difflet_b200.utils.media import encode_png

    run = pipeline_runner("black-forest-labs/FLUX.1-dev", {
        "parallel": DiffletParallelConfig(), "backend": "cuda", "height": 256, "width": 256,
        "random_init": True, "compile_cache_dir": str(tmp_path)})
    assert run({"__smoke__": True}) is None
    stages = []
    out = run({"prompt": "a red fox in the snow", "num_inference_steps": 2, "height": 256, "width": 256},
              on_stage=stages.append, request_id="req-1")
    assert stages == list(run.stages.stage_ids)
    assert out.device.type == "cpu" and out.dtype == torch.uint8 and tuple(out.shape) == (256, 256, 3)
    assert encode_png(out.numpy())[:8] == b"\x89PNG\r\n\x1a\n"
    cancelled = iter([False, True])
    from difflet_b200.serving.engines import RequestCancelled

    with pytest.raises(RequestCancelled):  # cancelled at the first denoise step
        run({"prompt": "x", "num_inference_steps": 4, "height": 256, "width": 256},
            should_cancel=lambda: next(cancelled, True))
