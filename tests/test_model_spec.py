"""Model specs as data: lookup, CLI / request refusals, prompt budgets, serving 400s."""

import argparse

import pytest
import torch
from fastapi.testclient import TestClient

from difflet_b200.models import spec as S
from difflet_b200.registry import registered_models
from difflet_b200.serving.api import create_app
from difflet_b200.serving.engines import InProcessEngine


def test_every_spec_matches_its_registry_entry():
    for name, sp in S.SPECS.items():
        assert sp.model_type == name
        entry = registered_models()[name]
        assert entry.output == sp.output
        for mid in sp.cli_model_ids:
            assert entry.matches(mid)
            assert S.spec_for_model_id(mid) is sp
        assert entry.default_shape.get("num_frames") == sp.default_num_frames
        assert sp.accepts_cfg_parallel == (entry.capabilities.supports_cfg_parallel and sp.guidance == "cfg")


def test_cli_refusals():
    ns = argparse.Namespace(guidance_scale_2=None, true_cfg_scale=None, num_frames=None, guidance_scale=None,
                            cfg_parallel=False)
    S.check_cli_args(S.SPECS["flux"], ns)  # nothing set: accepted
    ns.num_frames = 17
    with pytest.raises(S.SpecRefusal, match="num-frames"):
        S.check_cli_args(S.SPECS["flux"], ns)
    ns.num_frames = None
    ns.cfg_parallel = True
    with pytest.raises(S.SpecRefusal, match="cfg-parallel"):
        S.check_cli_args(S.SPECS["minimax_h3"], ns)
    S.check_cli_args(S.SPECS["wan"], ns)  # true CFG model: cfg-parallel accepted


def test_generate_kwarg_refusals_and_guidance_range():
    S.check_generate_kwargs(S.SPECS["wan"], {"guidance_scale": 4.0, "guidance_scale_2": 3.0, "negative_prompt": "x"})
    with pytest.raises(S.SpecRefusal, match="guidance_scale_2"):
        S.check_generate_kwargs(S.SPECS["flux"], {"guidance_scale_2": 3.0})
    with pytest.raises(S.SpecRefusal, match="guidance_scale must be"):
        S.check_generate_kwargs(S.SPECS["flux"], {"guidance_scale": 99.0})
    with pytest.raises(S.SpecRefusal, match="guidance_scale"):
        S.check_generate_kwargs(S.SPECS["minimax_h3"], {"guidance_scale": 2.0})


def test_prompt_budgets():
    wan = S.SPECS["wan"]
    S.check_prompt_budgets(wan, {"prompt": {"umt5": 512}})
    with pytest.raises(S.SpecRefusal, match="negative_prompt exceeds"):
        S.check_prompt_budgets(wan, {"negative_prompt": {"umt5": 600}})
    S.check_prompt_budgets(S.SPECS["flux"], {"negative_prompt": {"t5": 900}})  # FLUX budget: prompt only


def test_defaults():
    d = S.generate_defaults(S.SPECS["flux"])
    assert d == {"height": 1024, "width": 1024, "num_inference_steps": 28, "guidance_scale": 3.5}
    assert "guidance_scale" not in S.generate_defaults(S.SPECS["minimax_h3"])


def test_serving_refuses_with_400():
    img = lambda req: torch.zeros(8, 8, 3, dtype=torch.uint8)  # noqa: E731
    c = TestClient(create_app(InProcessEngine(img), "black-forest-labs/FLUX.1-dev"))
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "a"}],
                                             "extra_body": {"guidance_scale_2": 2.0}})
    assert r.status_code == 400 and "guidance_scale_2" in r.text
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "a"}]})
    assert r.status_code == 200
