"""Precision schedules (artefacts, synthesis, calibration, apply) and the latent metric collector."""

import json

import pytest
import torch

from difflet_b200.pipeline import precision_schedule as ps
from difflet_b200.pipeline.latent_metrics import SCHEMA, LatentMetricCollector


def _table():
    return {"rows": [{"block": 0, "linear": "transformer_blocks/attn.to_q", "cosine": 0.9999},
                     {"block": 0, "linear": "transformer_blocks/attn.to_k", "cosine": 0.995},
                     {"block": 1, "linear": "transformer_blocks/ff.net.2",
                      "metrics": {"e4m3": {"cosine": 0.99}, "e5m2": {"cosine": 0.998}}}]}


def test_schedule_synthesis_roundtrip(tmp_path):
    s = ps.synthesize_schedule(_table(), 0.999, model_id="m", bundle="b")
    assert s.assignments["0:transformer_blocks/attn.to_q"] == ps.PRECISION_MXFP8_E4M3
    assert s.assignments["0:transformer_blocks/attn.to_k"] == ps.PRECISION_BF16
    assert s.mx_coverage == pytest.approx(1 / 3)
    p = s.write_json(tmp_path / "s.json")
    assert ps.PrecisionSchedule.read_json(p) == s
    assert json.loads(p.read_text())["schema_version"] == 1
    s2 = ps.synthesize_two_threshold_schedule(_table(), 0.999, 0.997, model_id="m", bundle="b")
    assert s2.assignments["1:transformer_blocks/ff.net.2"] == ps.PRECISION_MXFP8_E5M2
    assert s2.coverage_by_precision[ps.PRECISION_MXFP8_E5M2] == pytest.approx(1 / 3)
    fr = ps.two_threshold_frontier(_table(), [(0.999, 0.99)], model_id="m", bundle="b")
    assert len(fr) == 4 and fr[1].mx_coverage == 1.0
    with pytest.raises(ValueError):
        ps.normalize_precision("int4")
    assert ps.cell_of("single_transformer_blocks.7.proj_mlp") == "7:single_transformer_blocks/proj_mlp"


def test_calibrate_and_apply_on_tiny_flux():
    from difflet_b200.models.mmdit import MMDiT
    from difflet_b200.models.mmdit.weights import convert_diffusers
    from difflet_b200.ops import fused as F
    from tests.test_quant import _tiny_flux_sd

    cfg, _, sd = _tiny_flux_sd()
    m = MMDiT(cfg, convert_diffusers(cfg, {k: v.float() for k, v in sd.items()}))
    table = ps.calibrate(m, probe_rows=32)
    assert table["rows"] and all(0.9 < r["cosine"] <= 1.0 + 1e-6 for r in table["rows"])
    # all-E4M3 except the single blocks' output projection (its attn half kept bf16)
    a = {ps.cell_key(r["block"], r["linear"]): "e4m3" for r in table["rows"]}
    a["0:single_transformer_blocks/proj_out_attn"] = "bf16"
    res = ps.apply_schedule(m, ps.PrecisionSchedule("tiny", "b", None, a))
    assert "single.0.proj.w" in res["partial"] and "single.0.proj.w" not in res["quantized"]
    assert isinstance(m.w["double.0.img_qkv.w"], F.MXWeight)
    assert not isinstance(m.w["single.0.proj.w"], F.MXWeight)


def test_latent_metrics_collector(tmp_path):
    coll = LatentMetricCollector(fork_cosine_threshold=0.999)
    g = torch.Generator().manual_seed(0)
    base = torch.randn(1, 64, generator=g)
    for step in range(4):
        noise = torch.randn(3, 64, generator=g) * (0.0 if step < 2 else 1.0)
        coll.callback(step, base.expand(3, 64) + noise)
    m = coll.to_metrics_dict()
    assert m["schema"] == SCHEMA and m["num_steps"] == 4 and m["num_candidates"] == 3
    assert m["shared_prefix_steps"] == 2 and m["shared_prefix_fraction"] == 0.5
    assert m["per_step"][0]["cross_candidate_cosine_vs_0"] == pytest.approx([1.0, 1.0, 1.0])
    coll.record(4, base.expand(3, 64), reference=base)
    assert coll.steps[-1]["cosine_vs_reference"] == pytest.approx([1.0] * 3)
    p = coll.write_json(tmp_path / "m.json")
    assert json.loads(p.read_text())["final_latents_shape"] == [3, 64]
