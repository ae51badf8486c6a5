"""MXFP8 quantization (difflet tests/unit/quant/*): spec serialisation and cache fields, the
per-model target tables, the offline checkpoint writer / reader and its refusals, the
fake-quant oracle, and a quantized model against its fake-quant twin."""

import json

import pytest
import torch

from difflet_b200.quant import QuantSpec, default_spec, quant_cache_fields
from difflet_b200.quant import checkpoint as qc
from difflet_b200.quant.apply import apply_quant, dequantize_state_dict


def test_spec_roundtrip_and_cache_fields():
    s = default_spec("flux", tp_degree=2)
    d = s.to_dict()
    assert d["format"] == "mxfp8" and d["split_linears"]
    assert QuantSpec.from_dict(json.loads(json.dumps(d))) == s
    assert quant_cache_fields(None) == {}
    f = s.cache_fields()
    assert f["quant_tp_degree"] == 2 and len(f["quant_targets_sha256"]) == 16
    assert QuantSpec(targets=("a",), compute="nki").compute == "mx"
    with pytest.raises(ValueError):
        QuantSpec(targets=())
    with pytest.raises(ValueError):
        QuantSpec(targets=("a",), compute="bogus")
    assert s.matches("transformer.transformer_blocks.3.attn.to_q")
    assert not s.matches("transformer_blocks.3.attn.to_out.0")
    assert s.k_shards("transformer_blocks.0.ff.net.2") == 2 and s.k_shards("transformer_blocks.0.ff.net.0.proj") == 1


def test_target_tables(monkeypatch):
    with pytest.raises(ValueError):
        default_spec("hunyuan_video_15")
    monkeypatch.setenv("DIFFLET_QUANT_TARGETS", "G1,G3")
    s = default_spec("hunyuan_video_15")
    assert s.matches("transformer_blocks.0.attn.to_q") and s.matches("transformer_blocks.5.ff.net.2")
    assert not s.matches("transformer_blocks.0.attn.add_q_proj")
    monkeypatch.delenv("DIFFLET_QUANT_TARGETS")
    for model in ("flux", "qwen_image", "wan", "hunyuan_video", "ltx_2"):
        assert default_spec(model).targets
    with pytest.raises(ValueError):
        default_spec("nope")


def _tiny_flux_sd():
    from difflet_b200.models.mmdit import MMDiT, get_config
    from difflet_b200.models.mmdit.weights import to_diffusers

    cfg = get_config("tiny128")
    m = MMDiT.random_init(cfg, dtype=torch.float32, seed=1)
    return cfg, m, {k: v.to(torch.bfloat16) for k, v in to_diffusers(cfg, m.w).items()}


def test_writer_reader_roundtrip(tmp_path):
    cfg, _, sd = _tiny_flux_sd()
    spec = default_spec("flux")
    out = qc.write_quantized_dir(sd, tmp_path / "q", spec)
    man = qc.read_manifest(out)
    assert man["counts"]["fp8"] > 0
    qc.check_quantized_dir(out, None, spec)
    with pytest.raises(ValueError):
        qc.check_quantized_dir(out, None, default_spec("flux", tp_degree=2))
    names = qc.quantized_linear_names(out)
    assert "single_transformer_blocks.0.proj_out_attn" in names
    assert "transformer_blocks.0.attn.to_out.0" not in names
    q = qc.load_quantized(out)
    assert q["transformer_blocks.0.attn.to_q.weight"].dtype == torch.float8_e4m3fn
    back = dequantize_state_dict(q)
    assert set(back) == set(sd)
    # dequantized weights equal the fake-quant oracle (exact in bf16); untargeted ones are copied
    from difflet_b200.quant.fake_linear import fake_quant

    k = "transformer_blocks.0.attn.to_q.weight"
    assert torch.equal(back[k], fake_quant(sd[k]))
    k = "transformer_blocks.0.attn.to_out.0.weight"
    assert torch.equal(back[k], sd[k])
    # an earlier quantized checkpoint is replaced; a directory holding anything else is refused
    assert qc.write_quantized_dir(sd, out, spec) == out
    other = tmp_path / "mine"
    other.mkdir()
    (other / "notes.txt").write_text("keep")
    with pytest.raises(ValueError):
        qc.write_quantized_dir(sd, other, spec)
    assert (other / "notes.txt").read_text() == "keep"


def test_writer_refuses_dead_and_fused_patterns():
    _, _, sd = _tiny_flux_sd()
    with pytest.raises(ValueError, match="match no linear"):
        qc.plan(sd, QuantSpec(targets=(r"nothing\.here",)))
    with pytest.raises(ValueError, match="fused split"):
        qc.plan(sd, QuantSpec(targets=(r"single_transformer_blocks\.\d+\.proj_out",),
                              split_linears=(r"single_transformer_blocks\.\d+\.proj_out",)))


def test_quantized_checkpoint_equals_quantize_at_load(tmp_path):
    from difflet_b200.models.mmdit import MMDiT, pack_latents
    from difflet_b200.models.mmdit.weights import convert_diffusers

    cfg, _, sd = _tiny_flux_sd()
    spec = default_spec("flux")
    m1 = MMDiT(cfg, convert_diffusers(cfg, {k: v.float() for k, v in sd.items()}))
    res = apply_quant(m1, spec)
    assert res["quantized"] and not res["partial"]
    out = qc.write_quantized_dir(sd, tmp_path / "q", spec)
    sd2 = dequantize_state_dict(qc.load_quantized(out), dtype=torch.float32)
    m2 = MMDiT(cfg, convert_diffusers(cfg, sd2))
    apply_quant(m2, spec)
    for k in res["quantized"]:
        assert torch.equal(m1.w[k].q.view(torch.uint8), m2.w[k].q.view(torch.uint8)), k
        assert torch.equal(m1.w[k].sf, m2.w[k].sf), k
    g = torch.Generator().manual_seed(0)
    x = pack_latents(torch.randn(1, 16, 16, 16, generator=g))
    txt = torch.randn(1, 16, cfg.text_dim, generator=g)
    pooled = torch.randn(1, cfg.pooled_dim, generator=g)
    t, gd = torch.tensor([0.5]), torch.tensor([3.5])
    assert torch.equal(m1(x, txt, pooled, t, gd, img_hw=(8, 8)), m2(x, txt, pooled, t, gd, img_hw=(8, 8)))


def test_fake_quant_linear():
    from difflet_b200.quant.fake_linear import FakeQuantMXLinear, fake_quantize_model_

    torch.manual_seed(0)
    lin = torch.nn.Linear(64, 32)
    fq = FakeQuantMXLinear(lin)
    x = torch.randn(5, 64)
    y, ref = fq(x), lin(x)
    assert ((y - ref).norm() / ref.norm()).item() < 0.08
    model = torch.nn.Sequential(torch.nn.Linear(64, 64), torch.nn.ReLU(), torch.nn.Linear(64, 32))
    names = fake_quantize_model_(model, QuantSpec(targets=(r"0",)))
    assert names == ["0"] and isinstance(model[0], FakeQuantMXLinear) and isinstance(model[2], torch.nn.Linear)
