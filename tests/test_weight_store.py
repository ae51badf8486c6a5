"""Pre-sharded weight store: miss writes this rank's shard, hit reads it back bit-exactly
(bf16 and MXFP8 tensors), a changed layout or checkpoint is another entry, a damaged file is a
miss, and the FLUX engine loads a checkpoint through it."""

import json

import torch

from difflet_b200.ops import fused as F
from difflet_b200.utils import weight_store as ws


def test_store_roundtrip(tmp_path, monkeypatch):
    monkeypatch.setenv("DIFFLET_WEIGHT_STORE", str(tmp_path / "store"))
    ckpt = tmp_path / "ckpt"
    ckpt.mkdir()
    (ckpt / "model.safetensors").write_bytes(b"x" * 10)
    w = {"a.w": torch.randn(8, 128).to(torch.bfloat16), "b": torch.arange(4, dtype=torch.float32),
         "m.w": F.MXWeight.quantize(torch.randn(256, 128))}
    calls = []

    def build():
        calls.append(1)
        return w

    got, st = ws.load_or_build("m", ckpt, torch.bfloat16, 2, 1, {"p": 1}, "cpu", build)
    assert st == "miss" and len(calls) == 1
    got, st = ws.load_or_build("m", ckpt, torch.bfloat16, 2, 1, {"p": 1}, "cpu", build)
    assert st == "hit" and len(calls) == 1
    assert torch.equal(got["a.w"], w["a.w"]) and torch.equal(got["b"], w["b"])
    assert isinstance(got["m.w"], F.MXWeight) and torch.equal(got["m.w"].sf, w["m.w"].sf)
    assert torch.equal(got["m.w"].q.view(torch.uint8), w["m.w"].q.view(torch.uint8))
    # another layout -> another entry
    _, st = ws.load_or_build("m", ckpt, torch.bfloat16, 2, 1, {"p": 2}, "cpu", build)
    assert st == "miss"
    # a damaged file is a miss (the manifest no longer matches)
    entry = ws.entry_dir("m", ckpt, torch.bfloat16, 2, {"p": 1})
    f = entry / "tp1-of-2.safetensors"
    f.write_bytes(f.read_bytes()[:-8])
    assert ws.load(entry, 1, 2, "cpu") is None
    man = json.loads((entry / "tp1-of-2.safetensors.manifest.json").read_text())
    assert man["format"] == ws.FORMAT
    monkeypatch.setenv("DIFFLET_WEIGHT_STORE", "off")
    _, st = ws.load_or_build("m", ckpt, torch.bfloat16, 2, 1, {"p": 1}, "cpu", build)
    assert st == "off"


def test_flux_engine_loads_through_store(tmp_path, monkeypatch):
    """A tiny FLUX checkpoint (diffusers names) loads, is stored, and the second load hits."""
    from difflet_b200.models.flux.config import get_config
    from difflet_b200.models.flux.entry import FluxEngine
    from difflet_b200.models.mmdit.weights import to_diffusers
    from difflet_b200.models.flux.model import FluxTransformer
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
    from difflet_b200.registry import registered_models
    from safetensors.torch import save_file

    monkeypatch.setenv("DIFFLET_WEIGHT_STORE", str(tmp_path / "store"))
    cfg = get_config("tiny128")
    m = FluxTransformer.random_init(cfg, dtype=torch.float32, seed=2)
    ck = tmp_path / "flux" / "transformer"
    ck.mkdir(parents=True)
    save_file({k: v.contiguous() for k, v in to_diffusers(cfg, m.w).items()}, str(ck / "model.safetensors"))
    from difflet_b200.models.vae.autoencoder_kl import KLDecoder, KLDecoderConfig

    vae = tmp_path / "flux" / "vae"
    vae.mkdir()
    save_file({k: v.contiguous() for k, v in KLDecoder.random_init(KLDecoderConfig(), seed=1).w.items()},
              str(vae / "model.safetensors"))
    entry = registered_models()["flux"]
    outs = []
    for _ in range(2):
        eng = FluxEngine(entry=entry, model_path=str(tmp_path / "flux"), parallel=DiffletParallelConfig(),
                         dtype=torch.float32, shape={"height": 64, "width": 64}, backend="cpu",
                         application_kwargs={"preset": "tiny128"})
        eng.load(skip_warmup=True)
        outs.append(eng.weight_store)
        assert torch.equal(eng.app.dit.w["double.0.img_qkv.w"], m.w["double.0.img_qkv.w"])
    assert outs == ["miss", "hit"]
