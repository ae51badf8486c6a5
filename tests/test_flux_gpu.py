"""FLUX on the sm_100a kernels (bf16) against the CPU fp32 oracle of the same weights."""

import pytest
import torch

from difflet_b200.models.flux.config import get_config
from difflet_b200.models.flux.model import FluxTransformer, pack_latents
from difflet_b200.models.flux.pipeline import FluxApplication

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("B", [1, 2])
def test_flux_forward_gpu_vs_cpu(native, B):
    cfg = get_config("tiny128")
    cpu = FluxTransformer.random_init(cfg, dtype=torch.float32, seed=3)
    gpu = FluxTransformer(cfg, {k: v.to("cuda", torch.bfloat16) for k, v in cpu.w.items()})
    g = torch.Generator().manual_seed(0)
    x = pack_latents(torch.randn(B, 16, 32, 32, generator=g))
    txt = torch.randn(B, 64, cfg.text_dim, generator=g)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g)
    t = torch.full((B,), 0.6)
    gd = torch.full((B,), 3.5)
    ref = cpu(x, txt, pooled, t, gd, img_hw=(16, 16))
    out = gpu(x.cuda().bfloat16(), txt.cuda().bfloat16(), pooled.cuda(), t.cuda(), gd.cuda(), img_hw=(16, 16))
    torch.cuda.synchronize()
    assert _rel(out, ref) < 3e-2


def test_flux_pipeline_graph_matches_eager(native):
    cfg = get_config("tiny128")
    dit = FluxTransformer.random_init(cfg, device="cuda", dtype=torch.bfloat16, seed=5)
    a = FluxApplication(dit, None, text_len=64, use_cuda_graph=False)
    b = FluxApplication(dit, None, text_len=64, use_cuda_graph=True)
    la = a.generate(prompt="x", height=256, width=256, num_inference_steps=4, output_type="latent")
    lb = b.generate(prompt="x", height=256, width=256, num_inference_steps=4, output_type="latent")
    torch.cuda.synchronize()
    assert torch.equal(la, lb)


def test_flux_pipeline_gpu_vs_cpu(native):
    cfg = get_config("tiny128")
    cpu = FluxTransformer.random_init(cfg, dtype=torch.float32, seed=9)
    gpu = FluxTransformer(cfg, {k: v.to("cuda", torch.bfloat16) for k, v in cpu.w.items()})
    lc = FluxApplication(cpu, None, text_len=64).generate(prompt="p", height=256, width=256,
                                                         num_inference_steps=4, output_type="latent")
    lg = FluxApplication(gpu, None, text_len=64).generate(prompt="p", height=256, width=256,
                                                         num_inference_steps=4, output_type="latent")
    torch.cuda.synchronize()
    assert _rel(lg, lc) < 3e-2
