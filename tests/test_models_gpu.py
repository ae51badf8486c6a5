"""Wan / HunyuanVideo / Qwen-Image on the sm_100a kernels (bf16) vs the CPU fp32 path."""

import pytest
import torch

from difflet_b200.models.mmdit import MMDiT, get_config, pack_latents
from difflet_b200.models.wan.model import WanTransformer, get_wan_config, patchify

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


def test_wan_gpu_vs_cpu(native):
    cfg = get_wan_config("tiny-wan", text_len=32)
    cpu = WanTransformer.random_init(cfg, seed=2)
    gpu = WanTransformer(cfg, {k: (v.cuda() if k.endswith("sst") else v.to("cuda", torch.bfloat16))
                               for k, v in cpu.w.items()})
    g = torch.Generator().manual_seed(0)
    x = patchify(torch.randn(2, 16, 3, 16, 16, generator=g))
    text = torch.randn(2, cfg.text_len, cfg.text_dim, generator=g)
    t = torch.tensor([800.0, 100.0])
    ref = cpu(x, t, cpu.prepare_context(text), grid=(3, 8, 8))
    out = gpu(x.cuda().bfloat16(), t.cuda(), gpu.prepare_context(text.cuda().bfloat16()), grid=(3, 8, 8))
    torch.cuda.synchronize()
    assert _rel(out, ref) < 3e-2


@pytest.mark.parametrize("name", ["tiny-hunyuan", "tiny-qwen"])
def test_mmdit_family_gpu_vs_cpu(native, name):
    cfg = get_config(name)
    cpu = MMDiT.random_init(cfg, seed=4)
    gpu = MMDiT(cfg, {k: v.to("cuda", torch.bfloat16) for k, v in cpu.w.items()})
    g = torch.Generator().manual_seed(1)
    if cfg.family == "hunyuan_video":
        x = pack_latents(torch.randn(1, 16, 3, 16, 16, generator=g))
        grid = (3, 8, 8)
    else:
        x = pack_latents(torch.randn(1, 16, 16, 24, generator=g))
        grid = (1, 8, 12)
    txt = torch.randn(1, 32, cfg.text_dim, generator=g)
    pooled = torch.randn(1, cfg.pooled_dim, generator=g) if cfg.pooled_dim else None
    t = torch.tensor([0.6])
    gd = torch.tensor([6.0])
    valid = torch.tensor([20]) if cfg.family == "hunyuan_video" else None
    ref = cpu(x, txt, pooled, t, gd, grid=grid, txt_valid=valid)
    out = gpu(x.cuda().bfloat16(), txt.cuda().bfloat16(), None if pooled is None else pooled.cuda(), t.cuda(),
              gd.cuda(), grid=grid, txt_valid=None if valid is None else valid.cuda())
    torch.cuda.synchronize()
    assert _rel(out, ref) < 3e-2
