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


def test_ltx2_gpu_vs_cpu(native):
    from difflet_b200.models.ltx_2.model import LTX2Transformer, audio_coords, get_ltx2_config, video_coords

    cfg = get_ltx2_config("tiny-ltx2")
    cpu = LTX2Transformer.random_init(cfg, seed=5)
    gpu = LTX2Transformer(cfg, {k: (v.cuda() if k.endswith("sst") or k.endswith("_av") or "sst_out" in k
                                    else v.to("cuda", torch.bfloat16)) for k, v in cpu.w.items()})
    g = torch.Generator().manual_seed(2)
    B, Fr, H, W, Ta = 2, 2, 4, 4, 5
    v = torch.randn(B, Fr * H * W, cfg.in_channels, generator=g)
    a = torch.randn(B, Ta, cfg.audio_in_channels, generator=g)
    text = torch.randn(B, 9, cfg.text_dim, generator=g)
    t = torch.tensor([0.4, 0.7])
    valid = torch.tensor([6, 9])
    vc, ac = video_coords(Fr, H, W, cfg), audio_coords(Ta)
    rv, ra = cpu(v, a, t, cpu.prepare_context(text), vcoords=vc, acoords=ac, text_valid=valid)
    ov, oa = gpu(v.cuda().bfloat16(), a.cuda().bfloat16(), t.cuda(), gpu.prepare_context(text.cuda().bfloat16()),
                 vcoords=vc, acoords=ac, text_valid=valid.cuda())
    torch.cuda.synchronize()
    assert _rel(ov, rv) < 3e-2 and _rel(oa, ra) < 3e-2


def test_minimax_h3_gpu_vs_cpu(native):
    from difflet_b200.models.minimax_h3 import layout as L
    from difflet_b200.models.minimax_h3.model import MiniMaxH3Transformer, get_minimax_config

    cfg = get_minimax_config("tiny-minimax-h3")
    cpu = MiniMaxH3Transformer.random_init(cfg, seed=6)
    gpu = MiniMaxH3Transformer(cfg, {k: v.to("cuda", torch.bfloat16) for k, v in cpu.w.items()})
    lay = L.build_layout(num_text_tokens=8, height=64, width=96, num_frames=22, keyframe_anchors=("first",),
                         check_duration=False)
    g = torch.Generator().manual_seed(3)
    vr = torch.randn(1, lay.video_indices.numel(), cfg.patch_dim, generator=g)
    ar = torch.randn(1, lay.audio_indices.numel(), cfg.audio_in_channels, generator=g)
    text = torch.randn(1, 8, cfg.text_dim, generator=g)
    ts = torch.tensor([0.2, 0.5, 0.999])
    tidx = torch.ones(lay.sequence_length, dtype=torch.long)
    tidx[lay.audio_indices] = 0
    tidx[lay.video_indices[: lay.num_condition_rows]] = 2
    rv, ra = cpu(vr, ar, text, ts, tidx, lay)
    ov, oa = gpu(vr.cuda().bfloat16(), ar.cuda().bfloat16(), text.cuda().bfloat16(), ts.cuda(), tidx, lay)
    torch.cuda.synchronize()
    assert _rel(ov, rv) < 3e-2 and _rel(oa, ra) < 3e-2


def test_swiglu_rowmap_partial_rope_kernels(native):
    """The epilogue / norm / scatter features MiniMax-H3 adds, each against the CPU oracle."""
    from difflet_b200.ops import fused as F

    torch.manual_seed(9)
    M, K, Fh = 300, 256, 384
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(2 * Fh, K, device="cuda") * 0.05).bfloat16()
    b = torch.randn(2 * Fh, device="cuda", dtype=torch.bfloat16)
    y = F.linear(x, w, b, act="swiglu")
    ref = F.linear(x.cpu().float(), w.cpu().float(), b.cpu().float(), act="swiglu")
    torch.cuda.synchronize()
    assert y.shape == (M, Fh) and _rel(y, ref) < 2e-2
    gate = torch.randn(5, K, device="cuda")
    rmap = torch.randint(0, 5, (M,), device="cuda", dtype=torch.int32)
    out = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wo = (torch.randn(K, K, device="cuda") * 0.05).bfloat16()
    ref_o = F.linear(x.cpu().float(), wo.cpu().float(), gate=gate.cpu(), resid=out.cpu().float(),
                     gate_row_map=rmap.cpu())
    F.linear(x, wo, out=out, gate=gate, resid=out, gate_row_map=rmap)
    sh, sc = torch.randn(5, K, device="cuda"), torch.randn(5, K, device="cuda")
    n = F.ln_modulate(x, shift=sh, scale=sc, rms=True, row_map=rmap)
    ref_n = F.ln_modulate(x.cpu().float(), shift=sh.cpu(), scale=sc.cpu(), rms=True, row_map=rmap.cpu())
    torch.cuda.synchronize()
    assert _rel(out, ref_o) < 2e-2 and _rel(n, ref_n) < 2e-2
    # partial rotary (first 96 of 128 channels)
    S, H, dh = 40, 2, 128
    qkv = torch.randn(S, 3 * H * dh, device="cuda", dtype=torch.bfloat16)
    ang = torch.rand(S, 48) * 6
    cos, sin = ang.cos().cuda(), ang.sin().cuda()
    q = torch.empty(1, H, S, dh, device="cuda", dtype=torch.bfloat16)
    k, v = torch.empty_like(q), torch.empty_like(q)
    kw = dict(q_off=0, k_off=H * dh, v_off=2 * H * dh, S_src=S, H=H, dh=dh, S_dst=S, norm_mode=0, rope_half=True,
              heads_per_rank=H)
    F.qkv_scatter(qkv, q_dst=[q], k_dst=[k], v_dst=[v], cos=cos, sin=sin, **kw)
    qc, kc, vc = (torch.empty(1, H, S, dh) for _ in range(3))
    F.qkv_scatter(qkv.cpu().float(), q_dst=[qc], k_dst=[kc], v_dst=[vc], cos=cos.cpu(), sin=sin.cpu(), **kw)
    torch.cuda.synchronize()
    assert _rel(q, qc) < 1e-2 and _rel(k, kc) < 1e-2


def test_kl_decoder_native_conv_vs_cpu(native):
    """FLUX's KL decoder with its convolutions on the tcgen05 implicit-GEMM kernel."""
    from difflet_b200.models.vae.autoencoder_kl import KLDecoder, KLDecoderConfig

    cfg = KLDecoderConfig(block_out_channels=(64, 128, 128, 128))
    cpu = KLDecoder.random_init(cfg, seed=4)
    gpu = KLDecoder(cfg, {k: v.to("cuda", torch.bfloat16) for k, v in cpu.w.items()})
    z = torch.randn(1, 16, 16, 24, generator=torch.Generator().manual_seed(5))
    ref = cpu.decode(z)
    out = gpu.decode(z.cuda())
    torch.cuda.synchronize()
    assert "decoder.conv_in.cl" not in gpu.w  # 16 input channels: cuDNN
    assert "decoder.mid_block.resnets.0.conv1.cl" in gpu.w  # 128 channels: native
    assert _rel(out, ref) < 3e-2
