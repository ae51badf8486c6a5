"""The channels-last HunyuanVideo VAE decoder on the native-kernel path against the PyTorch
statement of the decoder (float64 on the CPU; bf16 kernels vs fp32 on a B200)."""

import pytest
import torch

from difflet_b200.models.vae.hunyuan_vae import HunyuanVAEConfig, HunyuanVAEDecoder, HunyuanVAENative

TINY = HunyuanVAEConfig(block_out_channels=(32, 32, 64, 64), layers_per_block=1, norm_groups=8, tile_latent=64)


def _pair(device, dtype):
    ref = HunyuanVAEDecoder.random_init(TINY, device=device, dtype=dtype, seed=5)
    return ref, HunyuanVAENative(TINY, ref.w)


def test_native_layout_matches_reference_cpu_float64():
    ref, nat = _pair("cpu", torch.float64)
    z = torch.randn(1, 16, 3, 6, 5, generator=torch.Generator().manual_seed(1), dtype=torch.float64)
    a, b = ref.decode(z), nat.decode(z)
    assert a.shape == b.shape == (1, 3, 9, 48, 40)
    assert (a - b).abs().max().item() < 1e-5  # the reference runs its GroupNorm in float32


def test_native_tiled_decode_matches_reference_cpu_float64():
    cfg = HunyuanVAEConfig(block_out_channels=(32, 32, 32, 32), layers_per_block=1, norm_groups=8, tile_latent=4,
                           tile_overlap=2)
    ref = HunyuanVAEDecoder.random_init(cfg, dtype=torch.float64, seed=8)
    nat = HunyuanVAENative(cfg, ref.w)
    z = torch.randn(1, 16, 2, 7, 6, generator=torch.Generator().manual_seed(3), dtype=torch.float64)
    assert (ref.decode(z) - nat.decode(z)).abs().max().item() < 1e-5


@pytest.mark.gpu
def test_native_hunyuan_vae_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    ref32, _ = _pair("cuda", torch.float32)
    nat = HunyuanVAENative(TINY, {k: v.bfloat16() for k, v in ref32.w.items()})
    z = torch.randn(1, 16, 5, 12, 10, generator=torch.Generator().manual_seed(4)).cuda()
    a = ref32.decode(z).float()
    b = nat.decode(z).float()
    torch.cuda.synchronize()
    assert a.shape == b.shape
    rel = ((a - b).norm() / a.norm()).item()
    assert rel < 3e-2, rel
    from difflet_b200 import _native

    _native.check_device_errors()


@pytest.mark.gpu
@pytest.mark.parametrize("C,G", [(32, 8), (128, 32), (512, 32)])
def test_gn_pad_upsample_kernels_gpu(C, G):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from difflet_b200.ops import fused as F

    torch.manual_seed(C)
    x = (torch.randn(1, 3, 9, 11, C, device="cuda") * 3 + 1).bfloat16()
    gamma, beta = torch.randn(C, device="cuda"), torch.randn(C, device="cuda")
    st = F.gn_stats(x, G, 1e-6)
    st_ref = F.gn_stats(x.cpu().double(), G, 1e-6)
    assert torch.allclose(st.cpu().double(), st_ref, rtol=1e-4, atol=1e-4)
    y = torch.zeros(1, 5, 11, 13, C, device="cuda", dtype=torch.bfloat16)
    F.gn_apply(x, st, gamma, beta, G, silu=True, y=y, offs=(2, 1, 1))
    F.pad_replicate(y, (2, 1, 1), (3, 9, 11))
    yr = torch.zeros(1, 5, 11, 13, C, dtype=torch.float64)
    F.gn_apply(x.cpu().double(), st_ref, gamma.cpu(), beta.cpu(), G, silu=True, y=yr, offs=(2, 1, 1))
    F.pad_replicate(yr, (2, 1, 1), (3, 9, 11))
    assert (y.cpu().double() - yr).abs().max().item() < 0.05 * yr.abs().max().item()
    u = torch.zeros(1, 7, 20, 24, C, device="cuda", dtype=torch.bfloat16)
    F.upsample_causal(x, True, u, (1, 1, 1))
    ur = torch.zeros(1, 7, 20, 24, C, dtype=torch.bfloat16)
    F.upsample_causal(x.cpu(), True, ur, (1, 1, 1))
    assert torch.equal(u.cpu(), ur)
