"""MXFP8 kernels on a B200: the quantizer equals the CPU oracle bit for bit, and the
block-scaled tcgen05 GEMM equals an fp32 matmul of the dequantized operands."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(out, ref, tol=2e-3):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale, f"max abs err {err:.4g} vs scale {scale:.4g}"


@pytest.mark.parametrize("R,K", [(300, 256), (64, 3072), (1000, 128)])
def test_quantize_matches_oracle(native, R, K):
    from difflet_b200.ops import fused as F
    from difflet_b200.ops.mx import quantize_mx

    g = torch.Generator().manual_seed(R)
    x = (torch.randn(R, K, generator=g) * torch.logspace(-4, 4, R)[:, None]).bfloat16()
    x[1, :64] = 0
    q_ref, s_ref = quantize_mx(x)
    q, s = F.mx_quantize(x.cuda(), blocked=False)
    torch.cuda.synchronize()
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))
    qb, sb = F.mx_quantize(x.cuda(), blocked=True)
    torch.cuda.synchronize()
    assert torch.equal(qb.cpu().view(torch.uint8), q_ref.view(torch.uint8))
    assert torch.equal(F.unblock_scales(sb.cpu(), R, K), s_ref)


def _deq(q, sb, R, K):
    from difflet_b200.ops import fused as F
    from difflet_b200.ops.mx import dequantize_mx

    return dequantize_mx(q.cpu(), F.unblock_scales(sb.cpu(), R, K), output_dtype=torch.float32)


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 384, 256), (1024, 2048, 1024), (4608, 3072, 3072)])
def test_gemm_mx_matches_dequantized(native, M, N, K):
    from difflet_b200.ops import fused as F

    torch.manual_seed(M + N)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    aq, asf = F.mx_quantize(a)
    wq, wsf = F.mx_quantize(w)
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    y = F.linear_mx(aq, asf, wq, wsf, bias, out_f32=True)
    ref = _deq(aq, asf, M, K) @ _deq(wq, wsf, N, K).t() + bias.float().cpu()
    torch.cuda.synchronize()
    _close(y.cpu(), ref)
    # MXFP8 against the bf16 product: quantization error only
    full = a.float() @ w.float().t() + bias.float()
    assert ((y - full).norm() / full.norm()).item() < 0.06


def test_gemm_mx_epilogues(native):
    from difflet_b200.ops import fused as F

    torch.manual_seed(3)
    M, N, K, B = 256, 512, 384, 2
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    aq, asf = F.mx_quantize(a)
    wq, wsf = F.mx_quantize(w)
    base = _deq(aq, asf, M, K) @ _deq(wq, wsf, N, K).t()
    y = F.linear_mx(aq, asf, wq, wsf, act="gelu", act_lo=128, act_hi=384)
    ref = base.clone()
    ref[:, 128:384] = torch.nn.functional.gelu(ref[:, 128:384], approximate="tanh")
    torch.cuda.synchronize()
    _close(y.cpu(), ref, tol=1e-2)
    gate = torch.randn(B, N, device="cuda")
    resid = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = resid.clone()
    F.linear_mx(aq, asf, wq, wsf, out=out, gate=gate, resid=out, rows_per_batch=M // B)
    ref = resid.float().cpu() + gate.cpu().repeat_interleave(M // B, 0) * base
    torch.cuda.synchronize()
    _close(out.cpu(), ref, tol=1e-2)


def test_matmul_mx_surface(native):
    import difflet_b200.ops as ops

    torch.manual_seed(5)
    a = torch.randn(200, 512, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(320, 512, device="cuda", dtype=torch.bfloat16)
    aq, as_ = ops.quantize_mx(a)
    wq, ws = ops.quantize_mx(w)
    y = ops.matmul_mx(aq, as_, wq, ws, out_dtype=torch.float32)
    ref = ops.matmul_mx(aq.cpu(), as_.cpu(), wq.cpu(), ws.cpu(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    _close(y.cpu(), ref)


def test_quantized_flux_model_matches_cpu_oracle(native):
    """A tiny FLUX with the default MXFP8 targets on the GPU (block-scaled GEMMs, on-the-fly
    activation quantization) against the same quantized model on the CPU oracle."""
    from difflet_b200.models.flux.config import get_config
    from difflet_b200.models.flux.model import FluxTransformer, pack_latents
    from difflet_b200.quant import default_spec
    from difflet_b200.quant.apply import apply_quant

    cfg = get_config("tiny128", hidden=512, heads=4)
    m_cpu = FluxTransformer.random_init(cfg, dtype=torch.float32, seed=3)
    m_gpu = FluxTransformer(cfg, {k: v.to("cuda", torch.bfloat16) for k, v in m_cpu.w.items()})
    spec = default_spec("flux")
    r1, r2 = apply_quant(m_cpu, spec), apply_quant(m_gpu, spec)
    assert r1["quantized"] == r2["quantized"] and r1["quantized"]
    g = torch.Generator().manual_seed(0)
    x = pack_latents(torch.randn(1, 16, 32, 32, generator=g))
    txt = torch.randn(1, 64, cfg.text_dim, generator=g)
    pooled = torch.randn(1, cfg.pooled_dim, generator=g)
    t, gd = torch.tensor([0.4]), torch.tensor([3.5])
    ref = m_cpu(x, txt, pooled, t, gd, img_hw=(16, 16))
    out = m_gpu(x.cuda().bfloat16(), txt.cuda().bfloat16(), pooled.cuda(), t.cuda(), gd.cuda(), img_hw=(16, 16))
    torch.cuda.synchronize()
    assert ((out.float().cpu() - ref).norm() / ref.norm()).item() < 3e-2
