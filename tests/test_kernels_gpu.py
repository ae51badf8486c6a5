"""Numerics of every sm_100a kernel against a plain fp32 PyTorch reference."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


# bf16 outputs of fp32-accumulated contractions: half a bf16 ulp is 2^-9 of the value, so a max-abs
# error of 5e-3 x max|ref| leaves 2.5x headroom over rounding; attention (P rounded to bf16 before PV)
# and the fused norm kernels keep the wider default.
GEMM_TOL = 5e-3


def _close(out, ref, tol=2e-2):
    out = out.float()
    ref = ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale, f"max abs err {err:.4g} vs scale {scale:.4g}"


@pytest.mark.parametrize("M,N,K", [(300, 384, 200), (1024, 2048, 512), (128, 64, 64), (4608, 3072, 3072)])
def test_gemm_plain_bias(native, M, N, K):
    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    out = native.gemm(a, b, bias)
    ref = a.float() @ b.float().t() + bias.float()
    torch.cuda.synchronize()
    _close(out, ref, tol=GEMM_TOL)
    out32 = native.gemm(a, b, None, out_f32=True)
    _close(out32, a.float() @ b.float().t(), tol=1e-3)


def test_gemm_gelu_window_and_strided_out(native):
    torch.manual_seed(1)
    M, N, K = 512, 1536, 256
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    big = torch.zeros(M, N + 256, device="cuda", dtype=torch.bfloat16)
    view = big[:, 128 : 128 + N]
    native.gemm(a, b, bias, out=view, epi=1, act_lo=512, act_hi=1024)
    ref = a.float() @ b.float().t() + bias.float()
    ref[:, 512:1024] = torch.nn.functional.gelu(ref[:, 512:1024], approximate="tanh")
    torch.cuda.synchronize()
    _close(view, ref, tol=GEMM_TOL)
    assert big[:, :128].abs().max().item() == 0 and big[:, 128 + N :].abs().max().item() == 0


def test_gemm_gate_residual(native):
    torch.manual_seed(2)
    B, S, N, K = 2, 200, 768, 384
    M = B * S
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    gate = torch.randn(B, N, device="cuda", dtype=torch.float32)
    resid = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    ref = resid.float() + gate.repeat_interleave(S, 0) * (a.float() @ w.float().t() + bias.float())
    native.gemm(a, w, bias, out=resid, epi=2, gate=gate, rows_per_batch=S, resid=resid)
    torch.cuda.synchronize()
    _close(resid, ref, tol=GEMM_TOL)


@pytest.mark.parametrize("D", [256, 3072, 5120])
def test_ln_modulate(native, D):
    torch.manual_seed(3)
    B, S = 2, 77
    x = torch.randn(B * S, D, device="cuda", dtype=torch.bfloat16) * 3 + 1
    shift = torch.randn(B, D, device="cuda")
    scale = torch.randn(B, D, device="cuda") * 0.1
    y = native.ln_modulate(x, shift=shift, scale=scale, rows_per_batch=S, eps=1e-6)
    xf = x.float()
    ref = torch.nn.functional.layer_norm(xf, (D,), eps=1e-6)
    ref = ref * (1 + scale.repeat_interleave(S, 0)) + shift.repeat_interleave(S, 0)
    torch.cuda.synchronize()
    _close(y, ref)
    w = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    y2 = native.ln_modulate(x, w=w, rms=True, eps=1e-6)
    ref2 = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    _close(y2, ref2)


def _rope_ref(x, cos, sin):
    # x [..., S, dh] fp32, interleaved pairs
    x0, x1 = x[..., 0::2], x[..., 1::2]
    o0 = x0 * cos - x1 * sin
    o1 = x1 * cos + x0 * sin
    return torch.stack([o0, o1], -1).flatten(-2)


@pytest.mark.parametrize("dh", [64, 128])
def test_qkv_scatter_norm_rope(native, dh):
    torch.manual_seed(4)
    B, S, H = 2, 50, 4
    D = H * dh
    qkv = torch.randn(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    S_dst, off = S + 10, 10
    pos = torch.arange(S_dst, device="cuda", dtype=torch.float32)[:, None]
    freqs = 1.0 / (10000 ** (torch.arange(0, dh, 2, device="cuda").float() / dh))
    ang = pos * freqs[None]
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    q = torch.zeros(B, H, S_dst, dh, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros_like(q)
    v = torch.zeros_like(q)
    native.qkv_scatter(qkv, 0, D, 2 * D, S, H, dh, 1, wq, wk, 1e-6, cos, sin, off, False, H,
                       [q.data_ptr()], [k.data_ptr()], [v.data_ptr()], S_dst, off, False, False, 0, 0, 0, 0, 0, None, 0)
    torch.cuda.synchronize()
    x = qkv.float().view(B, S, 3, H, dh).permute(2, 0, 3, 1, 4)  # 3,B,H,S,dh

    def norm(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()

    c, s_ = cos[off:], sin[off:]
    _close(q[:, :, off:], _rope_ref(norm(x[0], wq), c, s_))
    _close(k[:, :, off:], _rope_ref(norm(x[1], wk), c, s_))
    _close(v[:, :, off:], x[2])
    assert q[:, :, :off].abs().max().item() == 0


def test_qkv_scatter_across_heads_half_rope(native):
    torch.manual_seed(5)
    B, S, H, dh = 1, 33, 8, 128
    D = H * dh
    qkv = torch.randn(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    ang = torch.rand(S, dh // 2, device="cuda") * 6
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    q = torch.empty(B, S, D, device="cuda", dtype=torch.bfloat16)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    native.qkv_scatter(qkv, 0, D, 2 * D, S, H, dh, 2, wq, wk, 1e-6, cos, sin, 0, True, H,
                       [q.data_ptr()], [k.data_ptr()], [v.data_ptr()], S, 0, True, False, 0, 0, 0, 0, 0, None, 0)
    torch.cuda.synchronize()
    x = qkv.float().view(S, 3, D)
    qn = x[:, 0] * torch.rsqrt(x[:, 0].pow(2).mean(-1, keepdim=True) + 1e-6) * wq.float()
    qn = qn.view(S, H, dh)
    x1, x2 = qn[..., : dh // 2], qn[..., dh // 2 :]
    c, s_ = cos[:, None], sin[:, None]
    ref = torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_], -1).reshape(S, D)
    _close(q[0], ref)


def test_qkv_scatter_kv_replicate(native):
    """Gather-KV store pattern: k / v of all heads to every destination, q to a local buffer."""
    from difflet_b200.ops import fused as F

    torch.manual_seed(15)
    B, S, H, dh = 2, 40, 4, 128
    D = H * dh
    S_loc, row, S_all, pos = 64, 24, 160, 100
    qkv = torch.randn(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    ang = torch.rand(S_all, dh // 2, device="cuda") * 6
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    q = torch.zeros(B, H, S_loc, dh, device="cuda", dtype=torch.bfloat16)
    ks = [torch.zeros(B, H, S_all, dh, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    vs = [torch.zeros_like(ks[0]) for _ in range(3)]
    kw = dict(q_off=0, k_off=D, v_off=2 * D, S_src=S, H=H, dh=dh, norm_mode=1, wq=wq, wk=wk, eps=1e-6, cos=cos,
              sin=sin, rope_pos_off=pos, S_dst=S_all, seq_off=pos, kv_replicate=True, q_S_dst=S_loc, q_seq_off=row)
    F.qkv_scatter(qkv, q_dst=[q, None, None], k_dst=ks, v_dst=vs, **kw)
    qc = torch.zeros(B, H, S_loc, dh, dtype=torch.float32)
    kc = torch.zeros(B, H, S_all, dh, dtype=torch.float32)
    vc = torch.zeros_like(kc)
    kw.update(wq=wq.cpu().float(), wk=wk.cpu().float(), cos=cos.cpu(), sin=sin.cpu())
    F.qkv_scatter(qkv.cpu().float(), q_dst=[qc], k_dst=[kc], v_dst=[vc], **kw)
    torch.cuda.synchronize()
    _close(q, qc.cuda())
    for kd, vd in zip(ks, vs):
        _close(kd, kc.cuda())
        _close(vd, vc.cuda())


def test_gemv_and_timestep(native):
    torch.manual_seed(6)
    N, K, Bt = 3000, 3072, 2
    W = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    x = torch.randn(Bt, K, device="cuda")
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    y = native.gemv(W, x, bias, silu_in=True)
    ref = torch.nn.functional.silu(x) @ W.float().t() + bias.float()
    _close(y, ref, tol=1e-3)
    t = torch.tensor([999.0, 0.5], device="cuda")
    e = native.timestep_embed(t, 256, 10000.0, True, 0.0, 1.0)
    half = 128
    ex = -math.log(10000.0) * torch.arange(half, device="cuda", dtype=torch.float32) / half
    arg = t[:, None] * torch.exp(ex)[None]
    ref = torch.cat([arg.cos(), arg.sin()], -1)
    assert (e - ref).abs().max().item() < 2e-3


def test_euler_cfg(native):
    n = 16 * 4096
    x = torch.randn(n, device="cuda")
    x16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    u = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    c = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    ref = x + (-0.03) * (u.float() + 4.0 * (c.float() - u.float()))
    native.euler_step(x, x16, u, c, -0.03, 4.0)
    torch.cuda.synchronize()
    assert (x - ref).abs().max().item() < 1e-5
    assert (x16.float() - ref).abs().max().item() < 0.05


def _attn_ref(q, k, v, scale, lo=None, hi=None):
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) * scale
    if lo is not None:
        idx = torch.arange(k.shape[2], device=q.device)
        mask = (idx[None, :] >= lo[:, None]) & (idx[None, :] < hi[:, None])  # B, Sk
        s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.softmax(s, -1)
    return torch.einsum("bhqk,bhkd->bhqd", p, v.float()), lse


@pytest.mark.parametrize("B,H,Sq,Sk", [(1, 2, 128, 128), (2, 3, 300, 333), (1, 4, 1024, 2048)])
def test_attention(native, B, H, Sq, Sk):
    torch.manual_seed(7)
    q = torch.randn(B, H, Sq, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, H, Sk, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, H, Sk, 128, device="cuda", dtype=torch.bfloat16)
    scale = 1 / math.sqrt(128)
    lse = torch.empty(B, H, Sq, device="cuda")
    o = native.attention(q, k, v, scale, lse=lse)
    ref, ref_lse = _attn_ref(q, k, v, scale)
    torch.cuda.synchronize()
    _close(o, ref)
    assert (lse - ref_lse).abs().max().item() < 2e-2


def test_attention_lse_merge_over_key_blocks(native):
    """Ring emulated on one GPU: the keys in 3 blocks (one empty for a batch through its
    window), partials merged by the kernel epilogue, equal full attention."""
    from difflet_b200.ops import fused as F

    torch.manual_seed(16)
    B, H, Sq = 2, 3, 300
    blocks = [256, 200, 130]
    q = torch.randn(B, H, Sq, 128, device="cuda", dtype=torch.bfloat16) * 3
    ks = [torch.randn(B, H, n, 128, device="cuda", dtype=torch.bfloat16) * 3 for n in blocks]
    vs = [torch.randn(B, H, n, 128, device="cuda", dtype=torch.bfloat16) for n in blocks]
    his = [torch.tensor([256, 256], device="cuda", dtype=torch.int32),
           torch.tensor([0, 150], device="cuda", dtype=torch.int32),
           torch.tensor([130, 7], device="cuda", dtype=torch.int32)]
    scale = 1 / math.sqrt(128)
    acc_o = torch.empty(B, H, Sq, 128, device="cuda")
    acc_lse = torch.empty(B, H, Sq, device="cuda")
    out = torch.empty(B, Sq, H * 128, device="cuda", dtype=torch.bfloat16)
    o_view = out.view(B, Sq, H, 128).permute(0, 2, 1, 3)
    lse = torch.empty(B, H, Sq, device="cuda")
    for i, (k, v, hi) in enumerate(zip(ks, vs, his)):
        mode = F.MERGE_FIRST if i == 0 else (F.MERGE_LAST if i == len(blocks) - 1 else F.MERGE_MID)
        F.attention_partial(q, k, v, scale, acc_o, acc_lse, mode, out=o_view, lse=lse if i == 2 else None,
                            kv_hi=hi)
    # reference: concatenate the valid keys of each block
    kk, vv, keep = torch.cat(ks, 2), torch.cat(vs, 2), []
    for n, hi in zip(blocks, his):
        keep.append(torch.arange(n, device="cuda")[None] < hi[:, None].long())
    keep = torch.cat(keep, 1)  # [B, S_all]
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), kk.float()) * scale
    s = s.masked_fill(~keep[:, None, None, :], float("-inf"))
    ref_lse = torch.logsumexp(s, -1)
    ref = torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), vv.float())
    torch.cuda.synchronize()
    _close(o_view, ref)
    assert (lse - ref_lse).abs().max().item() < 2e-2


def test_attention_bounds_large_logits_token_major(native):
    torch.manual_seed(8)
    B, H, S = 2, 2, 384
    q = torch.randn(B, H, S, 128, device="cuda", dtype=torch.bfloat16) * 4
    k = torch.randn(B, H, S, 128, device="cuda", dtype=torch.bfloat16) * 4
    v = torch.randn(B, H, S, 128, device="cuda", dtype=torch.bfloat16)
    lo = torch.tensor([0, 70], device="cuda", dtype=torch.int32)
    hi = torch.tensor([300, 201], device="cuda", dtype=torch.int32)
    out = torch.empty(B, S, H * 128, device="cuda", dtype=torch.bfloat16)
    o_view = out.view(B, S, H, 128).permute(0, 2, 1, 3)
    scale = 1 / math.sqrt(128)
    native.attention(q, k, v, scale, out=o_view, kv_lo=lo, kv_hi=hi)
    ref, _ = _attn_ref(q, k, v, scale, lo, hi)
    torch.cuda.synchronize()
    _close(o_view, ref)


def test_attention_running_max_jumps(native):
    """Scores that jump after the first key tile take every running-max path of the softmax:
    growth beyond 2^64 inside the second half of a tile (rescale after the first half of PV),
    growth accepted on the stale max (second half, then rescaled by the next tile), growth in
    the first half (exact tile), and large random logits; half of the query rows see no jump."""
    torch.manual_seed(21)
    B, H, Sq, Sk = 1, 4, 256, 512
    q = torch.randn(B, H, Sq, 128, device="cuda") * 0.05
    k = torch.randn(B, H, Sk, 128, device="cuda") * 0.05
    v = torch.randn(B, H, Sk, 128, device="cuda")
    q[..., 0] = (torch.arange(Sq, device="cuda") % 2).float()  # odd rows see the jump
    k[..., 0] = 0.0
    k[0, 0, 228, 0] = 60.0  # tile 1, second half: 2^86 above the running max
    k[0, 1, 218, 0] = 20.0  # tile 1, second half: 2^29, accepted on the stale max
    k[0, 2, 266, 0] = 60.0  # tile 2, first half
    k[0, 3] = torch.randn(Sk, 128, device="cuda") * 2.0
    q[0, 3] = torch.randn(Sq, 128, device="cuda") * 2.0
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    scale = 1.0
    ref, ref_lse = _attn_ref(q, k, v, scale)
    lse = torch.empty(B, H, Sq, device="cuda")
    o = native.attention(q, k, v, scale, lse=lse)
    torch.cuda.synchronize()
    _close(o, ref)
    assert (lse - ref_lse).abs().max().item() < 5e-2
    assert native.error_word(torch.cuda.current_device()).cpu().tolist() == [0, 0, 0, 0]


def test_error_word_clean(native):
    torch.cuda.synchronize()
    assert native.error_word(torch.cuda.current_device()).cpu().tolist() == [0, 0, 0, 0]


def test_rel_l1_probe_twice(native):
    torch.manual_seed(9)
    for n in (1 << 20, 12345):
        a = torch.randn(n, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
        ref = ((a.float() - b.float()).abs().sum() / b.float().abs().sum()).item()
        for _ in range(2):  # second call reuses the scratch (ticket must be back at zero)
            out = native.rel_l1(a, b)
            torch.cuda.synchronize()
            assert abs(out.item() - ref) < 1e-4 * abs(ref)


def test_cfg_combine_local_pointer(native):
    n = 4096 * 64 + 3
    u = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    c = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(n, device="cuda")
    native.cfg_combine(c, u.data_ptr(), out, 4.0, True)   # this rank holds cond
    ref = u.float() + 4.0 * (c.float() - u.float())
    torch.cuda.synchronize()
    assert (out - ref).abs().max().item() < 1e-4
    native.cfg_combine(u, c.data_ptr(), out, 4.0, False)  # this rank holds uncond
    torch.cuda.synchronize()
    assert (out - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize("N,T,H,W,Ci,Co,k,causal", [
    (1, 1, 40, 72, 128, 128, (1, 3, 3), True),     # 2-D (KL decoder), partial 128-wide row tiles
    (1, 5, 12, 150, 96, 96, (3, 3, 3), True),      # causal 3-D, 32-channel steps (Wan widths)
    (2, 3, 8, 20, 64, 256, (3, 3, 3), False),      # symmetric temporal padding, BN 256
    (1, 4, 6, 130, 192, 64, (1, 1, 1), True),      # 1x1x1 shortcut
    (1, 3, 10, 70, 96, 192, (3, 3, 3), True),      # BN 192
    (1, 2, 9, 33, 384, 96, (3, 3, 3), True),       # BN 96 (one N tile), 64-channel steps
])
def test_conv_cl_matches_torch(native, N, T, H, W, Ci, Co, k, causal):
    from difflet_b200.ops import fused as F

    torch.manual_seed(11)
    x = torch.randn(N, T, H, W, Ci, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(Co, Ci, *k, device="cuda") / (Ci * k[0] * k[1] * k[2]) ** 0.5).bfloat16()
    b = torch.randn(Co, device="cuda", dtype=torch.bfloat16)
    resid = torch.randn(N, T, H, W, Co, device="cuda", dtype=torch.bfloat16)
    w2 = F.conv_weight(w)
    y = F.conv_cl(x, w2, b, kt=k[0], kh=k[1], kw=k[2], causal=causal, resid=resid)
    ref = F.conv_cl(x.cpu().float(), w2.cpu().float(), b.cpu().float(), kt=k[0], kh=k[1], kw=k[2], causal=causal,
                    resid=resid.cpu().float())
    torch.cuda.synchronize()
    _close(y.cpu(), ref, tol=GEMM_TOL)


@pytest.mark.parametrize("T,H,W,Ci,Co,valid", [
    (4, 7, 24, 128, 128, "th"),    # a 5-row decode slab with its two halo rows, cached frames in front
    (3, 12, 24, 64, 64, "th"),     # a 10-row slab
    (2, 3, 40, 96, 96, "h"),       # one output row
    (4, 9, 18, 64, 128, "thw"),    # replicate-padded clip (every border carried by the input)
    (3, 6, 130, 32, 96, "tw"),     # two 128-wide column tiles of a valid-W row
])
def test_conv_cl_valid_padding_matches_torch(native, T, H, W, Ci, Co, valid):
    """valid_t / valid_h / valid_w: no padding along the axis, the input already carries the
    context (causal frames, halo rows of a slab, replicate-padded borders); small slabs included."""
    from difflet_b200.ops import fused as F

    torch.manual_seed(12)
    vt, vh, vw = ("t" in valid), ("h" in valid), ("w" in valid)
    x = torch.randn(1, T, H, W, Ci, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(Co, Ci, 3, 3, 3, device="cuda") / (Ci * 27) ** 0.5).bfloat16()
    b = torch.randn(Co, device="cuda", dtype=torch.bfloat16)
    w2 = F.conv_weight(w)
    y = F.conv_cl(x, w2, b, valid_t=vt, valid_h=vh, valid_w=vw)
    ref = F.conv_cl(x.cpu().float(), w2.cpu().float(), b.cpu().float(), valid_t=vt, valid_h=vh, valid_w=vw)
    torch.cuda.synchronize()
    assert y.shape == ref.shape == (1, T - 2 if vt else T, H - 2 if vh else H, W - 2 if vw else W, Co)
    _close(y.cpu(), ref, tol=GEMM_TOL)


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (1000, 1280, 512), (4608, 3072, 3072), (300, 2304, 128)])
def test_gemm_cta_pair(native, M, N, K):
    """The 2-CTA (cta_group::2) GEMM: plain, GELU window and gated residual epilogues."""
    torch.manual_seed(M + K)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    ref = a.float() @ b.float().t() + bias.float()
    out = native.gemm(a, b, bias, cta_mode=2)
    torch.cuda.synchronize()
    _close(out, ref, tol=GEMM_TOL)
    g = native.gemm(a, b, bias, epi=1, act_lo=128, act_hi=N, cta_mode=2)
    ref_g = ref.clone()
    ref_g[:, 128:] = torch.nn.functional.gelu(ref_g[:, 128:], approximate="tanh")
    gate = torch.randn(2, N, device="cuda")
    resid = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    r = resid.clone()
    native.gemm(a, b, bias, out=r, epi=2, gate=gate, rows_per_batch=(M + 1) // 2, resid=r, cta_mode=2)
    rows = torch.arange(M, device="cuda") // ((M + 1) // 2)
    ref_r = resid.float() + gate[rows] * ref
    torch.cuda.synchronize()
    _close(g, ref_g, tol=GEMM_TOL)
    _close(r, ref_r, tol=GEMM_TOL)
    assert native.error_word(0)[0].item() == 0


def test_row_sumsq_and_external_rms_norm(native):
    """Across-heads q/k RMS from supplied per-row sums (the tensor-parallel path): the
    sums kernel and qkv_scatter norm_mode 3 against the fp32 oracle."""
    from difflet_b200.ops import fused as F

    torch.manual_seed(31)
    S, H, dh = 70, 4, 128
    D = H * dh
    qkv = torch.randn(S, 3 * D, device="cuda", dtype=torch.bfloat16)
    rs = F.row_sumsq(qkv, 0, D, D)
    ref = torch.stack([qkv[:, :D].float().pow(2).sum(1), qkv[:, D:2 * D].float().pow(2).sum(1)], 1)
    _close(rs, ref, 1e-4)
    rs_total = rs * 2.0  # as if the other half of the heads lived on another rank with equal sums
    wq = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    q = torch.empty(1, H, S, dh, device="cuda", dtype=torch.bfloat16)
    k, v = torch.empty_like(q), torch.empty_like(q)
    kw = dict(q_off=0, k_off=D, v_off=2 * D, S_src=S, H=H, dh=dh, S_dst=S, norm_mode=3, eps=1e-6,
              norm_total=2 * D, heads_per_rank=H)
    F.qkv_scatter(qkv, q_dst=[q], k_dst=[k], v_dst=[v], wq=wq, wk=wk, row_sumsq=rs_total, **kw)
    qc, kc, vc = (torch.zeros(1, H, S, dh) for _ in range(3))
    F.qkv_scatter(qkv.cpu().float(), q_dst=[qc], k_dst=[kc], v_dst=[vc], wq=wq.cpu().float(), wk=wk.cpu().float(),
                  row_sumsq=rs_total.cpu(), **kw)
    torch.cuda.synchronize()
    _close(q, qc.cuda())
    _close(k, kc.cuda())
    _close(v, vc.cuda())


# the planner picks 2 ranges for (576, 3072, 15360), 3 for (512, 3072, 12288) and (256, 1024, 4096),
# 4 for (256, 1024, 16384) and (256, 512, 8192) (128-column tiles)
@pytest.mark.parametrize("M,N,K", [(300, 3072, 4096), (576, 3072, 15360), (64, 1536, 2048), (512, 3072, 12288),
                                   (256, 1024, 4096), (256, 1024, 16384), (256, 512, 8192)])
def test_gemm_split_k_small_m(native, monkeypatch, M, N, K):
    """Small-M GEMMs split K across SMs (serial f32 fixup): plain + bias and the gated residual
    epilogue against the fp32 reference, repeated calls (the counters return to 0), and a
    grouped launch of two split problems."""
    from difflet_b200.ops import fused as F

    torch.manual_seed(41)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.03
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    ref = a.float() @ b.float().t() + bias.float()
    for _ in range(3):
        _close(F.linear(a, b, bias), ref, tol=GEMM_TOL)
    gate = torch.randn(1, N, device="cuda")
    resid = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = resid.clone()
    F.linear(a, b, bias, out=out, gate=gate, resid=out, rows_per_batch=M)
    _close(out, resid.float() + gate * ref, tol=GEMM_TOL)
    a2 = torch.randn(M // 2 + 8, K, device="cuda", dtype=torch.bfloat16)
    o1, o2 = F.linear_group([dict(x=a, w=b, b=bias), dict(x=a2, w=b, b=bias)])
    _close(o1, ref, tol=GEMM_TOL)
    _close(o2, a2.float() @ b.float().t() + bias.float(), tol=GEMM_TOL)
    monkeypatch.setenv("DIFFLET_GEMM_SPLITK", "0")  # registered already: the switch only affects new devices
    torch.cuda.synchronize()
    from difflet_b200 import _native

    _native.check_device_errors()


@pytest.mark.parametrize("split", [-1, 2, 5])
def test_attention_split_kv(native, split):
    """Key-range splits (chunks + log-sum-exp combine): auto choice (a 3-head launch that would
    leave SMs idle) and forced counts, with a per-batch key window and LSE output."""
    torch.manual_seed(17)
    B, H, Sq, Sk = 2, 3, 1100, 2600
    q = torch.randn(B, H, Sq, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, H, Sk, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, H, Sk, 128, device="cuda", dtype=torch.bfloat16)
    scale = 1 / math.sqrt(128)
    lo = torch.tensor([0, 300], device="cuda", dtype=torch.int32)
    hi = torch.tensor([2600, 1700], device="cuda", dtype=torch.int32)
    lse = torch.empty(B, H, Sq, device="cuda")
    o = native.attention(q, k, v, scale, lse=lse, kv_lo=lo, kv_hi=hi, kv_split=split)
    ref, ref_lse = _attn_ref(q, k, v, scale, lo.long(), hi.long())
    torch.cuda.synchronize()
    _close(o, ref)
    assert (lse - ref_lse).abs().max().item() < 2e-2


@pytest.mark.parametrize("n0,n1,split", [(0, 300, 1), (0, 300, 3), (64, 236, 1), (64, 236, 2)])
def test_attention_output_scatter_to_owning_ranks(native, n0, n1, split):
    """The Ulysses heads->sequence exchange in the attention epilogue: each output row goes to
    the rank that owns it (rank r owns rows [r n0, (r+1) n0) of the first segment and
    [r n1, (r+1) n1) of the second, stored at local rows [0, n0) and [n0, n0 + n1)), at this
    rank's head columns.  The owners' buffers are local tensors here.  n0 = 0 is a single-stream
    sequence (Wan); the split runs the key-chunk combine pass, which stores the same way."""
    torch.manual_seed(19)
    world, B, Hl, dh = 3, 2, 2, 128
    S_loc = n0 + n1
    S = world * S_loc
    q = torch.randn(B, Hl, S, dh, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, Hl, S, dh, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, Hl, S, dh, device="cuda", dtype=torch.bfloat16)
    rank = 1  # this rank's heads fill columns [rank Hl dh, (rank + 1) Hl dh) of every owner's rows
    ld = world * Hl * dh
    owners = [torch.zeros(B * S_loc + 1, ld, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    col = rank * Hl * dh * 2
    scale = 1 / math.sqrt(dh)
    native.attention(q, k, v, scale, None, None, None, None, [t.data_ptr() + col for t in owners], n0 * world, n0,
                     n1, [S_loc * ld, dh, ld], kv_split=split)
    ref, _ = _attn_ref(q, k, v, scale, None, None)  # [B, Hl, S, dh]
    torch.cuda.synchronize()
    rows = torch.cat([torch.arange(r * n0, (r + 1) * n0) for r in range(world)] +
                     [n0 * world + torch.arange(r * n1, (r + 1) * n1) for r in range(world)]).cuda()
    own = torch.cat([torch.full((n0,), r) for r in range(world)] + [torch.full((n1,), r) for r in range(world)]).cuda()
    lrow = torch.cat([torch.arange(n0) for _ in range(world)] + [n0 + torch.arange(n1) for _ in range(world)]).cuda()
    for r in range(world):
        sel = own == r
        mine = owners[r][: B * S_loc].view(B, S_loc, world, Hl, dh)[:, :, rank]  # [B, S_loc, Hl, dh]
        want = torch.zeros(B, S_loc, Hl, dh, device="cuda")
        want[:, lrow[sel]] = ref[:, :, rows[sel]].permute(0, 2, 1, 3).float()
        _close(mine, want)
        assert owners[r][B * S_loc:].abs().sum() == 0  # nothing past the owner's rows
        other = owners[r][: B * S_loc].view(B, S_loc, world, Hl * dh)
        assert other[:, :, [c for c in range(world) if c != rank]].abs().sum() == 0  # other ranks' columns


@pytest.mark.parametrize("n,swap", [(1 << 20, False), (12345, True), (7, False)])
def test_guided_step_unipc_matches_oracle(native, n, swap):
    """The fused CFG combine + UniPC step (csrc/sched.cu) over several steps against the same
    update run by the CPU oracle in fp32; ``swap`` feeds the cond branch as ``a``."""
    from difflet_b200.schedulers.guided import GuidedSampler
    from difflet_b200.schedulers.unipc import UniPCScheduler

    torch.manual_seed(n)
    x0 = torch.randn(n)
    gpu = GuidedSampler(UniPCScheduler(shift=5.0).set_timesteps(6), x0.cuda().clone(),
                        torch.empty(n, device="cuda", dtype=torch.bfloat16))
    cpu = GuidedSampler(UniPCScheduler(shift=5.0).set_timesteps(6), x0.clone())
    for _ in range(6):
        u = torch.randn(n).bfloat16()
        c = torch.randn(n).bfloat16()
        if swap:
            gpu.step(c.cuda(), u.cuda(), 5.0, swap=True)
        else:
            gpu.step(u.cuda(), c.cuda(), 5.0)
        cpu.step(u, c, 5.0)
    torch.cuda.synchronize()
    ref = cpu.x
    assert (gpu.x.cpu() - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()
    assert torch.equal(gpu.x16.cpu(), gpu.x.cpu().bfloat16())
    assert native.error_word(torch.cuda.current_device()).cpu().tolist() == [0, 0, 0, 0]


def test_guided_step_euler(native):
    from difflet_b200.schedulers import FlowMatchEulerScheduler
    from difflet_b200.schedulers.guided import GuidedSampler

    n = 4096 + 3
    sched = FlowMatchEulerScheduler(use_dynamic_shifting=False, shift=3.0).set_timesteps(4)
    x = torch.randn(n, device="cuda")
    ref = x.clone()
    s = GuidedSampler(sched, x)
    for i in range(4):
        u = torch.randn(n, device="cuda", dtype=torch.bfloat16)
        c = torch.randn(n, device="cuda", dtype=torch.bfloat16)
        s.step(u, c, 4.0)
        ref = ref + sched.dt(i) * (u.float() + 4.0 * (c.float() - u.float()))
    torch.cuda.synchronize()
    assert (x - ref).abs().max().item() <= 1e-5 * ref.abs().max().item()


def test_peer_barrier_timeout_fails_fast(native):
    """A barrier slot that nothing ever sets: the bounded wait runs out, the kernel records a
    communication timeout and returns (the context stays usable), the host raises
    CommTimeoutError, and the next barrier returns at once instead of waiting again."""
    import time

    from difflet_b200 import _native
    from difflet_b200.utils.errors import CommTimeoutError

    torch.cuda.synchronize()
    _native.clear_device_errors()
    world = 2
    mine = torch.zeros(world, device="cuda", dtype=torch.int32)    # this rank's slots
    ghost = torch.zeros(world, device="cuda", dtype=torch.int32)   # a "peer" that never arrives
    counter = torch.zeros(1, device="cuda", dtype=torch.int32)
    flags = [mine.data_ptr(), ghost.data_ptr()]
    native.peer_barrier(flags, counter, 0, 20_000_000)  # ~10 ms at 2 GHz
    torch.cuda.synchronize()
    with pytest.raises(CommTimeoutError):
        _native.check_device_errors()
    t0 = time.perf_counter()
    native.peer_barrier(flags, counter, 0, 4_000_000_000)  # would wait ~2 s if it waited at all
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.5
    with pytest.raises(CommTimeoutError):  # still recorded: later collectives keep failing fast
        _native.check_device_errors()
    _native.clear_device_errors()
    _native.check_device_errors()
    x = torch.randn(256, 256, device="cuda", dtype=torch.bfloat16)
    assert torch.isfinite(native.gemm(x, x, None).float()).all()  # the context is still usable


def test_refused_launch_raises_with_its_status(native):
    """A launch the host code refuses (an operand off its 16-byte alignment) raises a Python
    error naming the status code; no kernel runs and the context stays usable."""
    x = torch.randn(128 * 64 + 8, device="cuda", dtype=torch.bfloat16)
    a = x[1:1 + 128 * 64].view(128, 64)  # 2 bytes past an aligned address
    b = torch.randn(64, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match=r"gemm launch failed with status -3"):
        native.gemm(a, b, None)
    y = native.gemm(b, b, None)
    torch.cuda.synchronize()
    _close(y, b.float() @ b.float().t(), tol=GEMM_TOL)
    # a row scatter whose owners cannot hold every row (2 owners x 40 rows for 128 rows)
    owners = [torch.zeros(64, 64, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    with pytest.raises(RuntimeError, match=r"gemm launch failed with status -10"):
        native.gemm(b.repeat(2, 1), b, None, None, 0, out_peer=[t.data_ptr() for t in owners], rows_per_rank=40,
                    peer_row_off=0, ldd=64)
    torch.cuda.synchronize()
    assert all(t.abs().sum() == 0 for t in owners)


def test_vae_chan_norm_and_upsample_with_halo_stores(native):
    """Channel RMS + SiLU and the nearest upsampler write their rows at the halo offset and their
    boundary rows into the neighbouring slabs' halo rows (here local tensors stand in for the
    peers' buffers, with different row counts, as the last slab of an uneven split has)."""
    from difflet_b200.ops import fused as F

    torch.manual_seed(5)
    Fr, rows, W, C = 3, 5, 24, 96
    x = torch.randn(Fr, rows, W, C, device="cuda", dtype=torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(C, device="cuda")).bfloat16()
    y = torch.zeros(Fr, rows + 2, W, C, device="cuda", dtype=torch.bfloat16)
    up = torch.zeros(Fr, 7 + 2, W, C, device="cuda", dtype=torch.bfloat16)
    down = torch.zeros(Fr, 4 + 2, W, C, device="cuda", dtype=torch.bfloat16)
    F.vae_chan_norm(x, gamma, y, silu=True, halo=1, up=up.data_ptr(), up_rows=7, down=down.data_ptr(), down_rows=4)
    xf = x.float()
    ref = torch.nn.functional.silu(xf / xf.norm(dim=-1, keepdim=True) * C ** 0.5 * gamma.float())
    torch.cuda.synchronize()
    _close(y[:, 1:rows + 1], ref)
    assert torch.equal(up[:, 8], y[:, 1]) and torch.equal(down[:, 0], y[:, rows])
    assert y[:, 0].abs().sum() == 0 and y[:, rows + 1].abs().sum() == 0  # own halo rows untouched
    assert up[:, :8].abs().sum() == 0 and down[:, 1:].abs().sum() == 0
    u = torch.zeros(Fr, 2 * rows + 2, 2 * W, C, device="cuda", dtype=torch.bfloat16)
    up2 = torch.zeros(Fr, 6 + 2, 2 * W, C, device="cuda", dtype=torch.bfloat16)
    F.vae_upsample2x(x, u, halo=1, up=up2.data_ptr(), up_rows=6)
    ref_u = x.repeat_interleave(2, 1).repeat_interleave(2, 2)
    torch.cuda.synchronize()
    assert torch.equal(u[:, 1:2 * rows + 1], ref_u) and torch.equal(up2[:, 7], ref_u[:, 0])


def test_wan_vae_native_decoder_matches_reference(native):
    """The channels-last Wan VAE decoder on the native kernels (bf16) against the NCTHW
    PyTorch decoder in fp32 on the CPU, three latent frames (first-chunk and cached paths)."""
    from difflet_b200.models.vae.wan_vae import WanVAEConfig, WanVAEDecoder, WanVAEReference

    cfg = WanVAEConfig(base_dim=32)
    dec = WanVAEDecoder.random_init(cfg, device="cuda", dtype=torch.bfloat16, seed=4)
    z = torch.randn(1, 16, 3, 6, 20, generator=torch.Generator().manual_seed(1))
    out = dec.decode(z.cuda().bfloat16()).float().cpu()
    ref = WanVAEReference(cfg, {k: v.float().cpu() for k, v in dec.w.items()}).decode(z)
    assert out.shape == ref.shape == (1, 3, 9, 48, 160)
    assert ((out - ref).norm() / ref.norm()).item() < 3e-2
