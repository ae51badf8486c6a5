"""CPU oracle of the head scatter: two-segment placement and the linear_qkv fallback."""

import torch

from difflet_b200.ops import fused as F


def _kw(H, dh, S_src, S_dst, cos, sin):
    D = H * dh
    return dict(q_off=0, k_off=D, v_off=2 * D, S_src=S_src, H=H, dh=dh, S_dst=S_dst, norm_mode=1, eps=1e-6, cos=cos,
                sin=sin)


def test_two_segments_equal_two_calls():
    torch.manual_seed(0)
    B, S_src, H, dh, seg, S_dst = 2, 12, 2, 8, 5, 40
    qkv = torch.randn(B * S_src, 3 * H * dh, dtype=torch.float64)
    ang = torch.rand(S_dst, dh // 2, dtype=torch.float64)
    cos, sin = ang.cos(), ang.sin()
    a = [torch.zeros(B, H, S_dst, dh, dtype=torch.float64) for _ in range(3)]
    F.qkv_scatter(qkv, q_dst=[a[0]], k_dst=[a[1]], v_dst=[a[2]], seq_off=3, rope_pos_off=3, seg_rows=seg,
                  seg1_seq_off=25, seg1_rope_off=25, **_kw(H, dh, S_src, S_dst, cos, sin))
    r = [torch.zeros_like(t) for t in a]
    x3 = qkv.view(B, S_src, -1)
    F.qkv_scatter(x3[:, :seg].reshape(B * seg, -1), q_dst=[r[0]], k_dst=[r[1]], v_dst=[r[2]], seq_off=3,
                  rope_pos_off=3, **_kw(H, dh, seg, S_dst, cos, sin))
    F.qkv_scatter(x3[:, seg:].reshape(B * (S_src - seg), -1), q_dst=[r[0]], k_dst=[r[1]], v_dst=[r[2]], seq_off=25,
                  rope_pos_off=25, **_kw(H, dh, S_src - seg, S_dst, cos, sin))
    for t, u in zip(a, r):
        assert torch.equal(t, u)
    assert a[0][:, :, 3 + seg:25].abs().max() == 0


def test_linear_qkv_cpu_is_linear_then_scatter():
    torch.manual_seed(1)
    M, H, dh, Fm = 10, 2, 8, 16
    D = H * dh
    N = 3 * D + Fm
    x = torch.randn(M, 12, dtype=torch.float64)
    w = torch.randn(N, 12, dtype=torch.float64)
    b = torch.randn(N, dtype=torch.float64)
    ang = torch.rand(M, dh // 2, dtype=torch.float64)
    cos, sin = ang.cos(), ang.sin()
    kw = dict(q_off=0, k_off=D + Fm, v_off=2 * D + Fm, S_src=M, H=H, dh=dh, S_dst=M, norm_mode=1, eps=1e-6, cos=cos,
              sin=sin)
    a = [torch.zeros(1, H, M, dh, dtype=torch.float64) for _ in range(3)]
    out = torch.zeros(M, N, dtype=torch.float64)
    F.linear_qkv(x, w, b, out=out, act="gelu", act_lo=D, act_hi=D + Fm,
                 scatter=dict(kw, q_dst=[a[0]], k_dst=[a[1]], v_dst=[a[2]]))
    y = F.linear(x, w, b, act="gelu", act_lo=D, act_hi=D + Fm)
    r = [torch.zeros_like(t) for t in a]
    F.qkv_scatter(y, q_dst=[r[0]], k_dst=[r[1]], v_dst=[r[2]], **kw)
    assert torch.allclose(out[:, D:D + Fm], y[:, D:D + Fm])
    for t, u in zip(a, r):
        assert torch.allclose(t, u)
