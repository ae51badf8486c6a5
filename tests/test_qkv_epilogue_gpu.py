"""The qkv GEMM epilogue (per-head q/k RMSNorm + RoPE + head scatter straight from the
tensor-memory accumulator) against the unfused path (GEMM stored, then the standalone
scatter kernel) and against the fp32 CPU oracle."""

import pytest
import torch

from difflet_b200.ops import fused as F

pytestmark = pytest.mark.gpu


def _close(out, ref, tol=2e-2):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale, f"max abs err {err:.4g} vs scale {scale:.4g}"


def _tables(S, width, device="cuda"):
    ang = torch.rand(S, width, device=device) * 6
    return ang.cos().contiguous(), ang.sin().contiguous()


def _run(monkeypatch, fuse, x, w, b, scatter_fn, out_shape=None, **kw):
    """One linear_qkv call into fresh zeroed destinations; returns (dst tensors, out)."""
    monkeypatch.setenv("DIFFLET_FUSE_QKV", "1" if fuse else "0")
    dsts, sc = scatter_fn()
    out = None if out_shape is None else torch.zeros(out_shape, device=x.device, dtype=torch.bfloat16)
    if not fuse and out is None:
        out = torch.zeros(x.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
    F.linear_qkv(x, w, b, scatter=sc, out=out, **kw)
    torch.cuda.synchronize()
    return dsts, out


@pytest.mark.parametrize("M,H,cta_mode", [(300, 4, "one"), (1100, 4, "pair"), (200, 2, "narrow")])
def test_qkv_epilogue_matches_unfused(native, monkeypatch, M, H, cta_mode):
    torch.manual_seed(11)
    dh, S_dst, off = 128, M + 16, 16
    D = H * dh
    x = torch.randn(M, 256, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3 * D, 256, device="cuda", dtype=torch.bfloat16) * 0.06
    b = torch.randn(3 * D, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    cos, sin = _tables(S_dst, dh // 2)

    def scatter():
        q, k, v = (torch.zeros(1, H, S_dst, dh, device="cuda", dtype=torch.bfloat16) for _ in range(3))
        return (q, k, v), dict(q_off=0, k_off=D, v_off=2 * D, S_src=M, H=H, dh=dh, q_dst=[q], k_dst=[k], v_dst=[v],
                               S_dst=S_dst, seq_off=off, norm_mode=1, wq=wq, wk=wk, eps=1e-6, cos=cos, sin=sin,
                               rope_pos_off=off)

    fused, _ = _run(monkeypatch, True, x, w, b, scatter)
    ref, _ = _run(monkeypatch, False, x, w, b, scatter)
    for a, r in zip(fused, ref):
        _close(a, r, 1e-2)
        assert a[:, :, :off].abs().max().item() == 0
    # and against the fp32 CPU oracle
    qc, kc, vc = (torch.zeros(1, H, S_dst, dh) for _ in range(3))
    F.linear_qkv(x.cpu().float(), w.cpu().float(), b.cpu().float(),
                 scatter=dict(q_off=0, k_off=D, v_off=2 * D, S_src=M, H=H, dh=dh, q_dst=[qc], k_dst=[kc], v_dst=[vc],
                              S_dst=S_dst, seq_off=off, norm_mode=1, wq=wq.cpu().float(), wk=wk.cpu().float(),
                              eps=1e-6, cos=cos.cpu(), sin=sin.cpu(), rope_pos_off=off))
    for a, r in zip(fused, (qc, kc, vc)):
        _close(a, r.cuda())


def test_qkv_epilogue_single_block_layout(native, monkeypatch):
    """[q | mlp | k | v] projection: GELU columns land in `out`, q/k/v are scattered."""
    torch.manual_seed(12)
    M, H, dh, Fm = 520, 4, 128, 1024
    D = H * dh
    N = 3 * D + Fm
    x = torch.randn(M, 192, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, 192, device="cuda", dtype=torch.bfloat16) * 0.07
    b = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    cos, sin = _tables(M, dh // 2)

    def scatter():
        q, k, v = (torch.zeros(1, H, M, dh, device="cuda", dtype=torch.bfloat16) for _ in range(3))
        return (q, k, v), dict(q_off=0, k_off=D + Fm, v_off=2 * D + Fm, S_src=M, H=H, dh=dh, q_dst=[q], k_dst=[k],
                               v_dst=[v], S_dst=M, norm_mode=1, wq=wq, wk=wk, eps=1e-6, cos=cos, sin=sin)

    kw = dict(act="gelu", act_lo=D, act_hi=D + Fm)
    fused, out_f = _run(monkeypatch, True, x, w, b, scatter, out_shape=(M, N), **kw)
    ref, out_r = _run(monkeypatch, False, x, w, b, scatter, out_shape=(M, N), **kw)
    for a, r in zip(fused, ref):
        _close(a, r, 1e-2)
    _close(out_f[:, D:D + Fm], out_r[:, D:D + Fm], 1e-2)
    assert out_f[:, :D].abs().max().item() == 0  # the q slot is left for the attention output


def test_qkv_epilogue_half_rope_dh64_token_major_two_ranks_segments(native, monkeypatch):
    """dh 64, half-split RoPE, no norm / bias, token-major destinations split over two
    'ranks' (heads_per_rank), two row segments per batch, batch 2."""
    torch.manual_seed(13)
    B, S_src, H, dh = 2, 96, 4, 64
    D = H * dh
    seg, S_dst = 40, 300
    seq0, seq1 = 10, 150
    x = torch.randn(B * S_src, 128, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3 * D, 128, device="cuda", dtype=torch.bfloat16) * 0.08
    cos, sin = _tables(S_dst, dh // 2)

    def scatter():
        bufs = [torch.zeros(B, S_dst, (H // 2) * dh, device="cuda", dtype=torch.bfloat16) for _ in range(6)]
        return bufs, dict(q_off=0, k_off=D, v_off=2 * D, S_src=S_src, H=H, dh=dh, q_dst=bufs[0:2], k_dst=bufs[2:4],
                          v_dst=bufs[4:6], S_dst=S_dst, seq_off=seq0, norm_mode=0, cos=cos, sin=sin, rope_half=True,
                          rope_pos_off=seq0, heads_per_rank=H // 2, token_major=True, seg_rows=seg,
                          seg1_seq_off=seq1, seg1_rope_off=seq1)

    fused, _ = _run(monkeypatch, True, x, w, None, scatter)
    ref, _ = _run(monkeypatch, False, x, w, None, scatter)
    for a, r in zip(fused, ref):
        _close(a, r, 1e-2)
    assert fused[0][:, seq0 + seg:seq1].abs().max().item() == 0  # the gap between the segments stays empty


def test_qkv_epilogue_kv_replicate_per_head_tables(native, monkeypatch):
    """Gather-KV placement (k / v to every rank, q local) with per-head RoPE tables."""
    torch.manual_seed(14)
    M, H, dh = 130, 4, 128
    D = H * dh
    S_loc, row, S_all, pos = 160, 20, 400, 200
    x = torch.randn(M, 128, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3 * D, 128, device="cuda", dtype=torch.bfloat16) * 0.08
    b = torch.randn(3 * D, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    cos, sin = _tables(S_all, H * dh // 2)

    def scatter():
        q = torch.zeros(1, H, S_loc, dh, device="cuda", dtype=torch.bfloat16)
        ks = [torch.zeros(1, H, S_all, dh, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
        vs = [torch.zeros_like(ks[0]) for _ in range(3)]
        return [q] + ks + vs, dict(q_off=0, k_off=D, v_off=2 * D, S_src=M, H=H, dh=dh, q_dst=[q, None, None],
                                   k_dst=ks, v_dst=vs, S_dst=S_all, seq_off=pos, norm_mode=1, wq=wq, wk=wk, eps=1e-6,
                                   cos=cos, sin=sin, rope_pos_off=pos, kv_replicate=True, q_S_dst=S_loc,
                                   q_seq_off=row)

    fused, _ = _run(monkeypatch, True, x, w, b, scatter)
    ref, _ = _run(monkeypatch, False, x, w, b, scatter)
    for a, r in zip(fused, ref):
        _close(a, r, 1e-2)


def test_qkv_epilogue_mxfp8(native, monkeypatch):
    """The block-scaled MXFP8 GEMM takes the same epilogue."""
    torch.manual_seed(15)
    M, H, dh = 384, 4, 128
    D = H * dh
    x = torch.randn(M, 256, device="cuda", dtype=torch.bfloat16)
    w = F.MXWeight.quantize(torch.randn(3 * D, 256, device="cuda", dtype=torch.bfloat16) * 0.06)
    b = torch.randn(3 * D, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    cos, sin = _tables(M, dh // 2)

    def scatter():
        q, k, v = (torch.zeros(1, H, M, dh, device="cuda", dtype=torch.bfloat16) for _ in range(3))
        return (q, k, v), dict(q_off=0, k_off=D, v_off=2 * D, S_src=M, H=H, dh=dh, q_dst=[q], k_dst=[k], v_dst=[v],
                               S_dst=M, norm_mode=1, wq=wq, wk=wk, eps=1e-6, cos=cos, sin=sin)

    fused, _ = _run(monkeypatch, True, x, w, b, scatter)
    ref, _ = _run(monkeypatch, False, x, w, b, scatter)
    for a, r in zip(fused, ref):
        _close(a, r, 1e-2)


@pytest.mark.parametrize("epi", ["gate", "gelu", "qkv"])
def test_grouped_gemm_matches_separate(native, monkeypatch, epi):
    """Two problems (4096-row image stream + 512-row text stream shapes, scaled down) in one
    grouped launch equal two separate launches."""
    torch.manual_seed(16)
    H, dh = 4, 128
    D = H * dh
    shapes = [(1100, 256), (300, 256)]  # (rows, K): pair tiles for the first, shared by the second

    def problem(M, K):
        N = 3 * D if epi == "qkv" else (1536 if epi == "gelu" else D)
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.06
        b = torch.randn(N, device="cuda", dtype=torch.bfloat16)
        return x, w, b

    probs = [problem(M, K) for M, K in shapes]
    gates = [torch.randn(1, D, device="cuda") for _ in probs]
    resid0 = [torch.randn(M, D, device="cuda", dtype=torch.bfloat16) for M, _ in shapes]
    wq = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn(dh, device="cuda", dtype=torch.bfloat16)
    cos, sin = _tables(2000, dh // 2)

    def calls():
        out, dsts = [], []
        for (x, w, b), (M, _), g, r0 in zip(probs, shapes, gates, resid0):
            c = dict(x=x, w=w, b=b)
            if epi == "gate":
                o = r0.clone()
                c.update(out=o, gate=g, resid=o, rows_per_batch=M)
            elif epi == "gelu":
                o = torch.zeros(M, w.shape[0], device="cuda", dtype=torch.bfloat16)
                c.update(out=o, act="gelu")
            else:
                o = torch.zeros(M, w.shape[0], device="cuda", dtype=torch.bfloat16)
                qd, kd, vd = (torch.zeros(1, H, M, dh, device="cuda", dtype=torch.bfloat16) for _ in range(3))
                dsts += [qd, kd, vd]
                c.update(out=o, scatter=dict(q_off=0, k_off=D, v_off=2 * D, S_src=M, H=H, dh=dh, q_dst=[qd],
                                             k_dst=[kd], v_dst=[vd], S_dst=M, norm_mode=1, wq=wq, wk=wk, eps=1e-6,
                                             cos=cos, sin=sin))
            out.append(o)
            out_calls.append(c)
        return out, dsts

    monkeypatch.setenv("DIFFLET_GEMM_GROUP", "1")
    out_calls = []
    got, got_d = calls()
    before = F.LAUNCHES[0]
    F.linear_group(out_calls)
    assert F.LAUNCHES[0] - before == 1
    torch.cuda.synchronize()
    monkeypatch.setenv("DIFFLET_GEMM_GROUP", "0")
    out_calls = []
    ref, ref_d = calls()
    F.linear_group(out_calls)
    torch.cuda.synchronize()
    for a, r in zip(got + got_d, ref + ref_d):
        if epi == "qkv" and a.dim() == 2:
            continue  # the qkv columns of `out` are not written by the fused path
        _close(a, r, 1e-2)  # the small problem runs on the large one's tile shape when grouped
