"""The public op surface (difflet tests/unit/backends/test_neuron_attention_c3.py:45-362,
test_cpu_ops_impl.py): every exported name, the attention contract clauses, norms,
rotary laws, MX quantization, TP layers and the context-parallel ops on gloo ranks."""

import math

import pytest
import torch

import difflet_b200.ops as ops
from difflet_b200.parallel.testing import run_ranks


def test_every_export_resolves():
    for name in ops.__all__:
        assert getattr(ops, name) is not None, name
    with pytest.raises(AttributeError):
        ops.not_an_op  # noqa: B018


def _dense(q, k, v, scale, mask=None):
    s = torch.einsum("bhqd,bhkd->bhqk", q.double(), k.double()) * scale
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf")) if mask.dtype == torch.bool else s + mask.double()
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), v.double()), torch.logsumexp(s, -1)


def _qkv(B=2, H=3, Sq=17, Sk=23, D=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, H, Sq, D, generator=g), torch.randn(B, H, Sk, D, generator=g),
            torch.randn(B, H, Sk, D, generator=g))


def test_attention_scale_none_is_one_and_folded_layout():
    q, k, v = _qkv()
    ref, _ = _dense(q, k, v, 1.0)
    assert torch.allclose(ops.attention(q, k, v).double(), ref, atol=1e-5)
    out3 = ops.attention(q.flatten(0, 1), k.flatten(0, 1), v.flatten(0, 1), scale=0.5)
    ref3, _ = _dense(q, k, v, 0.5)
    assert out3.shape == (6, 17, 16)
    assert torch.allclose(out3.double(), ref3.flatten(0, 1), atol=1e-5)


def test_attention_masks_bounds_and_causal():
    q, k, v = _qkv()
    g = torch.Generator().manual_seed(3)
    bmask = torch.rand(2, 1, 17, 23, generator=g) > 0.3
    bmask[..., 0] = True
    ref, _ = _dense(q, k, v, 0.3, bmask)
    assert torch.allclose(ops.attention(q, k, v, scale=0.3, attention_mask=bmask).double(), ref, atol=1e-5)
    add = torch.randn(2, 1, 17, 23, generator=g)
    ref, _ = _dense(q, k, v, 0.3, add)
    assert torch.allclose(ops.attention(q, k, v, scale=0.3, attention_mask=add).double(), ref, atol=1e-5)
    # per-batch bounds (kernel window) and per-query bounds (mask path) agree with the mask law
    lo, hi = torch.tensor([2, 0]), torch.tensor([20, 9])
    idx = torch.arange(23)
    m = ((idx >= lo[:, None]) & (idx < hi[:, None]))[:, None, None, :]
    ref, _ = _dense(q, k, v, 0.3, m)
    assert torch.allclose(ops.attention(q, k, v, scale=0.3, bound_min=lo, bound_max=hi).double(), ref, atol=1e-5)
    lo_q = torch.randint(0, 5, (2, 1, 17, 1), generator=g)
    hi_q = lo_q + torch.randint(1, 15, (2, 1, 17, 1), generator=g)
    mq = (idx >= lo_q) & (idx < hi_q)
    ref, _ = _dense(q, k, v, 0.3, mq)
    assert torch.allclose(ops.attention(q, k, v, scale=0.3, bound_min=lo_q, bound_max=hi_q).double(), ref,
                          atol=1e-5)
    with pytest.raises(ValueError):
        ops.attention(q, k, v, bound_min=lo)
    with pytest.raises(ValueError):
        ops.attention(q, k, v, bound_min=lo, bound_max=hi, attention_mask=bmask)
    qq, kk, vv = _qkv(Sq=11, Sk=11)
    tri = torch.ones(11, 11, dtype=torch.bool).tril()
    ref, _ = _dense(qq, kk, vv, 0.3, tri)
    assert torch.allclose(ops.attention(qq, kk, vv, scale=0.3, causal=True).double(), ref, atol=1e-5)


def test_lse_and_merge_stable_at_large_logits():
    from difflet_b200.ops.attn import attention_with_lse, merge_partials

    q, k, v = _qkv()
    q = q * 40  # logsumexp far above exp's range
    ref, ref_lse = _dense(q, k, v, 1.0)
    o1, l1 = attention_with_lse(q, k[:, :, :10], v[:, :, :10], scale=1.0)
    o2, l2 = attention_with_lse(q, k[:, :, 10:], v[:, :, 10:], scale=1.0)
    assert torch.allclose(l1.double(), torch.logsumexp(torch.einsum("bhqd,bhkd->bhqk", q.double(),
                                                                    k[:, :, :10].double()), -1), atol=1e-3)
    o, lse = merge_partials(o1.float(), l1, o2.float(), l2)
    assert torch.allclose(o.double(), ref, atol=1e-4)
    assert torch.allclose(lse.double(), ref_lse, rtol=1e-5)
    # an empty partial weighs nothing
    o, lse = merge_partials(o1.float(), l1, torch.zeros_like(o1), torch.full_like(l1, float("-inf")))
    assert torch.equal(o, o1.float()) and torch.equal(lse, l1)


def test_cp_ops_at_cp1_are_dense():
    q, k, v = _qkv()
    ref = ops.attention(q, k, v, scale=0.2)
    assert torch.allclose(ops.ring_attention(q, k, v, scale=0.2), ref, atol=1e-6)
    assert torch.allclose(ops.ulysses_attention(q, k, v, scale=0.2), ref, atol=1e-6)
    tk, tv = k[:, :, :5], v[:, :, :5]
    out = ops.joint_ring_attention(q, k[:, :, 5:], v[:, :, 5:], tk, tv, scale=0.2)
    assert torch.allclose(out, ref, atol=1e-5)


def _cp_rank(rank, world):
    import torch.distributed as dist

    ops.init_parallel_mesh(cp=world)
    g = torch.Generator().manual_seed(5)
    B, H, S, D, T = 2, 4, 12 * world, 16, 6
    q, k, v = (torch.randn(B, H, S, D, generator=g, dtype=torch.float64) for _ in range(3))
    tq, tk, tv = (torch.randn(B, H, T, D, generator=g, dtype=torch.float64) for _ in range(3))
    n = S // world
    sh = slice(rank * n, (rank + 1) * n)
    errs = {}
    dense = ops.attention(q, k, v, scale=0.25)
    errs["ring"] = (ops.ring_attention(q[:, :, sh], k[:, :, sh], v[:, :, sh], scale=0.25) - dense[:, :, sh]).abs().max()
    errs["ulysses"] = (ops.ulysses_attention(q[:, :, sh], k[:, :, sh], v[:, :, sh], scale=0.25)
                       - dense[:, :, sh]).abs().max()
    # joint ring: queries [text ; image shard], image keys sharded, text replicated and padded
    valid = torch.tensor([4, 6])
    kj, vj = torch.cat([tk, k], 2), torch.cat([tv, v], 2)
    idx = torch.arange(T + S)
    keep = ((idx >= T) | (idx < valid[:, None]))[:, None, None, :]
    qj = torch.cat([tq, q[:, :, sh]], 2)
    dj = ops.attention(qj, kj, vj, scale=0.25, attention_mask=keep)
    out = ops.joint_ring_attention(qj, k[:, :, sh], v[:, :, sh], tk, tv, scale=0.25, text_valid_len=valid)
    errs["joint_ring"] = (out - dj).abs().max()
    # joint Ulysses: keys [image_full ; text] with a valid count
    kv_valid = torch.tensor([S + 3, S + T])
    kfull, vfull = torch.cat([k, tk], 2), torch.cat([v, tv], 2)
    idx = torch.arange(S + T)
    keep = (idx < kv_valid[:, None])[:, None, None, :]
    dfull = ops.attention(torch.cat([q, tq], 2), kfull, vfull, scale=0.25, attention_mask=keep)
    oi, ot = ops.joint_ulysses_attention(q[:, :, sh], tq, k[:, :, sh], v[:, :, sh], tk, tv, scale=0.25,
                                         key_valid_len=kv_valid)
    errs["joint_ulysses"] = max((oi - dfull[:, :, sh]).abs().max(), (ot - dfull[:, :, S:]).abs().max())
    dist.barrier()
    return {kk: float(vv) for kk, vv in errs.items()}


@pytest.mark.multirank
def test_cp_ops_on_gloo_ranks():
    for errs in run_ranks(_cp_rank, 2, timeout=240):
        assert max(errs.values()) < 1e-10, errs


def test_norms_and_rotary():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5, 64, generator=g)
    w = torch.randn(64, generator=g)
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    assert torch.allclose(ops.rms_norm_fp32(x, w, 1e-6), ref, atol=1e-6)
    n = ops.RMSNorm(64)
    with torch.no_grad():
        n.weight.copy_(w)
    assert torch.allclose(n(x), ref, atol=1e-6)
    ln = ops.LayerNorm(64)
    assert torch.allclose(ln(x), torch.nn.functional.layer_norm(x, (64,)), atol=1e-6)
    h = torch.randn(2, 3, 7, 16, generator=g)
    ang = torch.rand(7, 8, generator=g) * 6
    cos, sin = ang.cos().repeat_interleave(2, -1), ang.sin().repeat_interleave(2, -1)
    c = torch.view_as_complex(h.reshape(2, 3, 7, 8, 2).contiguous())
    ref = torch.view_as_real(c * torch.polar(torch.ones_like(ang), ang)).flatten(-2)
    assert torch.allclose(ops.apply_rotary_emb(h, cos, sin), ref, atol=1e-5)
    assert torch.allclose(ops.apply_rotary_emb_fp32(h, cos, sin), ref, atol=1e-5)
    assert torch.allclose(ops.apply_rotary_emb_slices(h, cos, sin), ref, atol=1e-5)
    a = torch.randn(3)
    assert ops.ModuleMarkerStartWrapper()(a) is a
    assert ops.ModuleMarkerEndWrapper()(a, a) == (a, a)
    assert ops.get_platform_target() in tuple(ops.hardware)


def test_mx_quantize_law_and_roundtrip():
    g = torch.Generator().manual_seed(2)
    x = (torch.randn(8, 128, generator=g) * torch.logspace(-3, 3, 8)[:, None]).bfloat16()
    x[3, 32:64] = 0
    data, scale = ops.quantize_mx(x)
    assert data.dtype == torch.float8_e4m3fn and scale.shape == (8, 4) and scale.dtype == torch.uint8
    amax = x.float().reshape(8, 4, 32).abs().amax(-1)
    nz = amax > 0
    e = scale.int() - 127
    assert torch.equal(e[nz], torch.floor(torch.log2(amax[nz])).int() - 8)  # largest binade - emax(E4M3)
    assert int(scale[3, 1]) == 0  # all-zero block
    back = ops.dequantize_mx(data, scale, output_dtype=torch.float32)
    err = (back - x.float()).abs().reshape(8, 4, 32).amax(-1)
    assert torch.all(err <= amax * 2.0 ** -3 + 1e-30)  # 3 mantissa bits
    assert torch.equal(back[3, 32:64], torch.zeros(32))
    # the reference's Trainium name is an alias
    d2, s2 = ops.quantize_mx(x, dtype="float8_e4m3fn_x4")
    assert torch.equal(s2, scale)


def test_mx_matmul_and_linear():
    g = torch.Generator().manual_seed(3)
    a = torch.randn(16, 96, generator=g).bfloat16()
    w = torch.randn(24, 96, generator=g).bfloat16()
    aq, as_ = ops.quantize_mx(a)
    wq, ws = ops.quantize_mx(w)
    y = ops.matmul_mx(aq, as_, wq, ws, out_dtype=torch.float32)
    ref = ops.dequantize_mx(aq, as_, output_dtype=torch.float32) @ ops.dequantize_mx(wq, ws,
                                                                                     output_dtype=torch.float32).t()
    assert torch.allclose(y, ref, atol=1e-4)
    lin = ops.linear_mx(a, w.t().contiguous(), None, out_dtype=torch.float32)
    full = a.float() @ w.float().t()
    assert ((lin - full).norm() / full.norm()).item() < 0.05


def test_tp_layers_at_tp1():
    g = torch.Generator().manual_seed(4)
    x = torch.randn(3, 5, 32, generator=g)
    col = ops.ColumnParallelLinear(32, 48)
    row = ops.RowParallelLinear(48, 16, skip_bias_add=True)
    y = col(x)
    assert torch.allclose(y, torch.nn.functional.linear(x, col.weight, col.bias), atol=1e-6)
    z, b = row(y)
    assert b is row.bias and torch.allclose(z, y @ row.weight.t(), atol=1e-5)
    emb = ops.ParallelEmbedding(10, 8)
    ids = torch.tensor([[1, 9]])
    assert torch.equal(emb(ids), emb.weight[ids])


def _tp_rank(rank, world):
    ops.init_parallel_mesh(tp=world)
    torch.manual_seed(0)  # same full weights on every rank
    W1, b1 = torch.randn(48, 32, dtype=torch.float64), torch.randn(48, dtype=torch.float64)
    W2, b2 = torch.randn(16, 48, dtype=torch.float64), torch.randn(16, dtype=torch.float64)
    x = torch.randn(4, 6, 32, dtype=torch.float64)
    ref = torch.nn.functional.linear(torch.nn.functional.linear(x, W1, b1), W2, b2)
    col = ops.ColumnParallelLinear(32, 48, gather_output=False, dtype=torch.float64)
    row = ops.RowParallelLinear(48, 16, input_is_parallel=True, dtype=torch.float64)
    n1, n2 = 48 // world, 48 // world
    with torch.no_grad():
        col.weight.copy_(W1[rank * n1:(rank + 1) * n1])
        col.bias.copy_(b1[rank * n1:(rank + 1) * n1])
        row.weight.copy_(W2[:, rank * n2:(rank + 1) * n2])
        row.bias.copy_(b2)
    out = row(col(x))
    # Megatron-SP: sequence-sharded in, reduce-scattered out (sequence dim 1)
    s = 6 // world
    col_sp = ops.ColumnParallelLinear(32, 48, gather_output=False, dtype=torch.float64,
                                      sequence_parallel_enabled=True, sequence_dimension=1)
    row_sp = ops.RowParallelLinear(48, 16, input_is_parallel=True, dtype=torch.float64,
                                   sequence_parallel_enabled=True, sequence_dimension=1)
    with torch.no_grad():
        col_sp.weight.copy_(col.weight)
        col_sp.bias.copy_(col.bias)
        row_sp.weight.copy_(row.weight)
        row_sp.bias.copy_(row.bias)
    out_sp = row_sp(col_sp(ops.scatter_to_sequence_parallel_region(x, dim=1)))
    emb = ops.ParallelEmbedding(10, 8, dtype=torch.float64)
    full = torch.randn(10, 8, dtype=torch.float64)
    with torch.no_grad():
        emb.weight.copy_(full[rank * 5:(rank + 1) * 5])
    ids = torch.tensor([[0, 9, 4, 5]])
    return (float((out - ref).abs().max()), float((out_sp - ref[:, rank * s:(rank + 1) * s]).abs().max()),
            float((emb(ids) - full[ids]).abs().max()))


@pytest.mark.multirank
def test_tp_layers_on_gloo_ranks():
    for errs in run_ranks(_tp_rank, 2, timeout=240):
        assert max(errs) < 1e-10, errs
