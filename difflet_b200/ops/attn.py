"""Public attention ops for model code (the reference's ``difflet.ops`` attention surface).

Contract (difflet/ops/attention.py:4-128, difflet/backends/cuda/ops_impl/attention.py:1-17):

* ``q, k, v``: ``[B, H, S, D]`` or ``[B*H, S, D]``; the result has ``q``'s shape.
* ``scale=None`` means 1.0 (not ``1/sqrt(D)``).
* ``attention_mask``: bool (True = attend) or additive; ``bound_min`` / ``bound_max``
  (both or neither, exclusive with a mask) select the keys ``[bound_min, bound_max)``.
* ``tp_q`` / ``tp_k`` / ``tp_out`` are layout hints of other hardware: accepted, ignored.

Dispatch: CUDA tensors with head dim 128, no mask, non-causal and bounds that are
per batch row (shape ``[B]`` or ``[B, 1, ...]``, the padded-text key windows every
model here uses) run the tcgen05 kernel (``csrc/attention.cu``).  Anything else on
CUDA (arbitrary masks, causal, other head dims, per-query windows) is the library
path: ``torch.nn.functional.scaled_dot_product_attention``.  CPU tensors run the
fp32 / fp64 oracle of ``ops.fused``.

Context-parallel ops (``ring_attention``, ``joint_ring_attention``,
``ulysses_attention``, ``joint_ulysses_attention``) run over the cp group of the
mesh (``parallel.groups``) with ``torch.distributed`` transfers; the built-in models
use the fused peer-memory transports of ``parallel.ulysses`` / ``parallel.ring``
instead.  Semantics: difflet/backends/neuron/ops_impl/attention.py:435-713.
"""

from __future__ import annotations

import torch
import torch.nn.functional as TF

from difflet_b200.ops import fused as F


def _bounds_to_mask(k, bound_min, bound_max, attention_mask):
    if bound_min is None and bound_max is None:
        return attention_mask
    if bound_min is None or bound_max is None:
        raise ValueError("bound_min and bound_max must both be provided")
    if attention_mask is not None:
        raise ValueError("attention_mask and bounds are mutually exclusive")
    idx = torch.arange(k.shape[-2], device=k.device)
    return (idx >= bound_min.to(k.device)) & (idx < bound_max.to(k.device))


def _per_batch(bound, B):
    """A [B] int32 window edge when ``bound`` does not vary over queries, else None."""
    if bound is None:
        return None
    b = torch.as_tensor(bound)
    if b.dim() == 0:
        b = b.expand(B)
    elif b.shape[0] == B and all(s == 1 for s in b.shape[1:]):
        b = b.reshape(B)
    else:
        return None
    return b


def attention(q, k, v, *, scale=None, causal=False, attention_mask=None, bound_min=None, bound_max=None,
              tp_q=False, tp_k=False, tp_out=False, lse=None, **kwargs):
    del tp_q, tp_k, tp_out, kwargs
    scale = 1.0 if scale is None else float(scale)
    folded = q.dim() == 3
    q4, k4, v4 = (t.unsqueeze(0) for t in (q, k, v)) if folded else (q, k, v)
    B = q4.shape[0]
    if (bound_min is None) != (bound_max is None):
        raise ValueError("bound_min and bound_max must both be provided")
    if attention_mask is not None and bound_min is not None:
        raise ValueError("attention_mask and bounds are mutually exclusive")
    lo, hi = _per_batch(bound_min, B), _per_batch(bound_max, B)
    simple = attention_mask is None and not causal and (bound_min is None or (lo is not None and hi is not None))
    kernel = q.is_cuda and simple and q.shape[-1] == 128 and q.dtype == torch.bfloat16
    if kernel or (simple and not q.is_cuda):
        if lo is not None:
            lo = lo.to(q.device, torch.int32 if q.is_cuda else torch.int64).contiguous()
            hi = hi.to(q.device, torch.int32 if q.is_cuda else torch.int64).contiguous()
        out = F.attention(q4, k4, v4, scale, lse=lse, kv_lo=lo, kv_hi=hi)
    else:
        mask = _bounds_to_mask(k4, bound_min, bound_max, attention_mask)
        if lse is not None or not q.is_cuda:  # math path (oracle, or LSE requested off the kernel)
            out = _oracle_masked(q4, k4, v4, scale, causal, mask, lse)
        else:
            out = _sdpa(q4, k4, v4, scale, causal, mask)
    return out.squeeze(0) if folded else out


def _sdpa(q, k, v, scale, causal, mask):
    if mask is None:
        return TF.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale)
    Lq, Lk = q.shape[-2], k.shape[-2]
    if mask.dtype == torch.bool:
        m = mask.to(q.device)
        if causal:
            m = m & torch.ones(Lq, Lk, dtype=torch.bool, device=q.device).tril()
        return TF.scaled_dot_product_attention(q, k, v, attn_mask=m, scale=scale)
    add = mask.to(device=q.device, dtype=q.dtype)
    if causal:
        tri = torch.ones(Lq, Lk, dtype=torch.bool, device=q.device).tril()
        add = add.masked_fill(~tri, torch.finfo(q.dtype).min)
    return TF.scaled_dot_product_attention(q, k, v, attn_mask=add, scale=scale)


def _oracle_masked(q, k, v, scale, causal, mask, lse=None):
    ct = torch.float64 if q.dtype == torch.float64 else torch.float32
    s = torch.einsum("bhqd,bhkd->bhqk", q.to(ct), k.to(ct)) * scale
    if mask is not None:
        if mask.dtype == torch.bool:
            s = s.masked_fill(~mask.to(s.device), float("-inf"))
        else:
            s = s + mask.to(device=s.device, dtype=ct)
    if causal:
        tri = torch.ones(s.shape[-2], s.shape[-1], dtype=torch.bool, device=s.device).tril()
        s = s.masked_fill(~tri, float("-inf"))
    if lse is not None:
        lse.copy_(torch.logsumexp(s, -1).to(lse.dtype).reshape(lse.shape))
    p = torch.nan_to_num(torch.softmax(s, -1), nan=0.0)
    return torch.einsum("bhqk,bhkd->bhqd", p, v.to(ct)).to(q.dtype)


def cross_attention(q, k, v, *, scale=None, attention_mask=None, **kwargs):
    for key in ("tp_q", "tp_k", "tp_out", "causal"):
        kwargs.pop(key, None)
    return attention(q, k, v, scale=scale, causal=False, attention_mask=attention_mask, **kwargs)


def attention_with_lse(q, k, v, *, scale, bound_min=None, bound_max=None):
    """(out, lse) of one key block: lse fp32 [B, H, Sq] (natural log)."""
    lse = torch.empty(q.shape[:-1], device=q.device, dtype=torch.float64 if q.dtype == torch.float64
                      else torch.float32)
    out = attention(q, k, v, scale=scale, bound_min=bound_min, bound_max=bound_max, lse=lse)
    return out, lse


def merge_partials(out, lse, o_r, l_r):
    """Log-sum-exp merge of two partial attentions (max-subtracted; empty partials weigh 0)."""
    m = torch.maximum(lse, l_r)
    safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w, w_r = torch.exp(lse - safe), torch.exp(l_r - safe)
    tot = w + w_r
    den = torch.where(tot > 0, tot, torch.ones_like(tot))
    merged = (out * w.unsqueeze(-1) + o_r * w_r.unsqueeze(-1)) / den.unsqueeze(-1)
    return merged, torch.where(tot > 0, safe + torch.log(den), torch.full_like(tot, float("-inf")))


# ----------------------------------------------------------------------------- context parallel
def _cp():
    import torch.distributed as dist

    from difflet_b200.parallel import groups

    ranks = groups.get_group_ranks("cp")
    if not dist.is_initialized() or len(ranks) == 1:
        return None, 1, 0
    return groups.get_group("cp"), len(ranks), ranks.index(dist.get_rank())


def _ring_partials(q, k, v, scale, group, cp, rank, out=None, lse=None):
    import torch.distributed as dist

    from difflet_b200.parallel import groups

    ranks = groups.get_group_ranks("cp")
    kv = torch.stack([k, v]).contiguous()
    nxt = torch.empty_like(kv)
    for step in range(cp):
        reqs = []
        if step < cp - 1:
            ops = [dist.P2POp(dist.isend, kv, ranks[(rank + 1) % cp], group=group),
                   dist.P2POp(dist.irecv, nxt, ranks[(rank - 1) % cp], group=group)]
            reqs = dist.batch_isend_irecv(ops)
        o_r, l_r = attention_with_lse(q, kv[0], kv[1], scale=scale)
        o_r = o_r.to(l_r.dtype)
        out, lse = (o_r, l_r) if out is None else merge_partials(out, lse, o_r, l_r)
        for r in reqs:
            r.wait()
        kv, nxt = nxt, kv
    return out, lse


def ring_attention(q, k, v, *, scale, causal=False):
    """q, k, v ``[B, H, S/cp, D]`` sequence-sharded over cp -> ``[B, H, S/cp, D]``."""
    if causal:
        raise NotImplementedError("ring_attention supports non-causal attention only")
    group, cp, rank = _cp()
    if cp == 1:
        return attention(q, k, v, scale=scale)
    out, _ = _ring_partials(q, k, v, scale, group, cp, rank)
    return out.to(q.dtype)


def joint_ring_attention(q, image_k, image_v, text_k, text_v, *, scale, causal=False, text_valid_len=None):
    """Image K/V sharded over cp, text K/V replicated: the text partial (masked past
    ``text_valid_len``) seeds the ring over the image blocks."""
    if causal:
        raise NotImplementedError("joint_ring_attention supports non-causal attention only")
    B = q.shape[0]
    lo = hi = None
    if text_valid_len is not None:
        lo = torch.zeros(B, dtype=torch.int32, device=q.device)
        hi = torch.as_tensor(text_valid_len).to(device=q.device, dtype=torch.int32)
    o_t, l_t = attention_with_lse(q, text_k, text_v, scale=scale, bound_min=lo, bound_max=hi)
    o_t = o_t.to(l_t.dtype)
    group, cp, rank = _cp()
    if cp == 1:
        o_i, l_i = attention_with_lse(q, image_k, image_v, scale=scale)
        out, _ = merge_partials(o_t, l_t, o_i.to(l_i.dtype), l_i)
        return out.to(q.dtype)
    out, _ = _ring_partials(q, image_k, image_v, scale, group, cp, rank, out=o_t, lse=l_t)
    return out.to(q.dtype)


def _a2a_heads_to_seq(x, group, cp):
    """[B, H, S/cp, D] sharded by sequence -> [B, H/cp, S, D] (full sequence, fewer heads)."""
    from difflet_b200.parallel.ulysses import all_to_all

    B, H, s, D = x.shape
    send = x.reshape(B, cp, H // cp, s, D).transpose(0, 1).contiguous()  # [cp, B, H/cp, s, D]
    recv = torch.empty_like(send)
    all_to_all(list(recv.unbind(0)), list(send.unbind(0)), group)
    return recv.permute(1, 2, 0, 3, 4).reshape(B, H // cp, cp * s, D)


def _a2a_seq_to_heads(x, group, cp):
    """[B, H/cp, S, D] -> [B, H, S/cp, D]."""
    from difflet_b200.parallel.ulysses import all_to_all

    B, h, S, D = x.shape
    s = S // cp
    send = x.reshape(B, h, cp, s, D).permute(2, 0, 1, 3, 4).contiguous()  # [cp, B, h, s, D]
    recv = torch.empty_like(send)
    all_to_all(list(recv.unbind(0)), list(send.unbind(0)), group)
    return recv.transpose(0, 1).reshape(B, cp * h, s, D)


def ulysses_attention(q, k, v, *, scale, causal=False):
    """q, k, v ``[B, H_local, S/cp, D]``; needs ``H_local % cp == 0``."""
    group, cp, _ = _cp()
    if cp == 1:
        return attention(q, k, v, scale=scale, causal=causal)
    if q.shape[1] % cp:
        raise ValueError(f"ulysses_attention needs heads % cp == 0, got {q.shape[1]} heads, cp={cp}")
    qf, kf, vf = (_a2a_heads_to_seq(t, group, cp) for t in (q, k, v))
    return _a2a_seq_to_heads(attention(qf, kf, vf, scale=scale, causal=causal), group, cp)


def joint_ulysses_attention(q_img, q_txt, image_k, image_v, text_k, text_v, *, scale, causal=False,
                            key_valid_len=None):
    """Image sharded over cp, text replicated; keys in ``[image_full ; text]`` order with an
    optional per-batch valid count.  Returns ``(img_out [B, H, S_img/cp, D], txt_out [B, H, S_txt, D])``."""
    import torch.distributed as dist

    if causal:
        raise NotImplementedError("joint_ulysses_attention supports non-causal attention only")
    group, cp, rank = _cp()
    B, H = q_img.shape[:2]
    if cp > 1 and H % cp:
        raise ValueError(f"joint_ulysses_attention needs heads % cp == 0, got {H} heads, cp={cp}")
    h = H // cp
    hs = slice(rank * h, (rank + 1) * h)
    if cp > 1:
        qi, ki, vi = (_a2a_heads_to_seq(t, group, cp) for t in (q_img, image_k, image_v))
    else:
        qi, ki, vi = q_img, image_k, image_v
    S_img = qi.shape[2]
    qj = torch.cat([qi, q_txt[:, hs]], 2)
    kj = torch.cat([ki, text_k[:, hs]], 2)
    vj = torch.cat([vi, text_v[:, hs]], 2)
    lo = hi = None
    if key_valid_len is not None:
        hi = torch.as_tensor(key_valid_len).to(device=q_img.device, dtype=torch.int32)
        lo = torch.zeros_like(hi)
    oj = attention(qj, kj, vj, scale=scale, bound_min=lo, bound_max=hi)
    o_img, o_txt = oj[:, :, :S_img], oj[:, :, S_img:]
    if cp == 1:
        return o_img.contiguous(), o_txt.contiguous()
    img_out = _a2a_seq_to_heads(o_img.contiguous(), group, cp)
    parts = [torch.empty_like(o_txt.contiguous()) for _ in range(cp)]
    dist.all_gather(parts, o_txt.contiguous(), group=group)
    return img_out, torch.cat(parts, 1)


__all__ = ["attention", "cross_attention", "ring_attention", "joint_ring_attention", "ulysses_attention",
           "joint_ulysses_attention", "attention_with_lse", "merge_partials"]
