"""Flash attention at video sequence lengths against an fp32 PyTorch reference.

Wan 2.x at 720p x 81 frames is 75,600 tokens per sequence and HunyuanVideo at 720p x 129
frames about 119k; the softmax runs in fp32 with a lazily rescaled running max, so these
lengths check that the running sums, the key-tile loop and the 64-bit row addressing stay
exact where the key count is largest.  The reference is computed in query chunks (fp32
scores, exact softmax)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_rows(q, k, v, scale, rows):
    """fp32 softmax(q k^T * scale) v for the query rows ``rows`` of each head ([B, H, R, D])."""
    qs = q[:, :, rows].float()
    s = torch.einsum("bhqd,bhkd->bhqk", qs, k.float()) * scale
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), v.float())


@pytest.mark.parametrize("S,H,n_blocks", [(75600, 2, 6), (119040, 1, 4)])
def test_attention_video_lengths(native, S, H, n_blocks):
    torch.manual_seed(31)
    q = torch.randn(1, H, S, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, H, S, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1, H, S, 128, device="cuda", dtype=torch.bfloat16)
    scale = 1 / math.sqrt(128)
    o = native.attention(q, k, v, scale)
    # query blocks spread over the sequence, the last one ending at the ragged tail
    starts = [int(i * (S - 512) / (n_blocks - 1)) for i in range(n_blocks)]
    for s0 in starts:
        rows = torch.arange(s0, s0 + 512, device="cuda")
        ref = _ref_rows(q, k, v, scale, rows)
        got = o[:, :, rows].float()
        err = (got - ref).abs().max().item()
        assert err <= 2e-2 * (ref.abs().max().item() + 1e-6), (S, s0, err)
    torch.cuda.synchronize()
    assert native.error_word(torch.cuda.current_device()).cpu().tolist() == [0, 0, 0, 0]
