"""``torch.ops.difflet.*``: dispatcher registration, fake (meta) kernels and agreement with
the PyTorch fp32 references of the same ops (CPU oracle; the CUDA path under ``-m gpu``)."""

import pytest
import torch

from difflet_b200.ops import library as L  # noqa: F401  (registers the ops)


def _inputs(dev, dtype=torch.float32):
    g = torch.Generator().manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=g).to(dev, dtype)  # noqa: E731
    return r


def _ref_attention(q, k, v, scale):
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    return torch.softmax(s, -1) @ v.float()


@pytest.mark.parametrize("name", L.OPS)
def test_registered(name):
    assert hasattr(torch.ops.difflet, name)


def test_cpu_values_and_opcheck():
    r = _inputs("cpu")
    q, k, v = r(1, 2, 16, 32), r(1, 2, 24, 32), r(1, 2, 24, 32)
    o = torch.ops.difflet.attention(q, k, v, 0.2)
    torch.testing.assert_close(o, _ref_attention(q, k, v, 0.2), atol=1e-5, rtol=1e-5)
    torch.library.opcheck(torch.ops.difflet.attention.default, (q, k, v, 0.2),
                          test_utils=("test_schema", "test_faketensor"))

    x, w, b = r(5, 64), r(96, 64), r(96)
    y = torch.ops.difflet.linear(x, w, b, "gelu", 32, 96)
    ref = x @ w.t() + b
    ref[:, 32:96] = torch.nn.functional.gelu(ref[:, 32:96], approximate="tanh")
    torch.testing.assert_close(y, ref, atol=1e-5, rtol=1e-5)
    torch.library.opcheck(torch.ops.difflet.linear.default, (x, w, b, "silu", 0, -1),
                          test_utils=("test_schema", "test_faketensor"))

    gate, resid = r(1, 96), r(5, 96)
    y = torch.ops.difflet.linear_gate_resid(x, w, b, gate, resid, 0)
    torch.testing.assert_close(y, resid + gate * (x @ w.t() + b), atol=1e-5, rtol=1e-5)

    xs = r(2, 6, 64)
    sh, sc = r(2, 64), r(2, 64)
    y = torch.ops.difflet.ln_modulate(xs.reshape(12, 64), sh, sc, None, None, 1e-6, False, 6)
    ln = torch.nn.functional.layer_norm(xs, (64,), eps=1e-6)
    torch.testing.assert_close(y.reshape(2, 6, 64), ln * (1 + sc[:, None]) + sh[:, None], atol=1e-5, rtol=1e-5)
    torch.library.opcheck(torch.ops.difflet.ln_modulate.default, (xs.reshape(12, 64), sh, sc, None, None, 1e-6, True, 6),
                          test_utils=("test_schema", "test_faketensor"))

    wn = r(64)
    y = torch.ops.difflet.rms_norm(xs, wn, 1e-6)
    torch.testing.assert_close(y, xs * torch.rsqrt(xs.pow(2).mean(-1, keepdim=True) + 1e-6) * wn)

    W, xv, bv = r(48, 64), r(3, 64), r(48)
    y = torch.ops.difflet.gemv(W, xv, bv, True, False)
    torch.testing.assert_close(y, torch.nn.functional.silu(xv) @ W.t() + bv, atol=1e-5, rtol=1e-5)


def test_cpu_mx_roundtrip():
    r = _inputs("cpu")
    a, bw = r(8, 128).bfloat16(), r(16, 128).bfloat16()
    aq, asf = torch.ops.difflet.quantize_mx(a)
    bq, bsf = torch.ops.difflet.quantize_mx(bw)
    assert aq.dtype == torch.float8_e4m3fn and asf.shape == (8, 4)
    y = torch.ops.difflet.linear_mx(aq, asf, bq, bsf, None)
    ref = a.float() @ bw.float().t()
    assert (y.float() - ref).norm() / ref.norm() < 0.08


@pytest.mark.gpu
def test_gpu_ops_match_fp32_reference():
    from difflet_b200 import _native

    _native.require()
    r = _inputs("cuda", torch.bfloat16)
    q, k, v = r(1, 4, 512, 128), r(1, 4, 640, 128), r(1, 4, 640, 128)
    o = torch.ops.difflet.attention(q, k, v, 0.088)
    torch.testing.assert_close(o.float(), _ref_attention(q, k, v, 0.088), atol=2e-2, rtol=2e-2)
    x, w, b = r(300, 256), r(512, 256) * 0.05, r(512)
    y = torch.ops.difflet.linear(x, w, b, "gelu", 0, -1)
    ref = torch.nn.functional.gelu(x.float() @ w.float().t() + b.float(), approximate="tanh")
    torch.testing.assert_close(y.float(), ref, atol=3e-2, rtol=3e-2)
    xs = r(4, 1024)
    y = torch.ops.difflet.rms_norm(xs, None, 1e-6)
    ref = xs.float() * torch.rsqrt(xs.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    torch.testing.assert_close(y.float(), ref, atol=2e-2, rtol=2e-2)
