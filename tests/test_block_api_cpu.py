"""CPU forms of the fused block entry points in ops/api.py: the attention node that
takes the block input (QKV projection + RoPE + causal attention) and the pre-norm
entry points that pass the residual stream through.  On the CPU they are the plain
compositions; the test pins them to the reference math and to each other (the GPU
forms are tested against the same math in tests/test_flash_gpu.py and
tests/test_kernels_gpu.py)."""
import math

import torch

from oxidizr_b200.ops import api
from oxidizr_b200.ops import reference as R


def test_attention_rope_is_projection_rope_attention():
    torch.manual_seed(0)
    B, S, H, nh, kvh, hd = 2, 12, 32, 4, 2, 8
    x = torch.randn(B, S, H, dtype=torch.float64, requires_grad=True)
    w = torch.randn((nh + 2 * kvh) * hd, H, dtype=torch.float64, requires_grad=True)
    cos, sin = R.rope_tables(hd, S, 10000.0, dtype=torch.float64)
    scale = 1.0 / math.sqrt(hd)
    o = api.attention_rope(x, w, cos, sin, nh, kvh, hd, scale)
    # by hand: projection, rotate-half RoPE on q and k, GQA causal softmax attention
    y = x @ w.t()
    q = y[..., :nh * hd].reshape(B, S, nh, hd).transpose(1, 2)
    k = y[..., nh * hd:(nh + kvh) * hd].reshape(B, S, kvh, hd).transpose(1, 2)
    v = y[..., (nh + kvh) * hd:].reshape(B, S, kvh, hd).transpose(1, 2)
    q, k = R.apply_rope(q, cos[:S], sin[:S]), R.apply_rope(k, cos[:S], sin[:S])
    k, v = k.repeat_interleave(nh // kvh, 1), v.repeat_interleave(nh // kvh, 1)
    s = (q @ k.transpose(-1, -2)) * scale
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    ref = (s.softmax(-1) @ v).transpose(1, 2).reshape(B, S, nh * hd)
    torch.testing.assert_close(o, ref, rtol=1e-10, atol=1e-10)
    g = torch.randn_like(o)
    gx, gw = torch.autograd.grad(o, (x, w), g)
    rx, rw = torch.autograd.grad(ref, (x, w), g)
    torch.testing.assert_close(gx, rx)
    torch.testing.assert_close(gw, rw)


def test_norm_resid_entry_points_pass_the_stream_through():
    torch.manual_seed(1)
    x = torch.randn(3, 5, 16, dtype=torch.float64, requires_grad=True)
    w = torch.rand(16, dtype=torch.float64) + 0.5
    b = torch.randn(16, dtype=torch.float64)
    h, r = api.rmsnorm_resid(x, w, 1e-5)
    torch.testing.assert_close(h, R.rmsnorm(x, w, 1e-5))
    assert r is x
    h2, r2 = api.layernorm_resid(x, w, b, 1e-6)
    torch.testing.assert_close(h2, R.layernorm(x, w, b, 1e-6))
    assert r2 is x
