"""tcgen05 flash attention vs the materialised fp32 reference."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, scale, causal=True):
    from oxidizr_b200.ops import reference as R
    o = R.attention(q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2), scale, causal)
    return o.transpose(1, 2)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,S,Hq,Hk", [(2, 300, 4, 2), (1, 128, 2, 2), (2, 512, 8, 1)])
def test_flash_fwd(D, B, S, Hq, Hk):
    from oxidizr_b200.ops._C import ext, status, check_status
    torch.manual_seed(D + S)
    # q|k|v fused in one buffer like the QKV GEMM produces
    qkv = torch.randn(B * S, (Hq + 2 * Hk) * D, device="cuda").bfloat16()
    q = qkv[:, :Hq * D]
    k = qkv[:, Hq * D:(Hq + Hk) * D]
    v = qkv[:, (Hq + Hk) * D:]
    o = torch.empty(B * S, Hq * D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, S, device="cuda")
    scale = 1.0 / math.sqrt(D)
    ext().flash_fwd(q, k, v, o, lse, B, S, Hq, Hk, D, D, scale, True, status("cuda"))
    torch.cuda.synchronize()
    check_status("cuda")
    qr, kr, vr = (t.reshape(B, S, -1, D) for t in (q, k, v))
    ref = _ref(qr, kr, vr, scale).reshape(B * S, Hq * D)
    err = ((o.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err
    # lse
    hq = qr.float().transpose(1, 2)
    hk = kr.float().transpose(1, 2).repeat_interleave(Hq // Hk, 1)
    s = hq @ hk.transpose(-1, -2) * scale
    s = s.masked_fill(torch.ones(S, S, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    assert torch.allclose(lse, torch.logsumexp(s, -1), atol=2e-2, rtol=1e-3)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,S,Hq,Hk", [(2, 300, 4, 2), (1, 256, 2, 2), (2, 384, 8, 1)])
def test_flash_bwd_qkv(D, B, S, Hq, Hk):
    from oxidizr_b200.ops.flash import FlashAttentionQKV
    from oxidizr_b200.ops._C import check_status
    torch.manual_seed(7 + D + S)
    N = (Hq + 2 * Hk) * D
    qkv = torch.randn(B, S, N, device="cuda").bfloat16().requires_grad_()
    scale = 1.0 / math.sqrt(D)
    o = FlashAttentionQKV.apply(qkv, Hq, Hk, D, scale, True)
    do = torch.randn_like(o)
    o.backward(do)
    torch.cuda.synchronize()
    check_status("cuda")
    x = qkv.detach().float().requires_grad_()
    q = x[..., :Hq * D].view(B, S, Hq, D)
    k = x[..., Hq * D:(Hq + Hk) * D].view(B, S, Hk, D)
    v = x[..., (Hq + Hk) * D:].view(B, S, Hk, D)
    ref = _ref(q, k, v, scale).reshape(B, S, Hq * D)
    ref.backward(do.float())
    err_o = ((o.float() - ref).norm() / ref.norm()).item()
    assert err_o < 1e-2, err_o
    g, gr = qkv.grad.float(), x.grad
    for name, sl in (("q", slice(0, Hq * D)), ("k", slice(Hq * D, (Hq + Hk) * D)), ("v", slice((Hq + Hk) * D, N))):
        e = ((g[..., sl] - gr[..., sl]).norm() / gr[..., sl].norm()).item()
        assert e < 3e-2, (name, e)


@pytest.mark.parametrize("Dqk,Dv", [(96, 64), (128, 64)])
@pytest.mark.parametrize("B,S,H", [(2, 300, 3), (1, 512, 12)])
def test_flash_mla_head_dims(Dqk, Dv, B, S, H):
    """Multi-head latent attention shapes: q/k carry a RoPE part (Dqk > Dv)."""
    from oxidizr_b200.ops.flash import FlashAttention
    from oxidizr_b200.ops._C import check_status
    torch.manual_seed(Dqk + S + H)
    q = torch.randn(B, S, H, Dqk, device="cuda").bfloat16().requires_grad_()
    k = torch.randn(B, S, H, Dqk, device="cuda").bfloat16().requires_grad_()
    # v as a strided view of a wider buffer, like the fused k|v up-projection output
    kv = torch.randn(B, S, 2 * H * Dv, device="cuda").bfloat16()
    v = kv[..., H * Dv:].view(B, S, H, Dv).requires_grad_()
    scale = 1.0 / math.sqrt(Dqk)
    o = FlashAttention.apply(q, k, v, scale, True)
    do = torch.randn_like(o)
    o.backward(do)
    torch.cuda.synchronize()
    check_status("cuda")
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = _ref(qr, kr, vr, scale)
    ref.backward(do.float())
    assert o.shape == (B, S, H, Dv)
    assert ((o.float() - ref).norm() / ref.norm()).item() < 1e-2
    for name, a, r in (("q", q.grad, qr.grad), ("k", k.grad, kr.grad), ("v", v.grad, vr.grad)):
        e = ((a.float() - r).norm() / r.norm()).item()
        assert e < 3e-2, (name, e)
