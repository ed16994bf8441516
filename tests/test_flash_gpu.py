"""tcgen05 flash attention vs the materialised fp32 reference."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


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


@pytest.mark.parametrize("B,S,nh,hd,dr", [(2, 128, 12, 64, 32), (1, 256, 4, 128, 64), (3, 64, 2, 64, 16)])
def test_mla_pack_matches_reference(B, S, nh, hd, dr):
    """MLA operand packing (RoPE on the rope parts, shared k_rope broadcast, v packed) and its
    backward against the fp32 PyTorch statement (model.rs:196-256)."""
    from oxidizr_b200.models.common import RopeCache
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops.mla import MlaPack
    torch.manual_seed(B + S + dr)
    qc = torch.randn(B, S, nh * hd, device="cuda").bfloat16().requires_grad_()
    kv = torch.randn(B, S, 2 * nh * hd, device="cuda").bfloat16().requires_grad_()
    big = torch.randn(B, S, 40 + dr + nh * dr, device="cuda").bfloat16()
    rp = big[..., 40:].detach().requires_grad_()  # a column block of a wider projection, like the model's
    cos, sin = RopeCache.get(dr, S, 10000.0, "cuda")
    q, k, v = MlaPack.apply(qc, kv, rp, cos, sin, nh, hd, dr)
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    (q.float() * gq.float()).sum().add((k.float() * gk.float()).sum()).add((v.float() * gv.float()).sum()).backward()
    # reference in f32
    qc_r, kv_r, rp_r = (t.detach().float().requires_grad_() for t in (qc, kv, rp))
    q_r = R.apply_rope(rp_r[..., dr:].reshape(B, S, nh, dr).transpose(1, 2), cos, sin).transpose(1, 2)
    k_r = R.apply_rope(rp_r[..., :dr].reshape(B, S, 1, dr).transpose(1, 2), cos, sin).transpose(1, 2)
    qr = torch.cat([qc_r.view(B, S, nh, hd), q_r], -1)
    kr = torch.cat([kv_r[..., :nh * hd].view(B, S, nh, hd), k_r.expand(B, S, nh, dr)], -1)
    vr = kv_r[..., nh * hd:].view(B, S, nh, hd)
    (qr * gq.float()).sum().add((kr * gk.float()).sum()).add((vr * gv.float()).sum()).backward()
    assert _rel(q, qr) < 5e-3 and _rel(k, kr) < 5e-3 and torch.equal(v.float(), vr.detach())
    assert _rel(qc.grad, qc_r.grad) < 5e-3
    assert _rel(kv.grad, kv_r.grad) < 5e-3
    assert _rel(rp.grad, rp_r.grad) < 1e-2


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("B,S,Hq,Hk,H", [(2, 300, 4, 2, 256), (1, 512, 8, 1, 512)])
def test_attention_rope_fused_backward(hd, B, S, Hq, Hk, H):
    """One attention node from the block input (QKV GEMM with RoPE, flash forward; the
    backward un-rotates dq / dk inside the flash backward) against fp32 torch: the
    output, dX and dW of the QKV projection."""
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops._C import check_status
    from oxidizr_b200.ops.fused import AttentionQKVRope
    from oxidizr_b200.models.common import RopeCache
    torch.manual_seed(hd + S)
    N = (Hq + 2 * Hk) * hd
    x = (torch.randn(B, S, H, device="cuda") * 0.5).bfloat16().requires_grad_()
    w = (torch.randn(N, H, device="cuda") / math.sqrt(H)).bfloat16().requires_grad_()
    cos, sin = RopeCache.get(hd, S, 10000.0, x.device)
    scale = 1.0 / math.sqrt(hd)
    o = AttentionQKVRope.apply(x, w, cos, sin, Hq, Hk, hd, scale)
    do = torch.randn_like(o)
    o.backward(do)
    torch.cuda.synchronize()
    check_status("cuda")
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    y = xr @ wr.t()
    q = y[..., :Hq * hd].reshape(B, S, Hq, hd).transpose(1, 2)
    k = y[..., Hq * hd:(Hq + Hk) * hd].reshape(B, S, Hk, hd).transpose(1, 2)
    v = y[..., (Hq + Hk) * hd:].reshape(B, S, Hk, hd)
    q = R.apply_rope(q, cos[:S], sin[:S]).transpose(1, 2)
    k = R.apply_rope(k, cos[:S], sin[:S]).transpose(1, 2)
    ref = _ref(q, k, v, scale).reshape(B, S, Hq * hd)
    ref.backward(do.float())
    assert _rel(o, ref) < 1e-2
    assert _rel(x.grad, xr.grad) < 3e-2, _rel(x.grad, xr.grad)
    # per block of the projection's rows: q, k (un-rotated in the flash backward) and v
    for name, sl in (("q", slice(0, Hq * hd)), ("k", slice(Hq * hd, (Hq + Hk) * hd)), ("v", slice((Hq + Hk) * hd, N))):
        e = _rel(w.grad[sl], wr.grad[sl])
        assert e < 3e-2, (name, e)
