"""SSM kernels (conv1d, SSD) vs the fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-8)).item()


@pytest.mark.parametrize("K", [2, 3, 4])
@pytest.mark.parametrize("act", [True, False])
@pytest.mark.parametrize("B,S,C", [(2, 100, 64), (1, 300, 1792), (3, 64, 8), (4, 1024, 1792)])
def test_conv1d(K, act, B, S, C):
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops.ssm_kernels import CausalConv1d
    torch.manual_seed(K + S + C)
    # input as a strided column slice of a wider projection, like in_proj output
    big = torch.randn(B, S, C + 16, device="cuda").bfloat16()
    x = big[..., 8:8 + C].detach().requires_grad_()
    w = (0.5 * torch.randn(C, 1, K, device="cuda")).bfloat16().requires_grad_()
    b = (0.1 * torch.randn(C, device="cuda")).bfloat16().requires_grad_()
    y = CausalConv1d.apply(x, w, b, act)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr, wr, br = (t.detach().float().requires_grad_() for t in (x, w, b))
    yr = R.causal_conv1d(xr, wr, br, act)
    yr.backward(dy.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    assert _rel(w.grad, wr.grad) < 2e-2
    assert _rel(b.grad, br.grad) < 2e-2


@pytest.mark.parametrize("G", [1, 2, 4])
@pytest.mark.parametrize("B,S,H,P,N", [(2, 70, 4, 16, 32), (1, 130, 4, 64, 128)])
def test_ssd_scan_mamba2(G, B, S, H, P, N):
    """Mamba2 SSD via the scan kernel vs the sequential recurrence (fwd + all grads)."""
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops import ssm
    torch.manual_seed(G + S + P)
    x = torch.randn(B, S, H, P, device="cuda").requires_grad_()
    dt = (torch.rand(B, S, H, device="cuda") * 0.09 + 0.01).requires_grad_()
    A = (-torch.rand(H, device="cuda") * 2 - 0.1).requires_grad_()
    Bg = torch.randn(B, S, G, N, device="cuda").requires_grad_()
    Cg = torch.randn(B, S, G, N, device="cuda").requires_grad_()
    y = ssm.ssd(x, dt, A, Bg, Cg, 32)
    dy = torch.randn_like(y)
    y.backward(dy)
    ref_in = [t.detach().double().requires_grad_() for t in (x, dt, A, Bg, Cg)]
    xr, dtr, Ar, Br, Cr = ref_in
    yr = R.ssd_sequential(xr, dtr, Ar, Br.repeat_interleave(H // G, 2), Cr.repeat_interleave(H // G, 2))
    yr.backward(dy.double())
    assert _rel(y, yr) < 1e-4
    for g, r in zip((x.grad, dt.grad, A.grad, Bg.grad, Cg.grad), (xr.grad, dtr.grad, Ar.grad, Br.grad, Cr.grad)):
        assert _rel(g, r) < 1e-3


@pytest.mark.parametrize("B,S,H,P,N", [(2, 50, 2, 32, 64), (1, 140, 2, 64, 128)])
def test_mamba3_scan(B, S, H, P, N):
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops import ssm
    torch.manual_seed(S + P)
    x = torch.randn(B, S, H, P, device="cuda").requires_grad_()
    dt = (torch.rand(B, S, H, device="cuda") * 0.09 + 0.01).requires_grad_()
    A = (-torch.rand(H, device="cuda") * 2 - 0.1).requires_grad_()
    Bm = torch.randn(B, S, H, N, device="cuda").requires_grad_()
    Cm = torch.randn(B, S, H, N, device="cuda").requires_grad_()
    lam = torch.rand(B, S, H, device="cuda").requires_grad_()
    y = ssm.mamba3_scan(x, dt, A, Bm, Cm, lam, 32)
    dy = torch.randn_like(y)
    y.backward(dy)
    ins = [t.detach().double().requires_grad_() for t in (x, dt, A, Bm, Cm, lam)]
    yr = R.mamba3_sequential(*ins)
    yr.backward(dy.double())
    assert _rel(y, yr) < 1e-4
    for g, r in zip((x.grad, dt.grad, A.grad, Bm.grad, Cm.grad, lam.grad), [t.grad for t in ins]):
        assert _rel(g, r) < 1e-3


@pytest.mark.parametrize("clamp", [None, 30.0])
@pytest.mark.parametrize("B,S,D", [(2, 40, 96), (1, 70, 100)])
def test_mamba1_scan(clamp, B, S, D):
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops import ssm
    torch.manual_seed(3)
    u = torch.randn(B, S, D, device="cuda").requires_grad_()
    delta = (torch.rand(B, S, D, device="cuda") * 0.5).requires_grad_()
    A = (-torch.rand(D, 16, device="cuda") * 3).requires_grad_()
    Bm = torch.randn(B, S, 16, device="cuda").requires_grad_()
    Cm = torch.randn(B, S, 16, device="cuda").requires_grad_()
    y = ssm.selective_scan(u, delta, A, Bm, Cm, clamp)
    dy = torch.randn_like(y)
    y.backward(dy)
    ins = [t.detach().double().requires_grad_() for t in (u, delta, A, Bm, Cm)]
    yr = R.selective_scan(*ins, clamp)
    yr.backward(dy.double())
    assert _rel(y, yr) < 1e-4
    for g, r in zip((u.grad, delta.grad, A.grad, Bm.grad, Cm.grad), [t.grad for t in ins]):
        assert _rel(g, r) < 1e-3


def _tc_inputs(B, S, H, P, N, G, seed):
    torch.manual_seed(seed)
    x = torch.randn(B, S, H, P, device="cuda").bfloat16().requires_grad_()
    dt = (torch.rand(B, S, H, device="cuda") * 0.09 + 0.01).requires_grad_()
    A = (-torch.rand(H, device="cuda") * 2 - 0.1).requires_grad_()
    Bg = (torch.randn(B, S, G, N, device="cuda") / N ** 0.25).bfloat16().requires_grad_()
    Cg = (torch.randn(B, S, G, N, device="cuda") / N ** 0.25).bfloat16().requires_grad_()
    return x, dt, A, Bg, Cg


@pytest.mark.parametrize("B,S,H,P,G", [(2, 256, 4, 64, 1), (1, 384, 4, 128, 2), (2, 128, 2, 64, 2)])
def test_ssd_tensor_core_mamba2(B, S, H, P, G):
    """tcgen05 chunked SSD (bf16 operands, f32 state) vs the fp64 sequential recurrence."""
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops.ssd_tc import ssd_tc, tc_ok
    from oxidizr_b200.ops._C import check_status
    N = 128
    x, dt, A, Bg, Cg = _tc_inputs(B, S, H, P, N, G, S + P + G)
    assert tc_ok(x, N, S)
    y = ssd_tc(x, dt, A, Bg, Cg)
    dy = torch.randn_like(y)
    y.backward(dy)
    torch.cuda.synchronize()
    check_status("cuda")
    ins = [t.detach().double().requires_grad_() for t in (x, dt, A, Bg, Cg)]
    xr, dtr, Ar, Br, Cr = ins
    yr = R.ssd_sequential(xr, dtr, Ar, Br.repeat_interleave(H // G, 2), Cr.repeat_interleave(H // G, 2))
    yr.backward(dy.double())
    assert _rel(y, yr) < 2e-2, _rel(y, yr)
    for name, g, r in zip(("x", "dt", "A", "B", "C"), (x.grad, dt.grad, A.grad, Bg.grad, Cg.grad), [t.grad for t in ins]):
        assert _rel(g, r) < 3e-2, (name, _rel(g, r))


@pytest.mark.parametrize("B,S,H,P", [(1, 128, 2, 64), (2, 256, 2, 128)])
def test_ssd_tensor_core_mamba3(B, S, H, P):
    """Mamba3 two-term scan through the shifted-state tensor-core SSD vs the fp64 sequential recurrence."""
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops.ssd_tc import mamba3_tc
    from oxidizr_b200.ops._C import check_status
    N = 128
    x, dt, A, Bm, Cm = _tc_inputs(B, S, H, P, N, H, S + P)
    lam = torch.rand(B, S, H, device="cuda").requires_grad_()
    from oxidizr_b200.ops.ssd_tc import tc_ok
    assert tc_ok(x, N, S)
    y = mamba3_tc(x, dt, A, Bm, Cm, lam)
    dy = torch.randn_like(y)
    y.backward(dy)
    torch.cuda.synchronize()
    check_status("cuda")
    ins = [t.detach().double().requires_grad_() for t in (x, dt, A, Bm, Cm, lam)]
    yr = R.mamba3_sequential(*ins)
    yr.backward(dy.double())
    assert _rel(y, yr) < 2e-2, _rel(y, yr)
    # dA sums d loga dt over every step and head, with cancellation: bf16 operand
    # rounding shows up there most
    for name, g, r in zip(("x", "dt", "A", "B", "C", "lam"), (x.grad, dt.grad, A.grad, Bm.grad, Cm.grad, lam.grad),
                          [t.grad for t in ins]):
        assert _rel(g, r) < (6e-2 if name == "A" else 3e-2), (name, _rel(g, r))


def test_mamba3_fused_prologue_matches_unfused():
    """Mamba3 mixer: fused B/C prologue + shifted-state tensor-core scan == the unfused torch path."""
    from oxidizr_b200.config import ModelConfig, _build
    from oxidizr_b200.models.mamba import Mamba3Mixer
    torch.manual_seed(0)
    cfg = _build(ModelConfig, {
        "name": "m3", "hidden_size": 256, "num_layers": 1, "num_heads": 4, "vocab_size": 100, "max_seq_len": 128,
        "rope_theta": 10000.0, "mamba_layers": [0], "mamba3_enabled": True, "mamba3_complex_rope": True,
        "mamba3_mimo_rank": 2, "mamba3_use_conv": False, "mamba2_num_heads": 4, "mamba2_head_dim": 128,
        "mamba2_state_size": 128, "mamba2_chunk_size": 64, "mamba2_n_groups": 1, "mamba2_expand": 2}, "model")
    mix = Mamba3Mixer(cfg, device="cuda", dtype=torch.bfloat16)
    mix.reset_parameters(0.05, torch.Generator(device="cuda").manual_seed(1))
    with torch.no_grad():
        mix.b_bias.add_(0.1 * torch.randn_like(mix.b_bias))
        mix.bc_norm.weight.add_(0.1 * torch.randn_like(mix.bc_norm.weight))
    h = torch.randn(2, 128, 256, device="cuda").bfloat16().requires_grad_()
    resid = torch.zeros(2, 128, 256, device="cuda").bfloat16()
    assert mix._fused_ok(h, h[..., :1], 128)
    y1 = mix(h, resid)
    dy = torch.randn_like(y1)
    g1 = torch.autograd.grad(y1, [h] + list(mix.parameters()), dy, allow_unused=True)
    mix._fused_ok = lambda *a: False
    y2 = mix(h, resid)
    g2 = torch.autograd.grad(y2, [h] + list(mix.parameters()), dy, allow_unused=True)
    assert _rel(y1, y2) < 3e-2, _rel(y1, y2)
    names = ["h"] + [n for n, _ in mix.named_parameters()]
    for n, a, b in zip(names, g1, g2):
        if a is None or b is None:
            assert a is None and b is None, n
            continue
        assert _rel(a, b) < 5e-2, (n, _rel(a, b))


def test_angle_cumsum_kernel():
    from oxidizr_b200.ops.ssd_tc import AngleCumsum
    torch.manual_seed(5)
    theta = torch.randn(2, 300, 3, 64, device="cuda").requires_grad_()
    dt = torch.rand(2, 300, 3, device="cuda").requires_grad_()
    ang = AngleCumsum.apply(theta, dt)
    g = torch.randn_like(ang)
    ang.backward(g)
    tr, dr = theta.detach().double().requires_grad_(), dt.detach().double().requires_grad_()
    ref = torch.cumsum(tr * dr[..., None], 1)
    ref.backward(g.double())
    assert _rel(ang, ref) < 1e-5
    assert _rel(theta.grad, tr.grad) < 1e-5
    assert _rel(dt.grad, dr.grad) < 1e-5


@pytest.mark.parametrize("B,S,H,G", [(2, 64, 4, 2), (1, 100, 32, 1), (2, 40, 16, 1), (1, 24, 64, 1), (1, 36, 8, 1)])
def test_mamba3_bc_prologue_kernel(B, S, H, G):
    """Fused B/C prologue vs torch: rmsnorm + bias + rotation, <B, C>, and grads (one B/C group
    with 8, 16, 32 or 64 heads takes the heads-per-warp backward)."""
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops.ssd_tc import Mamba3BC
    torch.manual_seed(7)
    N = 128
    wide = torch.randn(B, S, 2 * G * N + 8, device="cuda").bfloat16()
    braw = wide[..., :G * N].detach().requires_grad_()
    craw = wide[..., G * N:2 * G * N].detach().requires_grad_()
    w = (1 + 0.1 * torch.randn(N, device="cuda")).bfloat16().requires_grad_()
    bb = (1 + 0.1 * torch.randn(H, N, device="cuda")).bfloat16().requires_grad_()
    cb = (1 + 0.1 * torch.randn(H, N, device="cuda")).bfloat16().requires_grad_()
    # angles are cumulative sums over the sequence: include large ones
    ang = (3 * torch.randn(B, S, H, N // 2, device="cuda") + 2000 * torch.rand(B, S, 1, 1, device="cuda")
           ).requires_grad_()
    bo, co, dot = Mamba3BC.apply(braw, craw, w, bb, cb, ang, H, 1e-6)
    torch.cuda.synchronize()
    gb, gc = torch.randn_like(bo, dtype=torch.float32), torch.randn_like(co, dtype=torch.float32)
    gd = torch.randn_like(dot)
    ((bo.float() * gb + co.float() * gc).sum() + (dot * gd).sum()).backward()
    ins = [t.detach().double().requires_grad_() for t in (braw, craw, w, bb, cb, ang)]
    rb, rc, rw, rbb, rcb, ra = ins
    rep = lambda t: t.view(B, S, G, N).repeat_interleave(H // G, 2)
    nb = R.rmsnorm(rep(rb), rw, 1e-6) + rbb
    nc = R.rmsnorm(rep(rc), rw, 1e-6) + rcb
    bt, ct = R.mamba3_rotate(nb, ra), R.mamba3_rotate(nc, ra)
    dr = (bt * ct).sum(-1)
    assert _rel(bo, bt) < 1e-2 and _rel(co, ct) < 1e-2 and _rel(dot, dr) < 1e-2
    ((bt * gb.double() + ct * gc.double()).sum() + (dr * gd.double()).sum()).backward()
    for name, a, r in zip(("braw", "craw", "w", "b_bias", "c_bias", "ang"),
                          (braw.grad, craw.grad, w.grad, bb.grad, cb.grad, ang.grad), [t.grad for t in ins]):
        assert _rel(a, r) < 2e-2, (name, _rel(a, r))


def test_ssd_dloga_scan_kernel():
    """Reverse scan for SSD d loga vs the torch flip-cumsum formula."""
    from oxidizr_b200.ops._C import ext
    torch.manual_seed(9)
    B, S, H = 2, 300, 5
    e, ga, dg = (torch.randn(B, S, H, device="cuda") for _ in range(3))
    dla = ext().ssd_dloga(e, ga, dg)
    v = (ga * dg).double()
    v_next = torch.cat([v[:, 1:], torch.zeros_like(v[:, :1])], 1)
    q = torch.flip(torch.cumsum(torch.flip(e.double() - v_next, [1]), 1), [1])
    assert _rel(dla, q - v) < 1e-5


@pytest.mark.parametrize("P,per_row", [(64, False), (256, True), (128, True)])
def test_dskip_epilogue_kernels(P, per_row):
    """D-skip epilogue: bf16(y + d x) and its backward (dx, dd, <g, y>) vs torch fp32."""
    from oxidizr_b200.ops._C import ext
    torch.manual_seed(11)
    T, H = 300, 3
    y = torch.randn(T, H * P, device="cuda")
    x = torch.randn(T, H * P, device="cuda").bfloat16()
    d = torch.randn(T, H, device="cuda") if per_row else torch.randn(H, device="cuda")
    dx_scan = torch.randn(T, H * P, device="cuda")
    g = torch.randn(T, H * P, device="cuda").bfloat16()
    out = ext().dskip_fwd(y, x, d.contiguous(), H)
    dv = (d if per_row else d[None].expand(T, H))[..., None]
    ref = y.view(T, H, P) + dv * x.float().view(T, H, P)
    assert _rel(out.view(T, H, P), ref) < 1e-2
    dx, dd, e = ext().dskip_bwd(g, x, y, d.contiguous(), dx_scan, H)
    gf = g.float().view(T, H, P)
    assert _rel(dx.view(T, H, P), dx_scan.view(T, H, P) + dv * gf) < 1e-2
    assert _rel(dd, (gf * x.float().view(T, H, P)).sum(-1)) < 1e-5
    assert _rel(e, (gf * y.view(T, H, P)).sum(-1)) < 1e-5


@pytest.mark.parametrize("B,S,H", [(2, 100, 8), (1, 256, 32), (3, 7, 5)])
def test_mamba3_coefficients(B, S, H):
    """Step size, lambda and the shifted-state coefficients (csrc/m3_glue.cu) against the fp32
    torch statement: dt = clamp(softplus(dt_raw + dt_bias), 1e-3, 0.1), lam = sigmoid(l_raw),
    log alpha = A dt, c_t = (1 - lam_{t+1}) dt_{t+1} (0 at the end), gamma' = lam dt + c."""
    from oxidizr_b200.ops.ssd_tc import Mamba3Coef
    torch.manual_seed(B * S + H)
    # raw step sizes around the clamp edges so that both sides of each get exercised
    dt_raw = (torch.randn(B, S, H, device="cuda") * 3 - 3).bfloat16().requires_grad_()
    bias = (torch.randn(H, device="cuda") * 0.5).bfloat16().requires_grad_()
    l_raw = torch.randn(B, S, H, device="cuda").bfloat16().requires_grad_()
    A = (-torch.rand(H, device="cuda") * 2 - 0.1).requires_grad_()
    outs = Mamba3Coef.apply(dt_raw, bias, l_raw, A)
    gs = [torch.randn_like(o) for o in outs]
    sum((o * g).sum() for o, g in zip(outs, gs)).backward()
    dr, br, lr, Ar = (t.detach().float().requires_grad_() for t in (dt_raw, bias, l_raw, A))
    dt = torch.nn.functional.softplus(dr + br).clamp(1e-3, 0.1)
    lam = torch.sigmoid(lr)
    loga = Ar[None, None, :] * dt
    w = (1 - lam) * dt
    c = torch.cat([w[:, 1:], torch.zeros_like(w[:, :1])], 1)
    gp = lam * dt + c
    ref = (dt, loga, gp, c)
    sum((o * g).sum() for o, g in zip(ref, gs)).backward()
    for o, r in zip(outs, ref):
        assert _rel(o, r) < 1e-5
    assert _rel(dt_raw.grad, dr.grad) < 1e-2
    assert _rel(l_raw.grad, lr.grad) < 1e-2
    assert _rel(bias.grad, br.grad) < 1e-2
    assert _rel(A.grad, Ar.grad) < 1e-4
