"""Memory-bound kernels (norms, CE, embedding, RoPE bwd, AdamW) and the full
model on CUDA vs the fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-8)).item()


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("H", [256, 2048, 1536, 4096, 520])
def test_norms_fwd_bwd(mode, H):
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops.fused import Norm
    torch.manual_seed(mode * 7 + H)
    T = 333
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    g = torch.randn(T, H, device="cuda").bfloat16().requires_grad_() if mode == 2 else None
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_()
    b = (0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_() if mode == 1 else None
    y = Norm.apply(x, g, w, b, mode, 1e-5)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    gr = g.detach().float().requires_grad_() if mode == 2 else None
    br = b.detach().float().requires_grad_() if mode == 1 else None
    if mode == 0:
        yr = R.rmsnorm(xr, wr, 1e-5)
    elif mode == 1:
        yr = R.layernorm(xr, wr, br, 1e-5)
    else:
        yr = R.gated_rmsnorm(xr, gr, wr, 1e-5)
    yr.backward(dy.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    assert _rel(w.grad, wr.grad) < 2e-2
    if mode == 1:
        assert _rel(b.grad, br.grad) < 2e-2
    if mode == 2:
        assert _rel(g.grad, gr.grad) < 2e-2


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("H", [2048, 520])
def test_norm_resid_adds_residual_gradient_and_accumulates_main_grad(mode, H):
    """(norm(x), x) with the residual branch's gradient added inside the norm backward, and
    the weight / bias gradients added straight into existing main_grad buffers."""
    from oxidizr_b200.ops import reference as R
    from oxidizr_b200.ops.fused import NormResid
    torch.manual_seed(11 + mode + H)
    T = 333
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    w = torch.nn.Parameter((1 + 0.1 * torch.randn(H, device="cuda")).bfloat16())
    b = torch.nn.Parameter((0.1 * torch.randn(H, device="cuda")).bfloat16()) if mode == 1 else None
    w.main_grad = torch.full((H,), 0.25, device="cuda")
    if b is not None:
        b.main_grad = torch.full((H,), -0.5, device="cuda")
    y, xp = NormResid.apply(x, w, b, mode, 1e-5)
    dy, dr = torch.randn_like(y), torch.randn_like(y)
    torch.autograd.backward([y, xp], [dy, dr])
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    br = b.detach().float().requires_grad_() if mode == 1 else None
    yr = R.rmsnorm(xr, wr, 1e-5) if mode == 0 else R.layernorm(xr, wr, br, 1e-5)
    torch.autograd.backward([yr, xr * 1.0], [dy.float(), dr.float()])
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    assert w.grad is None
    assert _rel(w.main_grad - 0.25, wr.grad) < 2e-2
    if mode == 1:
        assert b.grad is None
        assert _rel(b.main_grad + 0.5, br.grad) < 2e-2


def test_linear_cross_entropy():
    from oxidizr_b200.ops.fused import LinearCrossEntropy
    torch.manual_seed(0)
    T, H, V = 1000, 512, 5003
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    w = (torch.randn(V, H, device="cuda") / H ** 0.5).bfloat16().requires_grad_()
    t = torch.randint(0, V, (T,), device="cuda")
    t[5] = -100
    loss = LinearCrossEntropy.apply(x, w, t, -100)
    loss.backward()
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    lr = torch.nn.functional.cross_entropy(xr @ wr.t(), t, ignore_index=-100)
    lr.backward()
    assert abs(loss.item() - lr.item()) < 2e-3 * abs(lr.item())
    assert _rel(x.grad, xr.grad) < 3e-2
    assert _rel(w.grad, wr.grad) < 3e-2


@pytest.mark.parametrize("T,H,V,chunk", [(1000, 512, 5003, 1024), (2048, 256, 30011, 8192), (300, 128, 777, 96)])
def test_linear_cross_entropy_logit_free(monkeypatch, T, H, V, chunk):
    """The chunked (logit-free) backward against the materialised one and fp32 torch; its
    peak extra memory is one [T, chunk] block, never the [T, V] logits."""
    from oxidizr_b200.ops import fused
    torch.manual_seed(T + V)
    x0 = torch.randn(T, H, device="cuda").bfloat16()
    w0 = (torch.randn(V, H, device="cuda") / H ** 0.5).bfloat16()
    t = torch.randint(0, V, (T,), device="cuda")
    t[::11] = -100
    res = {}
    for mode in ("full", "chunked"):
        monkeypatch.setenv("OXI_CE_MODE", mode)
        monkeypatch.setattr(fused, "CE_CHUNK", chunk)
        x = x0.clone().requires_grad_()
        w = w0.clone().requires_grad_()
        w.main_grad = torch.zeros(V, H, device="cuda")  # the trainer's f32 gradient view
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        loss = fused.LinearCrossEntropy.apply(x, w, t, -100)
        loss.backward()
        torch.cuda.synchronize()
        res[mode] = (loss.detach(), x.grad, w.main_grad, torch.cuda.max_memory_allocated() - base)
    lf, dxf, dwf, _ = res["full"]
    lc, dxc, dwc, peak = res["chunked"]
    assert abs(lc.item() - lf.item()) < 1e-5 * abs(lf.item())
    assert _rel(dxc, dxf) < 1e-2 and _rel(dwc, dwf) < 1e-2
    # the chunked path holds an f32 [T, H] dX, one [T, chunk] logits block and the
    # partials; the full logits alone would be 2 T V bytes
    if V > 4 * chunk:
        assert peak < 2 * T * V, (peak, 2 * T * V)
    xr = x0.float().requires_grad_()
    wr = w0.float().requires_grad_()
    lr = torch.nn.functional.cross_entropy(xr @ wr.t(), t, ignore_index=-100)
    lr.backward()
    assert abs(lc.item() - lr.item()) < 2e-3 * abs(lr.item())
    assert _rel(dxc, xr.grad) < 3e-2 and _rel(dwc, wr.grad) < 3e-2


def test_embedding_and_rope_bwd():
    from oxidizr_b200.ops._C import ext
    from oxidizr_b200.ops.fused import Embedding
    from oxidizr_b200.ops import reference as R
    torch.manual_seed(1)
    V, H = 1000, 256
    w = torch.randn(V, H, device="cuda").bfloat16().requires_grad_()
    ids = torch.randint(0, V, (4, 50), device="cuda")
    y = Embedding.apply(ids, w)
    assert torch.equal(y, w.detach()[ids])
    dy = torch.randn_like(y)
    y.backward(dy)
    ref = torch.zeros(V, H, device="cuda").index_add_(0, ids.reshape(-1), dy.reshape(-1, H).float())
    assert _rel(w.grad, ref) < 1e-2
    # rope backward == transpose of the forward rotation; columns past the rotated
    # heads (the v part of a fused qkv gradient) stay as they are
    for S, hd in ((64, 128), (50, 64)):
        cos, sin = R.rope_tables(hd, S, 10000.0, device="cuda")
        x = torch.randn(2, S, 3, hd, device="cuda")
        d = torch.randn(2 * S, 4 * hd, device="cuda").bfloat16()
        xr = x.requires_grad_()
        yr = R.apply_rope(xr.transpose(1, 2), cos, sin).transpose(1, 2)
        yr.backward(d[:, :3 * hd].float().view(2, S, 3, hd))
        dd = d.clone()
        ext().rope_bwd(dd, 3 * hd, hd, cos.contiguous(), sin.contiguous())
        assert _rel(dd[:, :3 * hd].reshape(2, S, 3, hd), xr.grad) < 1e-2
        assert torch.equal(dd[:, 3 * hd:], d[:, 3 * hd:])
        assert torch.equal(ext().rope_bwd_to(d, 3 * hd, hd, cos.contiguous(), sin.contiguous()), dd)


def test_adamw_kernel_matches_reference():
    from oxidizr_b200.ops._C import ext
    from oxidizr_b200.ops import reference as R
    torch.manual_seed(2)
    n = 10007
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    scale = torch.tensor([0.5], device="cuda")
    for step in (1, 2, 3):
        ext().adamw(p, p16, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1 - 0.9 ** step, 1 - 0.999 ** step, scale)
        R.adamw_step(pr, g, mr, vr, step, 1e-3, grad_scale=0.5)
    assert torch.allclose(p, pr, atol=1e-6, rtol=1e-5)
    assert torch.equal(p16, p.bfloat16())
    sq = torch.zeros(1, device="cuda")
    ext().sqsum(g, sq)
    assert abs(sq.item() - (g * g).sum().item()) < 1e-3 * (g * g).sum().item()


def _small_cfg(**kw):
    from oxidizr_b200.config import LitConfig
    m = {"name": "t", "hidden_size": 256, "num_layers": 2, "num_heads": 2, "kv_heads": 1, "intermediate_size": 256,
         "vocab_size": 1000, "max_seq_len": 64, "rope_theta": 10000.0, "dtype": "bf16"}
    m.update(kw)
    return LitConfig.from_dict({"model": m, "trainer": {
        "learning_rate": 1e-3, "batch_size": 2, "max_steps": 1, "num_epochs": 1, "gradient_accumulation": 1,
        "checkpoint_dir": "/tmp/x", "log_interval": 1, "save_interval": 10, "load_balance_alpha": 0.0,
        "group_size": 4, "beta_kl": 0.04}})


@pytest.mark.parametrize("hd_heads", [(256, 2, 1), (512, 8, 2)])
def test_gqa_model_matches_cpu_reference(hd_heads):
    from oxidizr_b200.models import build_model
    H, nh, kvh = hd_heads
    cfg = _small_cfg(hidden_size=H, num_heads=nh, kv_heads=kvh)
    torch.manual_seed(0)
    gpu = build_model(cfg.model, device="cuda", seed=3)
    cpu = build_model(cfg.model, device="cpu", seed=3, dtype=torch.float32)
    cpu.import_ref({k: v.float().cpu() for k, v in gpu.export_ref().items()})
    ids = torch.randint(0, 1000, (2, 65))
    lg, _ = gpu(ids[:, :-1].cuda(), ids[:, 1:].cuda())
    lc, _ = cpu(ids[:, :-1], ids[:, 1:])
    assert abs(lg.item() - lc.item()) < 2e-2
    lg.backward()
    lc.backward()
    gg = {k: v for k, v in zip([n for n, _ in gpu.named_parameters()], [p.grad for p in gpu.parameters()])}
    gc = {k: v for k, v in zip([n for n, _ in cpu.named_parameters()], [p.grad for p in cpu.parameters()])}
    for k in gc:
        assert _rel(gg[k].cpu(), gc[k]) < 6e-2, k


@pytest.mark.parametrize("T,H,I,E,k", [(300, 256, 128, 4, 2), (1000, 512, 256, 8, 3), (64, 256, 128, 16, 1),
                                       (500, 256, 128, 6, 2)])
def test_grouped_experts_vs_dense(T, H, I, E, k):
    """Sparse grouped-GEMM experts == per-token dense reference (fwd + grads)."""
    from oxidizr_b200.models.common import split_gu
    from oxidizr_b200.ops.moe_kernels import GroupedExperts
    torch.manual_seed(T + E)
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    w_gu = (torch.randn(E, 2 * I, H, device="cuda") / H ** 0.5).bfloat16().requires_grad_()
    w_down = (torch.randn(E, H, I, device="cuda") / I ** 0.5).bfloat16().requires_grad_()
    logits = torch.randn(T, E, device="cuda")
    topv, topi = torch.topk(logits, k, -1)
    topw = torch.softmax(topv, -1).requires_grad_()
    resid = torch.randn(T, H, device="cuda").bfloat16()
    y = GroupedExperts.apply(x, topi, topw, w_gu, w_down, resid)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr = x.detach().float().requires_grad_()
    gr = w_gu.detach().float().requires_grad_()
    dr = w_down.detach().float().requires_grad_()
    twr = topw.detach().clone().requires_grad_()
    out = resid.float().clone()
    for e in range(E):
        g, u = split_gu(gr[e])
        ye = torch.nn.functional.linear(torch.nn.functional.silu(xr @ g.t()) * (xr @ u.t()), dr[e])
        wsel = (twr * (topi == e)).sum(-1, keepdim=True)
        out = out + wsel * ye
    out.backward(dy.float())
    assert _rel(y, out) < 2e-2
    assert _rel(x.grad, xr.grad) < 3e-2
    assert _rel(w_gu.grad, gr.grad) < 3e-2
    assert _rel(w_down.grad, dr.grad) < 3e-2
    assert _rel(topw.grad, twr.grad) < 3e-2


@pytest.mark.parametrize("T,E,k,dt", [(1000, 32, 4, torch.bfloat16), (777, 64, 8, torch.float32),
                                      (300, 256, 16, torch.bfloat16), (50, 8, 2, torch.float32),
                                      (333, 12, 3, torch.float32), (129, 100, 5, torch.bfloat16)])
def test_router_topk_vs_torch(T, E, k, dt):
    from oxidizr_b200.models.moe import aux_from_usage, route
    from oxidizr_b200.ops.moe_kernels import RouterTopK
    torch.manual_seed(T + E)
    # distinct, exactly representable logits per row: no ties, so the top-k order is unique
    perm = torch.stack([torch.randperm(E) for _ in range(T)]).float()
    logits = ((perm - E / 2) / 32).to("cuda", dt).requires_grad_()
    topi, topw, usage, counts = RouterTopK.apply(logits, k)
    cw = torch.randn(T, k, device="cuda")
    aux = aux_from_usage(usage, counts, T * k, E, "mean_sq")
    ((topw * cw).sum() + 3.0 * aux).backward()
    lr = logits.detach().float().requires_grad_()
    probs, ti, tw = route(lr, k)
    assert torch.equal(topi.cpu(), ti.cpu())
    assert torch.allclose(topw, tw, atol=1e-5, rtol=1e-4)
    assert torch.allclose(usage, probs.mean(0), atol=1e-6, rtol=1e-4)
    assert torch.equal(counts.long().cpu(), torch.bincount(ti.reshape(-1), minlength=E).cpu())
    ((tw * cw).sum() + 3.0 * probs.mean(0).pow(2).mean()).backward()
    assert _rel(logits.grad, lr.grad) < (1e-2 if dt == torch.bfloat16 else 1e-4)


@pytest.mark.parametrize("T,N,ld", [(300, 1284, 1284), (4096, 256, 264), (5, 7, 7)])
def test_colsum_bias_grad_kernel(T, N, ld):
    from oxidizr_b200.ops._C import ext
    torch.manual_seed(3)
    x = torch.randn(T, ld, device="cuda").bfloat16()[:, :N]
    out = torch.ones(N, device="cuda")
    ext().colsum_add(x, out)
    ref = 1 + x.double().sum(0)
    assert torch.allclose(out.double(), ref, rtol=1e-4, atol=1e-3)
