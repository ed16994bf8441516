"""tcgen05 GEMM vs an fp32 PyTorch reference (all operand layouts, epilogues)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, a_t, b_t):
    A = (a.t() if a_t else a).float()
    B = (b.t() if b_t else b).float()
    return A @ B.t()


def _rel(x, y):
    return ((x.float() - y.float()).norm() / y.float().norm().clamp_min(1e-6)).item()


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 520, 200), (1024, 768, 512), (77, 1000, 136)])
def test_gemm_layouts(a_t, b_t, M, N, K):
    from oxidizr_b200.ops.gemm import mm
    from oxidizr_b200.ops._C import check_status
    torch.manual_seed(0)
    dev = "cuda"
    a = torch.randn((K, M) if a_t else (M, K), device=dev).bfloat16()
    b = torch.randn((K, N) if b_t else (N, K), device=dev).bfloat16()
    # MN-major operands need 16-byte aligned rows: pad storage when needed
    if a_t and M % 8:
        a = torch.nn.functional.pad(a, (0, 8 - M % 8))[:, :M]
    if b_t and N % 8:
        b = torch.nn.functional.pad(b, (0, 8 - N % 8))[:, :N]
    if not a_t and K % 8:
        a = torch.nn.functional.pad(a, (0, 8 - K % 8))[:, :K]
    if not b_t and K % 8:
        b = torch.nn.functional.pad(b, (0, 8 - K % 8))[:, :K]
    ref = _ref(a, b, a_t, b_t)
    out = mm(a, b, a_t=a_t, b_t=b_t)
    torch.cuda.synchronize()
    check_status(dev)
    assert _rel(out, ref) < 1e-2
    out32 = mm(a, b, a_t=a_t, b_t=b_t, out_dtype=torch.float32)
    assert _rel(out32, ref) < 1e-5 * K ** 0.5 + 1e-4
    # accumulate: out32 += A B^T
    mm(a, b, a_t=a_t, b_t=b_t, out=out32, beta=1.0)
    assert _rel(out32, 2 * ref) < 1e-4


def test_gemm_residual_inplace():
    from oxidizr_b200.ops.gemm import mm
    torch.manual_seed(1)
    x = torch.randn(512, 1024, device="cuda").bfloat16()
    w = torch.randn(768, 1024, device="cuda").bfloat16()
    r = torch.randn(512, 768, device="cuda").bfloat16()
    ref = _ref(x, w, False, False) + r.float()
    rr = r.clone()
    mm(x, w, out=rr, resid=rr)
    assert _rel(rr, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(300, 520, 200), (256, 1000, 512)])
def test_gemm_bias_epilogue(M, N, K):
    from oxidizr_b200.ops.gemm import mm
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    bias = torch.randn(N, device="cuda").bfloat16()
    r = torch.randn(M, N, device="cuda").bfloat16()
    ref = _ref(x, w, False, False) + bias.float()
    assert _rel(mm(x, w, bias=bias), ref) < 1e-2
    assert _rel(mm(x, w, bias=bias, resid=r), ref + r.float()) < 1e-2


def test_gemm_unaligned_rows_take_the_plain_path():
    """Rows that are not 16-byte aligned (a 4-wide projection) give the right answer."""
    from oxidizr_b200.ops.gemm import mm
    torch.manual_seed(4)
    dy = torch.randn(256, 4, device="cuda").bfloat16()
    w = torch.randn(4, 256, device="cuda").bfloat16()
    out = mm(dy, w, b_t=True)
    assert _rel(out, dy.float() @ w.float()) < 1e-2


def test_gemm_swiglu_fwd_bwd():
    from oxidizr_b200.ops._C import ext, status
    torch.manual_seed(2)
    M, H, I = 384, 512, 640
    x = (0.5 * torch.randn(M, H, device="cuda")).bfloat16()
    wg = (torch.randn(I, H, device="cuda") / H ** 0.5).bfloat16()
    wu = (torch.randn(I, H, device="cuda") / H ** 0.5).bfloat16()
    # interleave rows in blocks of 128: [g0..127, u0..127, g128.., u128..]
    w = torch.stack([wg.view(I // 128, 128, H), wu.view(I // 128, 128, H)], 1).reshape(2 * I, H).contiguous()
    h = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    ext().gemm_swiglu(x, w, h, gu, status("cuda"))
    g = x.float() @ wg.float().t()
    u = x.float() @ wu.float().t()
    ref = torch.nn.functional.silu(g) * u
    assert _rel(h, ref) < 1e-2
    gu_ref = torch.stack([g.view(M, I // 128, 128), u.view(M, I // 128, 128)], 2).reshape(M, 2 * I)
    assert _rel(gu, gu_ref) < 1e-2
    # backward: dh = dy @ w_down ; dg, du
    wd = (torch.randn(H, I, device="cuda") / I ** 0.5).bfloat16()
    dy = torch.randn(M, H, device="cuda").bfloat16()
    dgu = torch.empty_like(gu)
    ext().gemm_swiglu_bwd(dy, wd, gu, dgu, status("cuda"))
    dh = dy.float() @ wd.float()
    gb = gu.float().view(M, I // 128, 2, 128)
    gg, uu = gb[:, :, 0].reshape(M, I), gb[:, :, 1].reshape(M, I)
    s = torch.sigmoid(gg)
    dg = dh * uu * s * (1 + gg * (1 - s))
    du = dh * gg * s
    ref2 = torch.stack([dg.view(M, I // 128, 128), du.view(M, I // 128, 128)], 2).reshape(M, 2 * I)
    assert _rel(dgu, ref2) < 2e-2
    # the split form: plain dX GEMM, then the element-wise SwiGLU backward
    from oxidizr_b200.ops.gemm import mm
    dgu2 = torch.empty_like(gu)
    ext().swiglu_bwd(mm(dy, wd, b_t=True), gu, dgu2)
    assert _rel(dgu2, ref2) < 2e-2


def test_gemm_ce_partials():
    from oxidizr_b200.ops._C import ext, status
    torch.manual_seed(3)
    M, K, V = 300, 256, 1000
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(V, K, device="cuda") / K ** 0.5).bfloat16()
    tgt = torch.randint(0, V, (M,), device="cuda")
    tn = (V + 255) // 256
    pm = torch.empty(M, tn, device="cuda")
    ps = torch.empty(M, tn, device="cuda")
    tl = torch.empty(M, device="cuda")
    logits = torch.empty(M, 1008, device="cuda", dtype=torch.bfloat16)
    ext().gemm_ce(x, w, tgt, pm, ps, tl, logits, 1.0, status("cuda"))
    ref = x.float() @ w.float().t()
    lse = torch.logsumexp(ref, -1)
    lse_k = (pm + ps.log()).logsumexp(-1)
    assert torch.allclose(lse_k, lse, atol=2e-3, rtol=1e-4)
    assert torch.allclose(tl, ref.gather(1, tgt[:, None])[:, 0], atol=2e-3, rtol=1e-3)
    assert _rel(logits[:, :V], ref) < 1e-2


@pytest.mark.parametrize("hd", [64, 128])
def test_gemm_rope(hd):
    from oxidizr_b200.ops._C import ext, status
    torch.manual_seed(4)
    S, B, H = 64, 3, 256
    nh, kvh = 4, 2
    M = B * S
    N = (nh + 2 * kvh) * hd
    x = torch.randn(M, H, device="cuda").bfloat16()
    w = (torch.randn(N, H, device="cuda") / H ** 0.5).bfloat16()
    inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device="cuda").float() / hd))
    f = torch.arange(S, device="cuda").float()[:, None] * inv[None]
    cos, sin = f.cos().contiguous(), f.sin().contiguous()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm_rope(x, w, out, cos, sin, hd, nh * hd, kvh * hd, status("cuda"))
    y = (x.float() @ w.float().t()).view(B, S, nh + 2 * kvh, hd)
    c = torch.cat([cos, cos], -1)[None, :, None]
    s = torch.cat([sin, sin], -1)[None, :, None]
    rot = torch.cat([-y[..., hd // 2:], y[..., :hd // 2]], -1)
    yr = y * c + rot * s
    ref = torch.cat([yr[:, :, :nh + kvh], y[:, :, nh + kvh:]], 2).reshape(M, N)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 512, 4096), (128, 2048, 16384), (300, 1000, 3000)])
def test_gemm_splitk_accumulate(M, N, K):
    """Few output tiles and long K: the f32 accumulate path splits K across CTAs."""
    from oxidizr_b200.ops.gemm import mm
    torch.manual_seed(5)
    a = torch.randn(K, M, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    if M % 8:
        a = torch.nn.functional.pad(a, (0, 8 - M % 8))[:, :M]
    if N % 8:
        b = torch.nn.functional.pad(b, (0, 8 - N % 8))[:, :N]
    base = torch.randn(M, N, device="cuda")
    out = base.clone()
    mm(a, b, a_t=True, b_t=True, out=out, beta=1.0)
    ref = base + a.float().t() @ b.float()
    assert _rel(out, ref) < 1e-4


def test_gemm_first_cuda_call_of_a_new_thread():
    """Autograd runs backward on its own thread; a GEMM there may be the thread's first CUDA
    work, before any runtime call has made the context current (tensor-map encoding is a
    driver call)."""
    import threading
    from oxidizr_b200.ops._C import status
    from oxidizr_b200.ops.gemm import mm
    torch.manual_seed(0)
    a = torch.randn(512, 256, device="cuda").bfloat16()
    b = torch.randn(384, 256, device="cuda").bfloat16()
    out = torch.empty(512, 384, device="cuda", dtype=torch.bfloat16)
    status(a.device)
    torch.cuda.synchronize()
    err = []

    def work():
        try:
            mm(a, b, out=out)
        except Exception as e:  # noqa: BLE001 - reported below
            err.append(e)

    t = threading.Thread(target=work)
    t.start()
    t.join()
    assert not err, err
    torch.cuda.synchronize()
    ref = a.float() @ b.float().t()
    assert (out.float() - ref).abs().max().item() < 0.05 * ref.abs().max().item()
