"""Kernel micro-benchmarks timed with CUDA events (warm-up, L2 flush between
iterations, synchronize on both sides), reported against the measured peaks in
``MEASURED_PEAKS.json`` when present.

Usage::

    python -m oxidizr_b200.utils.kbench gemm [--shapes M,N,K ...]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def measured_peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


_FLUSH = {}


def flush_l2(device=None):
    """Write a buffer larger than the 126 MB L2."""
    dev = torch.device(device or "cuda")
    buf = _FLUSH.get(dev)
    if buf is None:
        buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
        _FLUSH[dev] = buf
    buf.zero_()


def time_fn(fn, iters: int = 20, warmup: int = 5, flush: bool = True) -> float:
    """Median milliseconds per call."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)


def bench_gemm(shapes, iters=20):
    from ..ops.gemm import mm
    peaks = measured_peaks()
    rows = []
    for (M, N, K, lay) in shapes:
        # layout: a_t / b_t letters (n: K-major, t: MN-major), "+" for an f32 += output (the
        # weight-gradient form: beta 1, split-K when the tiles do not fill the GPU)
        a_t, b_t, acc = lay[0] == "t", lay[1] == "t", lay.endswith("+")
        a = torch.randn((K, M) if a_t else (M, K), device="cuda").bfloat16()
        b = torch.randn((K, N) if b_t else (N, K), device="cuda").bfloat16()
        out = torch.zeros(M, N, device="cuda", dtype=torch.float32 if acc else torch.bfloat16)
        if acc:
            ms = time_fn(lambda: mm(a, b, a_t=a_t, b_t=b_t, out=out, beta=1.0), iters)
        else:
            ms = time_fn(lambda: mm(a, b, a_t=a_t, b_t=b_t, out=out), iters)
        A = a.t() if a_t else a
        B = b.t() if b_t else b
        ms_ref = time_fn(lambda: torch.matmul(A, B.t()), iters)
        tf = 2.0 * M * N * K / ms / 1e9
        tf_ref = 2.0 * M * N * K / ms_ref / 1e9
        rows.append({"M": M, "N": N, "K": K, "layout": lay, "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac_of_peak": round(tf / peaks["bf16_tflops"], 3), "peak_source": peaks["source"],
                     "torch_ms": round(ms_ref, 4), "torch_tflops": round(tf_ref, 1)})
        print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_attn(B=8, S=2048, Hq=16, Hk=8, D=128, iters=20):
    """Causal attention fwd and fwd+bwd vs torch SDPA; FLOPs count the causal half."""
    import math
    from ..ops.flash import FlashAttentionQKV
    peaks = measured_peaks()
    N = (Hq + 2 * Hk) * D
    qkv = torch.randn(B, S, N, device="cuda").bfloat16().requires_grad_()
    scale = 1.0 / math.sqrt(D)
    flops_f = 4.0 * B * Hq * S * S * D / 2
    def ours_f():
        with torch.no_grad():
            FlashAttentionQKV.apply(qkv, Hq, Hk, D, scale, True)
    do = torch.randn(B, S, Hq * D, device="cuda").bfloat16()
    def ours_fb():
        o = FlashAttentionQKV.apply(qkv, Hq, Hk, D, scale, True)
        o.backward(do)
    q = qkv[..., :Hq * D].view(B, S, Hq, D).transpose(1, 2)
    k = qkv[..., Hq * D:(Hq + Hk) * D].view(B, S, Hk, D).transpose(1, 2)
    v = qkv[..., (Hq + Hk) * D:].view(B, S, Hk, D).transpose(1, 2)
    sd = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale,
                                                                   enable_gqa=Hk != Hq)
    def ref_f():
        with torch.no_grad():
            sd()
    def ref_fb():
        o = sd()
        o.backward(do.view(B, S, Hq, D).transpose(1, 2))
    res = {}
    for name, fn, fl in (("ours_fwd", ours_f, flops_f), ("ours_fwd_bwd", ours_fb, 3.5 * flops_f),
                         ("sdpa_fwd", ref_f, flops_f), ("sdpa_fwd_bwd", ref_fb, 3.5 * flops_f)):
        ms = time_fn(fn, iters)
        res[name] = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1),
                     "frac_of_peak": round(fl / ms / 1e9 / peaks["bf16_tflops"], 3)}
    out = {"B": B, "S": S, "Hq": Hq, "Hk": Hk, "D": D, "peak_source": peaks["source"], **res}
    print(json.dumps(out), flush=True)
    return out


def bench_attn_mla(B=16, S=1024, H=12, Dqk=96, Dv=64, iters=20):
    """Multi-head latent attention shapes (q/k carry a RoPE part): ours vs torch SDPA."""
    import math
    from ..ops.flash import FlashAttention
    peaks = measured_peaks()
    q = torch.randn(B, S, H, Dqk, device="cuda").bfloat16().requires_grad_()
    k = torch.randn(B, S, H, Dqk, device="cuda").bfloat16().requires_grad_()
    v = torch.randn(B, S, H, Dv, device="cuda").bfloat16().requires_grad_()
    do = torch.randn(B, S, H, Dv, device="cuda").bfloat16()
    scale = 1.0 / math.sqrt(Dqk)
    flops_f = 2.0 * B * H * S * S * (Dqk + Dv) / 2
    def ours_f():
        with torch.no_grad():
            FlashAttention.apply(q, k, v, scale, True)
    def ours_fb():
        FlashAttention.apply(q, k, v, scale, True).backward(do)
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
    sd = lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=True, scale=scale)
    def ref_f():
        with torch.no_grad():
            sd()
    def ref_fb():
        sd().backward(do.transpose(1, 2))
    res = {}
    for name, fn, fl in (("ours_fwd", ours_f, flops_f), ("ours_fwd_bwd", ours_fb, 3.5 * flops_f),
                         ("sdpa_fwd", ref_f, flops_f), ("sdpa_fwd_bwd", ref_fb, 3.5 * flops_f)):
        ms = time_fn(fn, iters)
        res[name] = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1),
                     "frac_of_peak": round(fl / ms / 1e9 / peaks["bf16_tflops"], 3)}
    out = {"mla": True, "B": B, "S": S, "H": H, "Dqk": Dqk, "Dv": Dv, "peak_source": peaks["source"], **res}
    print(json.dumps(out), flush=True)
    return out


def bench_ce(shapes=((16384, 2048, 128354), (16384, 768, 100277)), iters=5, chunks=(4096, 8192, 16384)):
    """lm_head + cross-entropy forward + backward, logits materialised vs logit-free
    (chunked recompute): device time and peak extra memory at the bench configs' shapes."""
    import os
    from ..ops import fused
    peaks = measured_peaks()
    out = []
    for (T, H, V) in shapes:
        x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
        w = (torch.randn(V, H, device="cuda") / H ** 0.5).bfloat16().requires_grad_()
        w.main_grad = torch.zeros(V, H, device="cuda")
        t = torch.randint(0, V, (T,), device="cuda")

        def step():
            x.grad = None
            fused.LinearCrossEntropy.apply(x, w, t, -100).backward()

        row = {"T": T, "H": H, "V": V, "gemm_flops_per_gemm": 2.0 * T * V * H}
        for mode, chunk in [("full", None)] + [("chunked", c) for c in chunks]:
            os.environ["OXI_CE_MODE"] = mode
            if chunk:
                fused.CE_CHUNK = chunk
            torch.cuda.synchronize()
            base = torch.cuda.memory_allocated()
            torch.cuda.reset_peak_memory_stats()
            ms = time_fn(step, iters, warmup=2)
            peak = torch.cuda.max_memory_allocated() - base
            key = mode if chunk is None else f"chunked_{chunk}"
            gemms = 3 if mode == "full" else 4
            row[key] = {"ms": round(ms, 3), "peak_extra_gb": round(peak / 1e9, 2),
                        "tflops": round(gemms * row["gemm_flops_per_gemm"] / ms / 1e9, 1),
                        "frac_of_peak": round(gemms * row["gemm_flops_per_gemm"] / ms / 1e9
                                              / peaks["bf16_tflops"], 3)}
        os.environ.pop("OXI_CE_MODE", None)
        print(json.dumps(row), flush=True)
        out.append(row)
        del x, w, t
        torch.cuda.empty_cache()
    return out


def bench_moe_gemms(T=16384, H=2048, E=64, k=8, I=1024, iters=10):
    """The six grouped expert GEMMs of one MoE layer at the MoE config's per-GPU shape
    (one GPU holding all experts): useful TFLOP/s counts real rows only (set
    OXI_GEMM_CG=1 to time single-CTA tiles instead of CTA pairs)."""
    import os
    from ..ops._C import ext, status
    from ..ops.moe_kernels import rows_capacity, swiglu_bwd_grouped
    peaks = measured_peaks()
    torch.manual_seed(0)
    x = (torch.randn(T, H, device="cuda") * 0.5).bfloat16()
    topi = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)]) if T <= 4096 else \
        torch.randint(0, E, (T, k), device="cuda")
    cap = rows_capacity(T, k, E)
    counts, seg, pos, xp = ext().moe_permute(x, topi.contiguous(), E, cap)
    wgu = (torch.randn(E, 2 * I, H, device="cuda") * 0.02).bfloat16()
    wd = (torch.randn(E, H, I, device="cuda") * 0.02).bfloat16()
    h = torch.empty(cap, I, dtype=torch.bfloat16, device="cuda")
    gu = torch.empty(cap, 2 * I, dtype=torch.bfloat16, device="cuda")
    yp = torch.empty(cap, H, dtype=torch.bfloat16, device="cuda")
    dyp = torch.randn(cap, H, device="cuda").bfloat16()
    dgu = torch.empty_like(gu)
    dxp = torch.empty_like(xp)
    g_gu = torch.zeros(E, 2 * I, H, device="cuda")
    g_d = torch.zeros(E, H, I, device="cuda")
    st = status("cuda")
    rows = T * k
    cases = {
        "gate_up_swiglu": (lambda: ext().gemm_grouped(1, 2, xp, False, wgu.view(E * 2 * I, H), False, E, seg, 2 * I,
                                                      h, gu, None, st), 2.0 * rows * 2 * I * H),
        "down": (lambda: ext().gemm_grouped(1, 0, h, False, wd.view(E * H, I), False, E, seg, H, yp, None, None, st),
                 2.0 * rows * H * I),
        "down_dx_swiglu_bwd": (lambda: swiglu_bwd_grouped(dyp, wd, gu, dgu, E, seg, st), 2.0 * rows * H * I),
        "down_wgrad": (lambda: ext().gemm_grouped(2, 1, dyp, True, h, True, E, seg, 0, g_d, None, None, st),
                       2.0 * rows * H * I),
        "gate_up_dx": (lambda: ext().gemm_grouped(1, 0, dgu, False, wgu.view(E * 2 * I, H), True, E, seg, 2 * I, dxp,
                                                  None, None, st), 2.0 * rows * 2 * I * H),
        "gate_up_wgrad": (lambda: ext().gemm_grouped(2, 1, dgu, True, xp, True, E, seg, 0, g_gu, None, None, st),
                          2.0 * rows * 2 * I * H),
    }
    out = {"T": T, "E": E, "k": k, "H": H, "I": I, "rows_per_expert": rows / E, "cap": cap,
           "tiles": "single-CTA" if os.environ.get("OXI_GEMM_CG") == "1" else "CTA pairs"}
    for name, (fn, fl) in cases.items():
        ms = time_fn(fn, iters)
        out[name] = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1),
                     "frac_of_peak": round(fl / ms / 1e9 / peaks["bf16_tflops"], 3)}
    print(json.dumps(out), flush=True)
    return out


def bench_ssm(iters=10):
    """Selective-scan kernels at the hybrid (Mamba2) and Mamba3 bench shapes: time and the
    effective HBM rate of the scan inputs/outputs (f32)."""
    from ..ops import ssm
    peaks = measured_peaks()
    out = []
    for name, (B, S, H, P, N, three) in (("mamba2_cfg3", (16, 1024, 24, 64, 128, False)),
                                         ("mamba3_cfg4", (4, 4096, 32, 256, 128, True))):
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(B, S, H, P, device="cuda", generator=g).bfloat16().requires_grad_()
        dt = (torch.rand(B, S, H, device="cuda", generator=g) * 0.1 + 0.001).requires_grad_()
        A = -torch.rand(H, device="cuda", generator=g) - 0.5
        Bm = torch.randn(B, S, H if three else 1, N, device="cuda", generator=g).requires_grad_()
        Cm = torch.randn(B, S, H if three else 1, N, device="cuda", generator=g).requires_grad_()
        lam = torch.rand(B, S, H, device="cuda", generator=g).requires_grad_()
        if three:
            f = lambda: ssm.mamba3_scan(x, dt, A, Bm, Cm, lam, 256)
        else:
            f = lambda: ssm.ssd(x, dt, A, Bm, Cm, 256)
        dy = torch.randn(B, S, H, P, device="cuda", generator=g)
        def fwd():
            with torch.no_grad():
                f()
        def fb():
            f().backward(dy)
        ms_f = time_fn(fwd, iters)
        ms_fb = time_fn(fb, iters)
        # algorithmic f32 bytes of the scan: x, y, B, C, per-step scalars (fwd); x, y, dy, dx, B, C, dB, dC (bwd)
        nb = 4.0 * B * S * (H * P * 2 + 2 * (H if three else 1) * N + 3 * H)
        row = {"name": name, "B": B, "S": S, "H": H, "P": P, "N": N, "fwd_ms": round(ms_f, 3),
               "fwd_bwd_ms": round(ms_fb, 3), "fwd_GBps": round(nb / ms_f / 1e6, 1),
               "fwd_frac_of_hbm": round(nb / ms_f / 1e6 / peaks["hbm_gbs"], 3)}
        print(json.dumps(row), flush=True)
        out.append(row)
    return out


def run_once(what: str):
    """Launch one kernel of a small case a few times (targets for ncu captures)."""
    import math
    torch.manual_seed(0)
    if what in ("fa_fwd", "fa_bwd"):
        from ..ops.flash import FlashAttentionQKV
        B, S, Hq, Hk, D = 4, 2048, 16, 8, 128  # 512 backward CTAs: several waves, like the bench shape
        qkv = torch.randn(B, S, (Hq + 2 * Hk) * D, device="cuda").bfloat16().requires_grad_()
        for _ in range(3):
            o = FlashAttentionQKV.apply(qkv, Hq, Hk, D, 1.0 / math.sqrt(D), True)
            if what == "fa_bwd":
                o.backward(torch.ones_like(o))
    elif what in ("gemm", "gemm_torch"):
        # the same 8192 x 8192 x 4096 NN product through our kernel or through torch
        # (cuBLAS): the pair of captures compares the two kernels' counters
        from ..ops.gemm import mm
        a = torch.randn(8192, 4096, device="cuda").bfloat16()
        b = torch.randn(8192, 4096, device="cuda").bfloat16()
        for _ in range(3):
            if what == "gemm":
                mm(a, b)
            else:
                torch.matmul(a, b.t())
    elif what == "gemm_dw":
        from ..ops.gemm import mm
        a = torch.randn(16384, 2048, device="cuda").bfloat16()
        b = torch.randn(16384, 2048, device="cuda").bfloat16()
        out = torch.zeros(2048, 2048, device="cuda")
        for _ in range(3):
            mm(a, b, a_t=True, b_t=True, out=out, beta=1.0)
    elif what in ("ssd_m2", "ssd_m3"):
        # one tensor-core SSD forward + backward: the hybrid's Mamba2 shape at batch 4,
        # or the Mamba3 shape at batch 1 (P = 256 after the MIMO up-projection)
        from ..ops.ssd_tc import ssd_tc
        B, S, H, P = (4, 1024, 24, 64) if what == "ssd_m2" else (1, 4096, 32, 256)
        G = 1 if what == "ssd_m2" else H
        x = torch.randn(B, S, H, P, device="cuda").bfloat16().requires_grad_()
        dt = (torch.rand(B, S, H, device="cuda") * 0.1 + 0.001).requires_grad_()
        A = -torch.rand(H, device="cuda") - 0.5
        Bm = torch.randn(B, S, G, 128, device="cuda").bfloat16().requires_grad_()
        Cm = torch.randn(B, S, G, 128, device="cuda").bfloat16().requires_grad_()
        for _ in range(3):
            ssd_tc(x, dt, A, Bm, Cm).backward(torch.ones(B, S, H, P, device="cuda"))
    elif what == "norm":
        # RMSNorm forward + backward at the Llama shape (16384 tokens x 2048), x 64 MB
        from ..ops import api
        x = torch.randn(16384, 2048, device="cuda").bfloat16().requires_grad_()
        w = torch.nn.Parameter(torch.ones(2048, device="cuda").bfloat16())
        for _ in range(3):
            api.rmsnorm(x, w, 1e-5).backward(torch.ones(16384, 2048, device="cuda").bfloat16())
    elif what == "conv1d":
        # causal depthwise conv1d (k = 4) + SiLU at the hybrid's Mamba2 xBC shape
        from ..ops import api
        B, S, C = 16, 1024, 1792
        x = torch.randn(B, S, C, device="cuda").bfloat16().requires_grad_()
        w = torch.nn.Parameter((torch.randn(C, 1, 4, device="cuda") * 0.3).bfloat16())
        b = torch.nn.Parameter(torch.zeros(C, device="cuda").bfloat16())
        for _ in range(3):
            api.causal_conv1d(x, w, b, True).backward(torch.ones(B, S, C, device="cuda").bfloat16())
    elif what in ("swiglu", "qkv_rope"):
        # Llama shapes: gate/up GEMM with the SwiGLU epilogue + down GEMM, or the QKV GEMM
        # with the RoPE epilogue (16 q heads, 8 kv heads, head dim 128), forward + backward
        from ..ops import api
        T, H = 16384, 2048
        x = (torch.randn(T, H, device="cuda") * 0.5).bfloat16().requires_grad_()
        if what == "swiglu":
            wgu = torch.nn.Parameter((torch.randn(2 * 5632, H, device="cuda") * 0.02).bfloat16())
            wd = torch.nn.Parameter((torch.randn(H, 5632, device="cuda") * 0.02).bfloat16())
            f = lambda: api.swiglu_mlp(x, wgu, wd)
            gy = torch.ones(T, H, device="cuda").bfloat16()
        else:
            w = torch.nn.Parameter((torch.randn(4096, H, device="cuda") * 0.02).bfloat16())
            ang = torch.arange(2048, device="cuda")[:, None].float() * torch.pow(
                10000.0, -torch.arange(64, device="cuda").float() / 64)[None, :]
            cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
            xs = x.view(8, 2048, H)
            f = lambda: api.qkv_rope(xs, w, cos, sin, 128, 2048, 1024)
            gy = torch.ones(8, 2048, 4096, device="cuda").bfloat16()
        for _ in range(3):
            f().backward(gy)
    elif what == "ce":
        # lm_head GEMM with the cross-entropy epilogue over the 128354-token vocabulary, 4096 tokens
        from ..ops import api
        T, H, V = 4096, 2048, 128354
        x = (torch.randn(T, H, device="cuda") * 0.5).bfloat16().requires_grad_()
        w = torch.nn.Parameter((torch.randn(V, H, device="cuda") * 0.02).bfloat16())
        tgt = torch.randint(0, V, (T,), device="cuda")
        for _ in range(3):
            api.linear_cross_entropy(x, w, tgt).backward()
    elif what == "fa_mla":
        # latent attention of the hybrid config: 12 heads, q/k head dim 64 + 32 RoPE, v 64
        from ..ops.flash import FlashAttention
        B, S, H, Dqk, Dv = 4, 1024, 12, 96, 64
        q = torch.randn(B, S, H, Dqk, device="cuda").bfloat16().requires_grad_()
        k = torch.randn(B, S, H, Dqk, device="cuda").bfloat16().requires_grad_()
        v = torch.randn(B, S, H, Dv, device="cuda").bfloat16().requires_grad_()
        for _ in range(3):
            FlashAttention.apply(q, k, v, 1.0 / math.sqrt(Dqk), True).backward(
                torch.ones(B, S, H, Dv, device="cuda").bfloat16())
    elif what == "mla_pack":
        # MLA operand packing of the hybrid config (12 heads, head dim 64, rope dim 32, 16 x 1024 tokens)
        from ..models.common import RopeCache
        from ..ops.mla import MlaPack
        B, S, nh, hd, dr = 16, 1024, 12, 64, 32
        qc = torch.randn(B, S, nh * hd, device="cuda").bfloat16().requires_grad_()
        kv = torch.randn(B, S, 2 * nh * hd, device="cuda").bfloat16().requires_grad_()
        d = torch.randn(B, S, 768 + dr + nh * dr, device="cuda").bfloat16()
        rp = d[..., 768:].detach().requires_grad_()
        cos, sin = RopeCache.get(dr, S, 10000.0, "cuda")
        for _ in range(3):
            q, k, v = MlaPack.apply(qc, kv, rp, cos, sin, nh, hd, dr)
            (q.float().sum() + k.float().sum() + v.float().sum()).backward()
    elif what == "ce_chunked":
        # logit-free lm_head + cross-entropy backward (recomputed 8192-column chunks), 4096 tokens
        import os
        from ..ops import api
        os.environ["OXI_CE_MODE"] = "chunked"
        T, H, V = 4096, 2048, 128354
        x = (torch.randn(T, H, device="cuda") * 0.5).bfloat16().requires_grad_()
        w = torch.nn.Parameter((torch.randn(V, H, device="cuda") * 0.02).bfloat16())
        tgt = torch.randint(0, V, (T,), device="cuda")
        for _ in range(3):
            api.linear_cross_entropy(x, w, tgt).backward()
    elif what == "moe":
        # router top-8 of 64 + grouped expert SwiGLU GEMMs at the MoE config's shapes, 4096 tokens
        from ..ops.moe_kernels import GroupedExperts, RouterTopK
        T, H, E, k, I = 4096, 2048, 64, 8, 1024
        x = (torch.randn(T, H, device="cuda") * 0.5).bfloat16().requires_grad_()
        wr = torch.nn.Parameter((torch.randn(E, H, device="cuda") * 0.02).bfloat16())
        wgu = torch.nn.Parameter((torch.randn(E, 2 * I, H, device="cuda") * 0.02).bfloat16())
        wd = torch.nn.Parameter((torch.randn(E, H, I, device="cuda") * 0.02).bfloat16())
        for _ in range(3):
            topi, topw, usage, _ = RouterTopK.apply(x @ wr.t(), k)
            y = GroupedExperts.apply(x, topi, topw, wgu, wd, None)
            (y.float().sum() + usage.sum()).backward()
    elif what == "m3_bc":
        # Mamba3 B/C prologue (norm + bias + complex RoPE + <B, C>) at the Mamba3 config's
        # shape: 4 x 4096 tokens, 32 heads, one B/C group of state 128
        from ..ops.ssd_tc import Mamba3BC
        B, S, H, G = 4, 4096, 32, 1
        bc = torch.randn(B, S, 2 * G * 128, device="cuda").bfloat16().requires_grad_()
        w = torch.nn.Parameter(torch.ones(128, device="cuda").bfloat16())
        bb = torch.nn.Parameter(torch.ones(H, 128, device="cuda").bfloat16())
        cb = torch.nn.Parameter(torch.ones(H, 128, device="cuda").bfloat16())
        ang = torch.randn(B, S, H, 64, device="cuda") * 10
        for _ in range(3):
            bo, co, dot = Mamba3BC.apply(bc[..., :128], bc[..., 128:], w, bb, cb, ang, H, 1e-6)
            (bo.float().sum() + co.float().sum() + dot.sum()).backward()
    elif what == "mamba1":
        # Mamba1 selective scan forward + backward (state 16, f32 in / out) at a hidden-768 block:
        # 4 x 1024 tokens, d_inner 1536
        from ..ops.ssm_kernels import Mamba1Scan
        B, S, D, N = 4, 1024, 1536, 16
        u = torch.randn(B, S, D, device="cuda").requires_grad_()
        dl = (torch.rand(B, S, D, device="cuda") * 0.1).requires_grad_()
        A = (torch.rand(D, N, device="cuda") + 0.5).requires_grad_()
        Bm = torch.randn(B, S, N, device="cuda").requires_grad_()
        Cm = torch.randn(B, S, N, device="cuda").requires_grad_()
        for _ in range(3):
            Mamba1Scan.apply(u, dl, A, Bm, Cm, 30.0).backward(torch.ones(B, S, D, device="cuda"))
    elif what == "adamw":
        # global-norm + clip + AdamW over 128 M bf16 parameters (f32 master, m, v, grad)
        from ..optim import AdamW, AdamWConfig, FlatParams
        p = torch.nn.Parameter((torch.randn(128 << 20, device="cuda") * 0.02).bfloat16())
        opt = AdamW(FlatParams([("w", p)], torch.device("cuda")), AdamWConfig(lr=1e-4, max_grad_norm=1.0))
        for _ in range(3):
            opt.flat.grad.normal_()
            opt.step()
    else:
        raise SystemExit(f"unknown kernel target {what!r}")
    torch.cuda.synchronize()
    print(f"{what}: ok")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "attn", "ssm", "ce", "moe", "once"])
    ap.add_argument("--kernel", default="fa_fwd",
                    help="for 'once': fa_fwd | fa_bwd | fa_mla | gemm | gemm_torch | gemm_dw | ssd_m2 | ssd_m3 | norm | "
                         "conv1d | swiglu | qkv_rope | ce | ce_chunked | mla_pack | moe | m3_bc | mamba1 | adamw")
    ap.add_argument("--shapes", nargs="*", default=None,
                    help="M,N,K[,layout] with layout nn|nt|tt, a trailing + for an f32 += output")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    if args.what == "once":
        run_once(args.kernel)
        return
    if args.what == "attn":
        bench_attn(iters=args.iters)
        bench_attn(D=64, Hq=32, Hk=8, iters=args.iters)
        bench_attn_mla(iters=args.iters)
        return
    if args.what == "ssm":
        bench_ssm(iters=args.iters)
        return
    if args.what == "ce":
        bench_ce(iters=min(args.iters, 5))
        return
    if args.what == "moe":
        bench_moe_gemms(iters=min(args.iters, 10))
        bench_moe_gemms(T=16384, H=768, E=32, k=4, I=512, iters=min(args.iters, 10))
        return
    if args.what == "gemm":
        if args.shapes:
            shapes = []
            for s in args.shapes:
                parts = s.split(",")
                shapes.append((int(parts[0]), int(parts[1]), int(parts[2]), parts[3] if len(parts) > 3 else "nn"))
        else:
            T = 16384
            shapes = [(8192, 8192, 8192, "nn"), (T, 4096, 2048, "nn"), (T, 2048, 2048, "nn"),
                      (T, 11264, 2048, "nn"), (T, 2048, 5632, "nn"), (T, 2048, 5632, "nt"),
                      (5632, 2048, T, "tt"), (2048, 2048, T, "tt")]
        bench_gemm(shapes, args.iters)


if __name__ == "__main__":
    main()
