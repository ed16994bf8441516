"""Sparse mixture-of-experts compute over the grouped tcgen05 GEMMs (csrc/moe.cu).

Forward: counting-sort permutation of token rows into 256-aligned expert
segments; one grouped GEMM for every expert's gate|up projection with the
SwiGLU epilogue; one grouped GEMM for every expert's down projection; a
weighted combine (fused with the residual add).  Backward mirrors it with the
SwiGLU-backward epilogue, two per-expert weight-gradient GEMMs reducing over
each expert's token segment, and a gather-sum back to token order.  No host
synchronisation: segment offsets stay on the device.

Upstream: ``Router`` model.rs:485-499, ``MoeLayer::forward`` model.rs:541-593 (dense loop
model.rs:561-565, aux loss model.rs:585-590), ``top_k`` model.rs:604-654, routing matrix model.rs:722-751.
"""
from __future__ import annotations

import torch

from ._C import ext, status
from .fused import _ready


def rows_capacity(T: int, k: int, E: int) -> int:
    # expert segments start on 256-row boundaries (MOE_SEG_ALIGN, CTA-pair tiles)
    return ((T * k + E * 256) + 255) // 256 * 256


def swiglu_bwd_grouped(dy, w_down, gu, dgu, E, seg, st):
    """dGU of every expert's SwiGLU from the down projection's output gradient: the
    grouped dX GEMM with a plain epilogue, then the element-wise SwiGLU backward
    (or the fused epilogue with OXI_SWIGLU_BWD=fused, see ops/fused.py)."""
    from .fused import SWIGLU_BWD_SPLIT
    _, H, I = w_down.shape
    if SWIGLU_BWD_SPLIT:
        dh = torch.empty(dy.shape[0], I, dtype=dy.dtype, device=dy.device)
        ext().gemm_grouped(1, 0, dy, False, w_down.view(E * H, I), True, E, seg, H, dh, None, None, st)
        ext().swiglu_bwd(dh, gu, dgu)
    else:
        ext().gemm_grouped(1, 3, dy, False, w_down.view(E * H, I), True, E, seg, H, dgu, None, gu, st)


def _wgrad_grouped(p, a, b, seg, E):
    """dW[e] = a[seg_e]^T b[seg_e] accumulated into p.main_grad (or returned)."""
    mg = getattr(p, "main_grad", None)
    out = mg if mg is not None else torch.zeros(p.shape, dtype=torch.float32, device=p.device)
    ext().gemm_grouped(2, 1, a, True, b, True, E, seg, 0, out, None, None, status(a.device))
    if mg is not None:
        _ready(p)
        return None
    return out.to(p.dtype)


class GroupedExperts(torch.autograd.Function):
    """resid + sum_j topw[t, j] * SwiGLU_{topi[t, j]}(x_t) over the experts held here.

    x [T, H] bf16, topi [T, k] int64 (local expert ids), topw [T, k] f32,
    w_gu [E, 2I, H] (gate|up rows interleaved in 128-row blocks), w_down [E, H, I].
    """

    @staticmethod
    def forward(ctx, x, topi, topw, w_gu, w_down, resid):
        T, H = x.shape
        k = topi.shape[1]
        E, I2, _ = w_gu.shape
        I = I2 // 2
        cap = rows_capacity(T, k, E)
        xc = x if x.stride(1) == 1 else x.contiguous()
        counts, seg, pos, xp = ext().moe_permute(xc, topi.contiguous(), E, cap)
        h = torch.empty(cap, I, dtype=x.dtype, device=x.device)
        gu = torch.empty(cap, I2, dtype=x.dtype, device=x.device)
        st = status(x.device)
        ext().gemm_grouped(1, 2, xp, False, w_gu.view(E * I2, H), False, E, seg, I2, h, gu, None, st)
        yp = torch.empty(cap, H, dtype=x.dtype, device=x.device)
        ext().gemm_grouped(1, 0, h, False, w_down.view(E * H, I), False, E, seg, H, yp, None, None, st)
        tw = topw.float().contiguous()
        y = ext().moe_combine(yp, pos, tw, T, k, resid.contiguous() if resid is not None else None)
        ctx.save_for_backward(xp, h, gu, yp, pos, seg, counts, tw)
        ctx.w_gu, ctx.w_down, ctx.k, ctx.has_resid = w_gu, w_down, k, resid is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        xp, h, gu, yp, pos, seg, counts, tw = ctx.saved_tensors
        w_gu, w_down, k = ctx.w_gu, ctx.w_down, ctx.k
        E, I2, H = w_gu.shape
        I = I2 // 2
        T = dy.shape[0]
        dyc = dy.contiguous()
        st = status(dy.device)
        dyp, dtw = ext().moe_combine_bwd(dyc, yp, pos, tw, k)
        ext().moe_zero_pad(seg, counts, dyp)
        g_down = _wgrad_grouped(w_down, dyp, h, seg, E)
        dgu = torch.empty_like(gu)
        swiglu_bwd_grouped(dyp, w_down, gu, dgu, E, seg, st)
        g_gu = _wgrad_grouped(w_gu, dgu, xp, seg, E)
        dxp = torch.empty_like(xp)
        ext().gemm_grouped(1, 0, dgu, False, w_gu.view(E * I2, H), True, E, seg, I2, dxp, None, None, st)
        dx = ext().moe_gather_sum(dxp, pos, T, k)
        return dx, None, dtw, g_gu, g_down, (dy if ctx.has_resid else None)


def grouped_ok(x: torch.Tensor, w_gu: torch.Tensor) -> bool:
    E, I2, H = w_gu.shape
    return (x.is_cuda and x.dtype == torch.bfloat16 and I2 % 256 == 0 and H % 64 == 0
            and hasattr(ext(), "gemm_grouped"))


class RouterTopK(torch.autograd.Function):
    """Softmax router + top-k + renormalised weights + mean probability (csrc/router.cu).

    Returns ``(topi [T,k] int64, topw [T,k] f32, usage [E] f32, counts [E] int32)``;
    ``usage`` (mean routing probability per expert) and ``topw`` carry gradients.
    """

    @staticmethod
    def forward(ctx, logits, k: int):
        topi, topw, usage, counts = ext().router_fwd(logits, int(k))
        ctx.save_for_backward(logits, topi, topw)
        ctx.mark_non_differentiable(topi, counts)
        return topi, topw, usage, counts

    @staticmethod
    def backward(ctx, _dtopi, dtopw, dusage, _dcounts):
        logits, topi, topw = ctx.saved_tensors
        dtopw = torch.zeros_like(topw) if dtopw is None else dtopw.float().contiguous()
        du = None if dusage is None else dusage.float().contiguous()
        return ext().router_bwd(logits, topi, topw, dtopw, du), None


def router_ok(logits, k: int) -> bool:
    return (logits.is_cuda and logits.dim() == 2 and logits.shape[1] <= 256 and k <= 16
            and logits.dtype in (torch.bfloat16, torch.float32) and hasattr(ext(), "router_fwd"))
