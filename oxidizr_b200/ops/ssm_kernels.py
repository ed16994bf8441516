"""Autograd functions over the SSM kernels (csrc/conv1d.cu, csrc/ssd.cu).

Upstream: causal conv1d mamba2.rs:344-352, mamba.rs:137-141; Mamba1 selective scan
mamba.rs:212-291; chunked SSD mamba2.rs:381-482; Mamba3 trapezoidal scan mamba3.rs:638-752.
"""
from __future__ import annotations

import torch

from ._C import ext
from .fused import _vec_grad


class CausalConv1d(torch.autograd.Function):
    """x [B, S, C] bf16 (rows may be strided), w [C, 1, K], bias [C] -> act(conv(x))."""

    @staticmethod
    def forward(ctx, x, w, bias, act: bool = True):
        B, S, C = x.shape
        x2 = x.reshape(B * S, C)
        if x2.stride(1) != 1 or x2.stride(0) % 8:
            x2 = x2.contiguous()
        y = torch.empty(B * S, C, dtype=x.dtype, device=x.device)
        ext().conv1d_fwd(x2, w, bias, y, B, S, act)
        ctx.save_for_backward(x2)
        ctx.w, ctx.bias, ctx.act, ctx.shape = w, bias, act, (B, S, C)
        return y.view(B, S, C)

    @staticmethod
    def backward(ctx, dy):
        (x2,) = ctx.saved_tensors
        B, S, C = ctx.shape
        w, bias = ctx.w, ctx.bias
        dy2 = dy.reshape(B * S, C)
        if dy2.stride(1) != 1 or dy2.stride(0) % 8:
            dy2 = dy2.contiguous()
        dx = torch.empty(B * S, C, dtype=x2.dtype, device=x2.device)
        dw = torch.zeros(w.numel(), dtype=torch.float32, device=x2.device)
        db = torch.zeros(C, dtype=torch.float32, device=x2.device) if bias is not None else None
        ext().conv1d_bwd(x2, w, bias, dy2, dx, dw, db, B, S, ctx.act)
        gw = _vec_grad(w, dw)
        gb = _vec_grad(bias, db) if bias is not None else None
        return dx.view(B, S, C), gw, gb, None


def _prep_bc(Bg: torch.Tensor, H: int):
    """[B, S, G, N] group tensor -> f32 per-head view for the kernel.  G == 1
    becomes a zero head-stride view (the kernel then sums dB over heads)."""
    Bg = Bg.float()
    G = Bg.shape[2]
    if G == H:
        return Bg.contiguous(), "full"
    if G == 1:
        return Bg.contiguous().expand(-1, -1, H, -1), "shared"
    return Bg.repeat_interleave(H // G, dim=2).contiguous(), "repeat"


def _fold_bc(dB: torch.Tensor, mode: str, G: int, shape):
    if mode == "full":
        return dB
    if mode == "shared":
        return dB[:, :, :1].contiguous()
    Bsz, S, H, N = dB.shape
    return dB.view(Bsz, S, G, H // G, N).sum(3)


class SSMScan(torch.autograd.Function):
    """h_t = exp(loga_t) h_{t-1} + gamma_t B_t x_t^T (+ beta_t B_{t-1} x_{t-1}^T); y_t = C_t h_t.

    x [B, S, H, P]; Bg/Cg [B, S, G, N] (G divides H); loga/gamma/beta [B, S, H] f32.
    Returns y [B, S, H, P] f32.
    """

    @staticmethod
    def forward(ctx, x, Bg, Cg, loga, gamma, beta=None):
        H = x.shape[2]
        xf = x.float().contiguous()
        Bh, mode = _prep_bc(Bg, H)
        Ch, _ = _prep_bc(Cg, H)
        la, ga = loga.float().contiguous(), gamma.float().contiguous()
        be = beta.float().contiguous() if beta is not None else None
        y = ext().ssm_scan_fwd(xf, Bh, Ch, la, ga, be)
        ctx.save_for_backward(xf, Bh, Ch, la, ga, be, y)
        ctx.mode, ctx.G, ctx.xdtype = mode, Bg.shape[2], x.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        xf, Bh, Ch, la, ga, be, y = ctx.saved_tensors
        dyc = dy.float().contiguous()
        dx, dB, dC, dgam, dbet = ext().ssm_scan_bwd(xf, Bh, Ch, la, ga, be, dyc)
        # d loga from q_t = <dy_t, y_t> + q_{t+1} - v_{t+1} and dloga_t = q_t - v_t
        e = (dyc * y).sum(-1)
        v = ga * dgam + (be * dbet if be is not None else 0.0)
        v_next = torch.cat([v[:, 1:], torch.zeros_like(v[:, :1])], 1)
        q = torch.flip(torch.cumsum(torch.flip(e - v_next, [1]), 1), [1])
        dla = q - v
        dBg = _fold_bc(dB, ctx.mode, ctx.G, None)
        dCg = _fold_bc(dC, ctx.mode, ctx.G, None)
        return dx.to(ctx.xdtype), dBg, dCg, dla, dgam, (dbet if be is not None else None)


class Mamba1Scan(torch.autograd.Function):
    """Mamba1 selective scan: u/delta [B, S, D], A [D, 16], B/C [B, S, 16] -> y [B, S, D] (f32)."""

    @staticmethod
    def forward(ctx, u, delta, A, Bm, Cm, clamp=None):
        args = [t.float().contiguous() for t in (u, delta, A, Bm, Cm)]
        y, hs = ext().mamba1_scan_fwd(*args, float(clamp or 0.0))
        ctx.save_for_backward(*args, hs)
        ctx.clamp = float(clamp or 0.0)
        ctx.udtype = u.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        u, delta, A, Bm, Cm, hs = ctx.saved_tensors
        du, ddelta, dA, dB, dC = ext().mamba1_scan_bwd(u, delta, A, Bm, Cm, hs, dy.float(), ctx.clamp)
        return du.to(ctx.udtype), ddelta, dA, dB, dC, None
