"""Tensor-core chunked SSD (csrc/ssd.cu): Mamba2's scan and, through an
interleaved sequence, Mamba3's trapezoidal two-term scan.

``SSDChunkTC``: ``y_t = H_t^T C_t`` with ``H_t = exp(loga_t) H_{t-1} + gamma_t
B_t x_t^T`` (N = 128 state, chunks of 128 steps).  The forward keeps the state
in TMEM and stores the chunk-start states (bf16) for the backward; the
backward runs a reverse pass (dx, state adjoints) and a chunk-parallel pass
(dB, dC, d gamma).  d loga follows from the identity used by the CUDA-core
scan: with q_t = <G_t, H_t> (G the state adjoint), q_t = <dy_t, y_t> + q_{t+1}
- v_{t+1} and d loga_t = q_t - v_t, v_t = gamma_t d gamma_t.

Mamba3 (mamba3.rs:638-752) updates H_t = alpha_t H_{t-1} + gamma_t B_t x_t^T +
beta_t B_{t-1} x_{t-1}^T.  ``mamba3_tc`` runs it as the single-term recurrence
on 2S steps: step 2t adds beta_t B_{t-1} x_{t-1}^T after the decay alpha_t,
step 2t+1 adds gamma_t B_t x_t^T with no decay; y_t is read at step 2t+1.
"""
from __future__ import annotations

import torch

from ._C import ext, status


def tc_ok(x: torch.Tensor, N: int, S: int) -> bool:
    if not (x.is_cuda and x.dtype == torch.bfloat16):
        return False
    e = ext()
    return hasattr(e, "ssd_tc_fwd") and bool(e.ssd_tc_supported(N, x.shape[-1], S))


class SSDChunkTC(torch.autograd.Function):
    """x [B, S, H, P] bf16; Bg/Cg [B, S, G, 128] (G divides H); loga/gamma [B, S, H] -> y f32 [B, S, H, P]."""

    @staticmethod
    def forward(ctx, x, Bg, Cg, loga, gamma):
        Bsz, S, H, P = x.shape
        G, N = Bg.shape[2], Bg.shape[3]
        x2 = x.reshape(Bsz * S, H * P).to(torch.bfloat16).contiguous()
        B2 = Bg.reshape(Bsz * S, G * N).to(torch.bfloat16).contiguous()
        C2 = Cg.reshape(Bsz * S, G * N).to(torch.bfloat16).contiguous()
        la = loga.float().contiguous()
        ga = gamma.float().contiguous()
        y, hs = ext().ssd_tc_fwd(x2, B2, C2, la, ga, Bsz, S, H, P, G, status(x.device))
        ctx.save_for_backward(x2, B2, C2, la, ga, hs, y)
        ctx.shape = (Bsz, S, H, P, G, N)
        ctx.dtypes = (x.dtype, Bg.dtype, Cg.dtype)
        return y.view(Bsz, S, H, P)

    @staticmethod
    def backward(ctx, dy):
        x2, B2, C2, la, ga, hs, y = ctx.saved_tensors
        Bsz, S, H, P, G, N = ctx.shape
        dyf = dy.float().reshape(Bsz * S, H * P)
        dyb = dyf.to(torch.bfloat16).contiguous()
        dx, dB, dC, dg = ext().ssd_tc_bwd(x2, B2, C2, la, ga, hs, dyb, Bsz, S, H, P, G, status(dy.device))
        dB = dB.view(Bsz, S, G, H // G, N).sum(3)
        dC = dC.view(Bsz, S, G, H // G, N).sum(3)
        e = (dyf * y).view(Bsz, S, H, P).sum(-1)
        v = ga * dg
        v_next = torch.cat([v[:, 1:], torch.zeros_like(v[:, :1])], 1)
        q = torch.flip(torch.cumsum(torch.flip(e - v_next, [1]), 1), [1])
        dla = q - v
        xd, bd, cd = ctx.dtypes
        return dx.view(Bsz, S, H, P).to(xd), dB.to(bd), dC.to(cd), dla, dg


def ssd_tc(x, dt, A, Bm, Cm):
    """Mamba2 SSD core (no D skip): loga = A dt, gamma = dt."""
    dtf = dt.float()
    return SSDChunkTC.apply(x, Bm, Cm, A.float()[None, None, :] * dtf, dtf)


def mamba3_tc(x, dt, A, Bm, Cm, lam):
    """Mamba3 trapezoidal two-term scan (no D skip) via the interleaved single-term form."""
    Bsz, S, H, P = x.shape
    N = Bm.shape[-1]
    dtf, lamf = dt.float(), lam.float()
    loga = A.float()[None, None, :] * dtf
    gamma = lamf * dtf
    beta = (1 - lamf) * dtf * torch.exp(loga)
    pad = lambda t: torch.cat([torch.zeros_like(t[:, :1]), t[:, :-1]], 1)
    x2 = torch.stack([pad(x), x], 2).reshape(Bsz, 2 * S, H, P)
    B2 = torch.stack([pad(Bm), Bm], 2).reshape(Bsz, 2 * S, Bm.shape[2], N)
    C2 = torch.stack([torch.zeros_like(Cm), Cm], 2).reshape(Bsz, 2 * S, Cm.shape[2], N)
    la2 = torch.stack([loga, torch.zeros_like(loga)], 2).reshape(Bsz, 2 * S, H)
    g2 = torch.stack([beta, gamma], 2).reshape(Bsz, 2 * S, H)
    y2 = SSDChunkTC.apply(x2, B2, C2, la2, g2)
    return y2.view(Bsz, S, 2, H, P)[:, :, 1]


class Mamba3BC(torch.autograd.Function):
    """Fused Mamba3 B/C prologue (csrc/mamba3.cu): rmsnorm(B_raw) w + b_bias, complex RoPE by
    ``ang``, written as the interleaved [B, 2S, H, N] tensors of the two-term tensor-core scan
    (same for C with c_bias).  braw/craw [B, S, G*N] bf16 (views of the input projection)."""

    @staticmethod
    def forward(ctx, braw, craw, w, bbias, cbias, ang, H: int, eps: float):
        Bsz, S, GN = braw.shape
        G = GN // 128
        b2d, c2d = braw.reshape(Bsz * S, GN), craw.reshape(Bsz * S, GN)
        angc = ang.float().contiguous()
        b2, c2 = ext().m3_bc_fwd(b2d, c2d, w.contiguous(), bbias.contiguous(), cbias.contiguous(), angc, Bsz, S, H,
                                 G, eps)
        ctx.save_for_backward(b2d, c2d, w, bbias, cbias, angc)
        ctx.cfg = (Bsz, S, H, G, eps, braw.shape)
        return b2, c2

    @staticmethod
    def backward(ctx, db2, dc2):
        b2d, c2d, w, bbias, cbias, angc = ctx.saved_tensors
        Bsz, S, H, G, eps, shape = ctx.cfg
        z = lambda t: torch.zeros(Bsz, 2 * S, H, 128, device=angc.device) if t is None else t.float().contiguous()
        dbr, dcr, dw, dbb, dcb, dang = ext().m3_bc_bwd(b2d, c2d, w.contiguous(), bbias.contiguous(),
                                                       cbias.contiguous(), angc, z(db2), z(dc2), Bsz, S, H, G, eps)
        return (dbr.view(shape).to(b2d.dtype), dcr.view(shape).to(c2d.dtype), dw.to(w.dtype), dbb.to(bbias.dtype),
                dcb.to(cbias.dtype), dang, None, None)


def m3_bc_ok(braw: torch.Tensor, N: int, H: int, G: int) -> bool:
    return (braw.is_cuda and braw.dtype == torch.bfloat16 and N == 128 and H % G == 0
            and hasattr(ext(), "m3_bc_fwd"))


def mamba3_tc_interleaved(x, dt, A, b2, c2, lam):
    """Mamba3 two-term scan with B/C already in the interleaved layout (from Mamba3BC)."""
    Bsz, S, H, P = x.shape
    dtf, lamf = dt.float(), lam.float()
    loga = A.float()[None, None, :] * dtf
    gamma = lamf * dtf
    beta = (1 - lamf) * dtf * torch.exp(loga)
    x_prev = torch.cat([torch.zeros_like(x[:, :1]), x[:, :-1]], 1)
    x2 = torch.stack([x_prev, x], 2).reshape(Bsz, 2 * S, H, P)
    la2 = torch.stack([loga, torch.zeros_like(loga)], 2).reshape(Bsz, 2 * S, H)
    g2 = torch.stack([beta, gamma], 2).reshape(Bsz, 2 * S, H)
    y2 = SSDChunkTC.apply(x2, b2, c2, la2, g2)
    return y2.view(Bsz, S, 2, H, P)[:, :, 1]


class AngleCumsum(torch.autograd.Function):
    """ang[b, t, h, j] = sum_{u <= t} theta[b, u, h, j] dt[b, u, h] (csrc/cumsum.cu)."""

    @staticmethod
    def forward(ctx, theta, dt):
        th, d = theta.float().contiguous(), dt.float().contiguous()
        ctx.save_for_backward(th, d)
        return ext().angle_cumsum(th, d)

    @staticmethod
    def backward(ctx, dang):
        th, d = ctx.saved_tensors
        dtheta, ddt = ext().angle_cumsum_bwd(th, d, dang.float().contiguous())
        return dtheta, ddt


def angle_cumsum(theta, dt):
    if theta.is_cuda and theta.shape[-1] % 32 == 0 and hasattr(ext(), "angle_cumsum"):
        return AngleCumsum.apply(theta, dt)
    return torch.cumsum(theta * dt[..., None], 1)
