"""Tensor-core chunked SSD (csrc/ssd.cu): Mamba2's scan and, through an
interleaved sequence, Mamba3's trapezoidal two-term scan.

``SSDChunkTC``: ``y_t = H_t^T C_t`` with ``H_t = exp(loga_t) H_{t-1} + gamma_t
B_t x_t^T`` (N = 128 state, chunks of 128 steps).  The forward keeps the state
in TMEM and stores the chunk-start states (bf16) for the backward; the
backward runs a reverse pass (dx, state adjoints) and a chunk-parallel pass
(dB, dC, d gamma).  d loga follows from the identity used by the CUDA-core
scan: with q_t = <G_t, H_t> (G the state adjoint), q_t = <dy_t, y_t> + q_{t+1}
- v_{t+1} and d loga_t = q_t - v_t, v_t = gamma_t d gamma_t.

Mamba3 (mamba3.rs:638-752) updates H_t = alpha_t H_{t-1} + gamma_t u_t +
beta_t u_{t-1} with u_t = B_t x_t^T and beta_t = (1 - lam_t) dt_t alpha_t.  With
c_t = beta_{t+1} / alpha_{t+1} = (1 - lam_{t+1}) dt_{t+1} (c_{S-1} = 0) the
shifted state K_t = H_t + c_t u_t obeys the single-term recurrence
K_t = alpha_t K_{t-1} + (gamma_t + c_t) u_t, and y_t = C_t^T H_t =
C_t^T K_t - c_t <B_t, C_t> x_t.  ``mamba3_tc`` therefore runs the tensor-core
scan once over S steps with gamma' = gamma + c and folds the diagonal
correction into the D skip: no division by alpha, no extra sequence steps.
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
    """x [B, S, H, P] bf16; Bg/Cg [B, S, G, 128] (G divides H); loga/gamma [B, S, H].

    Without ``dskip``: y f32 [B, S, H, P].  With ``dskip`` ([H] per-head D, or [B, S, H]
    per token): the output kernel's D-skip epilogue returns bf16(y + dskip x); the
    backward's D-skip pass (csrc/ssm_glue.cu) supplies <dy, y> for d loga in the same
    pass that adds dskip dy to dx."""

    @staticmethod
    def forward(ctx, x, Bg, Cg, loga, gamma, dskip=None):
        Bsz, S, H, P = x.shape
        G, N = Bg.shape[2], Bg.shape[3]
        x2 = x.reshape(Bsz * S, H * P).to(torch.bfloat16).contiguous()
        B2 = Bg.reshape(Bsz * S, G * N).to(torch.bfloat16).contiguous()
        C2 = Cg.reshape(Bsz * S, G * N).to(torch.bfloat16).contiguous()
        la = loga.float().contiguous()
        ga = gamma.float().contiguous()
        ctx.shape = (Bsz, S, H, P, G, N)
        ctx.dtypes = (x.dtype, Bg.dtype, Cg.dtype, None if dskip is None else dskip.dtype)
        if dskip is None:
            y, hs = ext().ssd_tc_fwd(x2, B2, C2, la, ga, Bsz, S, H, P, G, status(x.device))
            ctx.save_for_backward(x2, B2, C2, la, ga, hs, y)
            return y.view(Bsz, S, H, P)
        dsk = dskip.float().contiguous()
        y, hs, out = ext().ssd_tc_fwd(x2, B2, C2, la, ga, Bsz, S, H, P, G, status(x.device), dsk)
        ctx.save_for_backward(x2, B2, C2, la, ga, hs, y, dsk)
        return out.view(Bsz, S, H, P)

    @staticmethod
    def backward(ctx, dy):
        saved = ctx.saved_tensors
        x2, B2, C2, la, ga, hs, y = saved[:7]
        Bsz, S, H, P, G, N = ctx.shape
        xd, bd, cd, dd_dtype = ctx.dtypes
        dyb = dy.reshape(Bsz * S, H * P).to(torch.bfloat16).contiguous()
        dx, dB, dC, dg = ext().ssd_tc_bwd(x2, B2, C2, la, ga, hs, dyb, Bsz, S, H, P, G, status(dy.device))
        if G < H:
            dB = dB.view(Bsz, S, G, H // G, N).sum(3)
            dC = dC.view(Bsz, S, G, H // G, N).sum(3)
        else:
            dB = dB.view(Bsz, S, G, N)
            dC = dC.view(Bsz, S, G, N)
        ddskip = None
        if dd_dtype is None:
            e = (dy.float().reshape(Bsz * S, H * P) * y).view(Bsz, S, H, P).sum(-1).contiguous()
            dx = dx.view(Bsz, S, H, P).to(xd)
        else:
            dsk = saved[7]
            dxb, dd, e = ext().dskip_bwd(dyb, x2, y, dsk, dx, H)
            dx = dxb.view(Bsz, S, H, P).to(xd)
            ddskip = (dd.view(Bsz, S, H) if dsk.numel() == Bsz * S * H else dd.sum(0)).to(dd_dtype)
        dla = ext().ssd_dloga(e.view(Bsz, S, H), ga.view(Bsz, S, H), dg.view(Bsz, S, H).contiguous())
        return dx, dB.to(bd), dC.to(cd), dla, dg, ddskip


def ssd_tc(x, dt, A, Bm, Cm, D=None):
    """Mamba2 SSD core: loga = A dt, gamma = dt.  f32 without ``D``; with the per-head
    skip ``D`` [H], bf16 y + D x from the fused epilogue."""
    dtf = dt.float()
    return SSDChunkTC.apply(x, Bm, Cm, A.float()[None, None, :] * dtf, dtf, D)


def mamba3_coeffs(dt, A, lam):
    """(loga, gamma', c) of the shifted single-term form, all f32 [B, S, H]."""
    dtf, lamf = dt.float(), lam.float()
    loga = A.float()[None, None, :] * dtf
    w = (1 - lamf) * dtf
    c = torch.cat([w[:, 1:], torch.zeros_like(w[:, :1])], 1)
    return loga, lamf * dtf + c, c


class Mamba3Coef(torch.autograd.Function):
    """Per-(token, head) inputs of the shifted-state Mamba3 scan in one kernel each way
    (csrc/m3_glue.cu): from the raw step-size projection ``dt_raw`` and the raw
    lambda projection ``lam_raw`` (bf16 [B, S, H]), ``dt_bias`` [H] and A [H]:
    dt = clamp(softplus(dt_raw + dt_bias), 1e-3, 0.1), log alpha = A dt,
    gamma' = sigmoid(lam_raw) dt + c and c_t = (1 - lambda_{t+1}) dt_{t+1}, all f32."""

    LO, HI = 1e-3, 0.1

    @staticmethod
    def forward(ctx, dt_raw, dt_bias, lam_raw, A):
        Bsz, S, H = dt_raw.shape
        dtc = dt_raw.to(torch.bfloat16).contiguous()
        lmc = lam_raw.to(torch.bfloat16).contiguous()
        bias = dt_bias.to(torch.bfloat16).contiguous()
        Af = A.float().contiguous()
        dt, loga, gp, c = ext().m3_coef_fwd(dtc, bias, lmc, Af, S, Mamba3Coef.LO, Mamba3Coef.HI)
        ctx.save_for_backward(dtc, bias, lmc, Af)
        ctx.S, ctx.dtypes = S, (dt_raw.dtype, dt_bias.dtype, lam_raw.dtype, A.dtype)
        sh = (Bsz, S, H)
        return dt.view(sh), loga.view(sh), gp.view(sh), c.view(sh)

    @staticmethod
    def backward(ctx, d_dt, d_loga, d_gp, d_c):
        dtc, bias, lmc, Af = ctx.saved_tensors
        f = lambda g: None if g is None else g.float().contiguous()
        ddt, dlam, dbias, dA = ext().m3_coef_bwd(dtc, bias, lmc, Af, ctx.S, Mamba3Coef.LO, Mamba3Coef.HI, f(d_dt),
                                                 f(d_loga), f(d_gp), f(d_c))
        t_dt, t_bias, t_lam, t_A = ctx.dtypes
        return ddt.view(dtc.shape).to(t_dt), dbias.to(t_bias), dlam.view(lmc.shape).to(t_lam), dA.to(t_A)


def mamba3_tc_skip_coef(x, dtv, loga, gp, c, Bm, Cm, D, bcdot):
    """Mamba3 scan + D skip from precomputed coefficients (``Mamba3Coef``):
    y = y_K + (D - c <B, C>) x, bf16 [B, S, H, P]."""
    dskip = D.float()[None, None, :] - c * bcdot
    return SSDChunkTC.apply(x, Bm, Cm, loga, gp, dskip)


def mamba3_tc_skip(x, dt, A, Bm, Cm, lam, D, bcdot):
    """Mamba3 scan + D skip through the shifted state, bf16 [B, S, H, P]:
    y = y_K + (D - c <B, C>) x.  Bm/Cm per head [B, S, H, N] bf16, bcdot = <B, C> [B, S, H]."""
    loga, gp, c = mamba3_coeffs(dt, A, lam)
    dskip = D.float()[None, None, :] - c * bcdot
    return SSDChunkTC.apply(x, Bm, Cm, loga, gp, dskip)


def mamba3_tc(x, dt, A, Bm, Cm, lam):
    """Mamba3 trapezoidal two-term scan (no D skip); Bm/Cm per head [B, S, H, N]."""
    Bb, Cb = Bm.to(torch.bfloat16), Cm.to(torch.bfloat16)
    loga, gp, c = mamba3_coeffs(dt, A, lam)
    y = SSDChunkTC.apply(x, Bb, Cb, loga, gp)
    bcdot = (Bb.float() * Cb.float()).sum(-1)
    return y - (c * bcdot)[..., None] * x.float()


class Mamba3BC(torch.autograd.Function):
    """Fused Mamba3 B/C prologue (csrc/mamba3.cu): rmsnorm(B_raw) w + b_bias, complex RoPE by
    ``ang``, as per-head bf16 [B, S, H, N] tensors (same for C with c_bias), plus
    bcdot = <B_rot, C_rot> f32 [B, S, H].  braw/craw [B, S, G*N] bf16 (views of the input
    projection)."""

    @staticmethod
    def forward(ctx, braw, craw, w, bbias, cbias, ang, H: int, eps: float):
        Bsz, S, GN = braw.shape
        G = GN // 128
        b2d, c2d = braw.reshape(Bsz * S, GN), craw.reshape(Bsz * S, GN)
        angc = ang.float().contiguous()
        bo, co, dot = ext().m3_bc_fwd(b2d, c2d, w.contiguous(), bbias.contiguous(), cbias.contiguous(), angc, Bsz,
                                      S, H, G, eps)
        ctx.save_for_backward(b2d, c2d, w, bbias, cbias, angc)
        ctx.cfg = (Bsz, S, H, G, eps, braw.shape)
        return bo, co, dot

    @staticmethod
    def backward(ctx, db, dc, ddot):
        b2d, c2d, w, bbias, cbias, angc = ctx.saved_tensors
        Bsz, S, H, G, eps, shape = ctx.cfg
        def z(t):  # bf16 gradients (per-head B/C from the tensor-core scan) are read as bf16
            if t is None:
                return torch.zeros(Bsz, S, H, 128, device=angc.device)
            return t.contiguous() if t.dtype == torch.bfloat16 else t.float().contiguous()
        dd = None if ddot is None else ddot.float().contiguous()
        dbr, dcr, dw, dbb, dcb, dang = ext().m3_bc_bwd(b2d, c2d, w.contiguous(), bbias.contiguous(),
                                                       cbias.contiguous(), angc, z(db), z(dc), dd, Bsz, S, H, G, eps)
        return (dbr.view(shape).to(b2d.dtype), dcr.view(shape).to(c2d.dtype), dw.to(w.dtype), dbb.to(bbias.dtype),
                dcb.to(cbias.dtype), dang, None, None)


def m3_bc_ok(braw: torch.Tensor, N: int, H: int, G: int) -> bool:
    return (braw.is_cuda and braw.dtype == torch.bfloat16 and N == 128 and H % G == 0
            and hasattr(ext(), "m3_bc_fwd"))


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
