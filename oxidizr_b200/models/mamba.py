"""Mamba1 (mamba.rs), Mamba2 SSD (mamba2.rs) and Mamba3 (mamba3.rs) blocks.

Default math is the intended one; ``compat: reference`` in the model config
reproduces the upstream quirks listed below for parity with upstream
checkpoints:

* Mamba1 ``A = exp(-a_log)`` (positive) with the +-30 state clamp
  (mamba.rs:178, mamba.rs:273); intended: ``A = -exp(a_log)``.
* Mamba2/3 ``compute_g`` uses ``C_l . B_l`` for all columns (mamba2.rs:523-536);
  intended: ``C_l . B_s``.
* Mamba3 inter-chunk state pairs the beta term with B_t (mamba3.rs:709-712);
  intended: with B_{t-1}, matching the recurrence.

In both modes the stored ``A_log`` is the offset from the S4D initialisation
``log(1..H)`` (upstream adds the init once at construction,
mamba2.rs:278-291), and here it is trainable.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import api, ssm
from .common import RefModule, _assign, normal_, take


def _softplus_dt(dt: torch.Tensor, bias: torch.Tensor, lo=1e-3, hi=0.1) -> torch.Tensor:
    return F.softplus(dt.float() + bias.float()).clamp(lo, hi)


def _dt_bias_init(n: int, device, gen=None, lo=1e-3, hi=0.1) -> torch.Tensor:
    """Inverse-softplus of log-uniform dt in [lo, hi] (the usual Mamba init)."""
    u = torch.rand(n, generator=gen, device=gen.device if gen is not None else device).to(device)
    dt = torch.exp(u * (math.log(hi) - math.log(lo)) + math.log(lo))
    return (dt + torch.log(-torch.expm1(-dt))).to(device)


class LinearB(RefModule):
    """Linear with optional bias and upstream parameter names ``weight``/``bias``."""

    def __init__(self, inp, out, bias=True, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out, inp, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.zeros(out, device=device, dtype=dtype)) if bias else None

    def reset_parameters(self, std, gen=None):
        normal_(self.weight, std, gen)
        if self.bias is not None:
            with torch.no_grad():
                self.bias.zero_()

    def forward(self, x, resid=None):
        return api.linear(x, self.weight, self.bias, resid)


class NormW(RefModule):
    """RMSNorm / LayerNorm parameter holder with upstream names."""

    def __init__(self, n, bias=False, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.zeros(n, device=device, dtype=dtype)) if bias else None

    def reset_parameters(self, std=None, gen=None):
        with torch.no_grad():
            self.weight.fill_(1.0)
            if self.bias is not None:
                self.bias.zero_()


class Conv1d(RefModule):
    """Depthwise causal conv1d parameters ``weight [C,1,k]``, ``bias [C]``."""

    def __init__(self, C, k, bias=True, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(C, 1, k, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.zeros(C, device=device, dtype=dtype)) if bias else None
        self.k = k

    def reset_parameters(self, std=None, gen=None):
        bound = 1.0 / math.sqrt(self.k)
        with torch.no_grad():
            dev = gen.device if gen is not None else self.weight.device
            w = torch.rand(self.weight.shape, generator=gen, device=dev) * 2 * bound - bound
            self.weight.copy_(w.to(self.weight.device, self.weight.dtype))
            if self.bias is not None:
                self.bias.zero_()

    def forward(self, x, act=True):
        return api.causal_conv1d(x, self.weight, self.bias, act)


# =========================================================================
# Mamba1
# =========================================================================
class Mamba1Mixer(RefModule):
    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        H = cfg.hidden_size
        self.d_inner = 2 * H
        self.d_state = 16
        self.compat = cfg.reference_compat
        self.in_proj = LinearB(H, 2 * self.d_inner, bias=False, device=device, dtype=dtype)
        self.conv1d = Conv1d(self.d_inner, 4, bias=True, device=device, dtype=dtype)
        self.x_proj = LinearB(self.d_inner, self.d_inner + 2 * self.d_state, bias=False, device=device, dtype=dtype)
        self.dt_proj = LinearB(self.d_inner, self.d_inner, bias=True, device=device, dtype=dtype)
        self.a_log = nn.Parameter(torch.empty(self.d_inner, self.d_state, device=device, dtype=dtype))
        self.d = nn.Parameter(torch.ones(self.d_inner, device=device, dtype=dtype))
        self.out_proj = LinearB(self.d_inner, H, bias=False, device=device, dtype=dtype)

    def reset_parameters(self, std, gen=None):
        for m in (self.in_proj, self.x_proj, self.dt_proj, self.out_proj):
            m.reset_parameters(std, gen)
        self.conv1d.reset_parameters(std, gen)
        with torch.no_grad():
            # S4D-real: A[d, n] = -(n + 1)
            a = torch.log(torch.arange(1, self.d_state + 1, dtype=torch.float32))
            self.a_log.copy_(a[None].expand(self.d_inner, -1).to(self.a_log.dtype))
            self.d.fill_(1.0)
            self.dt_proj.bias.copy_(_dt_bias_init(self.d_inner, self.dt_proj.bias.device, gen).to(self.dt_proj.bias.dtype))

    def forward(self, h, resid):
        xr = self.in_proj(h)
        x, res = xr[..., :self.d_inner], xr[..., self.d_inner:]
        x = self.conv1d(x.contiguous(), act=True)
        xd = self.x_proj(x)
        delta = xd[..., :self.d_inner]
        Bm = xd[..., self.d_inner:self.d_inner + self.d_state]
        Cm = xd[..., self.d_inner + self.d_state:]
        delta = F.softplus(self.dt_proj(delta.contiguous()).float())
        if self.compat:
            A = torch.exp(-self.a_log.float())
            clamp = 30.0
        else:
            A = -torch.exp(self.a_log.float())
            clamp = None
        y = ssm.selective_scan(x, delta, A, Bm, Cm, clamp)
        y = (y.float() + x.float() * self.d.float()) * F.silu(res.float())
        return self.out_proj(y.to(h.dtype), resid=resid)


class Mamba1Block(RefModule):
    """x + mixer(RMSNorm(x)) (model.rs:874-885); names ``mamba.*`` and ``norm.weight``."""

    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        self.mamba = Mamba1Mixer(cfg, device, dtype)
        self.norm = NormW(cfg.hidden_size, device=device, dtype=dtype)

    def reset_parameters(self, std, gen=None):
        self.mamba.reset_parameters(std, gen)
        self.norm.reset_parameters()

    def forward(self, x):
        h, x = api.rmsnorm_resid(x, self.norm.weight, 1e-5)
        return self.mamba(h, x), None


# =========================================================================
# Mamba2
# =========================================================================
class Mamba2Mixer(RefModule):
    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        H = cfg.hidden_size
        self.Hs = cfg.mamba2_num_heads
        self.P = cfg.mamba2_head_dim
        self.N = cfg.mamba2_state_size
        self.chunk = cfg.mamba2_chunk_size
        self.g = cfg.mamba2_n_groups or 1
        self.k = cfg.mamba2_conv_kernel or 4
        self.I = H * cfg.mamba2_expand
        self.conv_dim = self.I + 2 * self.g * self.N
        self.compat = cfg.reference_compat
        self.in_proj = LinearB(H, self.I + self.conv_dim + self.Hs, True, device, dtype)
        self.conv1d = Conv1d(self.conv_dim, self.k, True, device, dtype)
        self.dt_bias = nn.Parameter(torch.zeros(self.Hs, device=device, dtype=dtype))
        self.A_log = nn.Parameter(torch.zeros(self.Hs, device=device, dtype=dtype))
        self.D = nn.Parameter(torch.ones(self.Hs, device=device, dtype=dtype))
        self.norm = NormW(self.I, device=device, dtype=dtype)
        self.out_proj = LinearB(self.I, H, True, device, dtype)
        self.register_buffer("a_init", torch.log(torch.arange(1, self.Hs + 1, dtype=torch.float32)).to(device),
                             persistent=False)

    def reset_parameters(self, std, gen=None):
        self.in_proj.reset_parameters(std, gen)
        self.out_proj.reset_parameters(std, gen)
        self.conv1d.reset_parameters(std, gen)
        self.norm.reset_parameters()
        with torch.no_grad():
            self.A_log.zero_()
            self.D.fill_(1.0)
            self.dt_bias.copy_(_dt_bias_init(self.Hs, self.dt_bias.device, gen).to(self.dt_bias.dtype))

    def A(self):
        return -torch.exp(self.A_log.float() + self.a_init).clamp(1e-6, 1e6)

    def forward(self, h, resid):
        B, S, _ = h.shape
        p = self.in_proj(h)
        gate, xBC, dt = api.split_cols(p, [self.I, self.conv_dim, self.Hs])
        xBC = self.conv1d(xBC.contiguous(), act=True)
        x = xBC[..., :self.I].reshape(B, S, self.Hs, self.P)
        gn = self.g * self.N
        Bm = xBC[..., self.I:self.I + gn].reshape(B, S, self.g, self.N)
        Cm = xBC[..., self.I + gn:].reshape(B, S, self.g, self.N)
        dtv = _softplus_dt(dt, self.dt_bias)
        y = ssm.ssd_skip(x, dtv, self.A(), Bm, Cm, self.D, self.chunk, diag_only_g=self.compat)
        y = y.to(h.dtype).reshape(B, S, self.I)
        y = api.gated_rmsnorm(y, gate.contiguous(), self.norm.weight, 1e-6)
        return self.out_proj(y, resid=resid)


class Mamba2Block(RefModule):
    """x + mixer(LayerNorm(x)) with names ``mamba2.norm.*``, ``mamba2.mixer.*``."""

    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        self.norm = NormW(cfg.hidden_size, bias=True, device=device, dtype=dtype)
        self.mixer = Mamba2Mixer(cfg, device, dtype)

    def reset_parameters(self, std, gen=None):
        self.norm.reset_parameters()
        self.mixer.reset_parameters(std, gen)

    def forward(self, x):
        h, x = api.layernorm_resid(x, self.norm.weight, self.norm.bias, 1e-6)
        return self.mixer(h, x), None


# =========================================================================
# Mamba3
# =========================================================================
class Mamba3Mixer(RefModule):
    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        H = cfg.hidden_size
        self.Hs = cfg.mamba2_num_heads
        self.P = cfg.mamba2_head_dim
        self.N = cfg.mamba2_state_size
        self.chunk = cfg.mamba2_chunk_size
        self.g = cfg.mamba2_n_groups or 1
        self.I = H * cfg.mamba2_expand
        self.complex_rope = True if cfg.mamba3_complex_rope is None else cfg.mamba3_complex_rope
        self.R = cfg.mamba3_mimo_rank or 0
        self.use_conv = bool(cfg.mamba3_use_conv)
        self.k = cfg.mamba2_conv_kernel or 4
        self.compat = cfg.reference_compat
        if self.complex_rope and self.N % 2:
            raise ValueError(f"Mamba3 with complex RoPE requires even state_size, got {self.N}")
        bc = self.g * self.N
        self.in_proj = LinearB(H, 2 * self.I + 2 * bc + self.Hs, True, device, dtype)
        self.out_proj = LinearB(self.I, H, True, device, dtype)
        self.lambda_proj = LinearB(H, self.Hs, True, device, dtype)
        self.theta_proj = LinearB(H, self.Hs * (self.N // 2), True, device, dtype) if self.complex_rope else None
        self.b_bias = nn.Parameter(torch.ones(self.Hs, self.N, device=device, dtype=dtype))
        self.c_bias = nn.Parameter(torch.ones(self.Hs, self.N, device=device, dtype=dtype))
        self.dt_bias = nn.Parameter(torch.zeros(self.Hs, device=device, dtype=dtype))
        self.A_log = nn.Parameter(torch.zeros(self.Hs, device=device, dtype=dtype))
        self.D = nn.Parameter(torch.ones(self.Hs, device=device, dtype=dtype))
        self.bc_norm = NormW(self.N, device=device, dtype=dtype)
        self.norm = NormW(self.I, device=device, dtype=dtype)
        self.conv1d = Conv1d(self.I + 2 * bc, self.k, True, device, dtype) if self.use_conv else None
        if self.R > 0:
            self.mimo_x_up = LinearB(self.P, self.P * self.R, True, device, dtype)
            self.mimo_x_down = LinearB(self.P * self.R, self.P, True, device, dtype)
        else:
            self.mimo_x_up = self.mimo_x_down = None
        self.register_buffer("a_init", torch.log(torch.arange(1, self.Hs + 1, dtype=torch.float32)).to(device),
                             persistent=False)

    def reset_parameters(self, std, gen=None):
        for m in (self.in_proj, self.out_proj, self.lambda_proj, self.theta_proj, self.mimo_x_up, self.mimo_x_down):
            if m is not None:
                m.reset_parameters(std, gen)
        if self.conv1d is not None:
            self.conv1d.reset_parameters(std, gen)
        self.bc_norm.reset_parameters()
        self.norm.reset_parameters()
        with torch.no_grad():
            self.b_bias.fill_(1.0)
            self.c_bias.fill_(1.0)
            self.A_log.zero_()
            self.D.fill_(1.0)
            self.dt_bias.copy_(_dt_bias_init(self.Hs, self.dt_bias.device, gen).to(self.dt_bias.dtype))

    def A(self):
        return -torch.exp(self.A_log.float() + self.a_init).clamp(1e-6, 1e6)

    def forward(self, h, resid):
        B, S, _ = h.shape
        bc = self.g * self.N
        p = self.in_proj(h)
        gate, x, Bm, Cm, dt = api.split_cols(p, [self.I, self.I, bc, bc, self.Hs])
        if self.conv1d is not None:
            xbc = self.conv1d(torch.cat([x, Bm, Cm], -1).contiguous(), act=True)
            x = xbc[..., :self.I]
            Bm = xbc[..., self.I:self.I + bc]
            Cm = xbc[..., self.I + bc:]
        else:
            x = F.silu(x)
        fused = self._fused_ok(h, x, S)
        if fused:
            # step size, lambda and the shifted-state coefficients in one kernel
            from ..ops.ssd_tc import Mamba3Coef
            dtv, loga, gp, cshift = Mamba3Coef.apply(dt, self.dt_bias, self.lambda_proj(h), self.A())
            # fused prologue (norm + bias + complex RoPE) straight into the tensor-core scan layout
            from ..ops.ssd_tc import Mamba3BC
            if self.complex_rope:
                from ..ops.ssd_tc import angle_cumsum
                theta = self.theta_proj(h).float().reshape(B, S, self.Hs, self.N // 2)
                ang = angle_cumsum(theta, dtv)
            else:
                ang = torch.zeros(B, S, self.Hs, self.N // 2, device=h.device)
            bro, cro, bcdot = Mamba3BC.apply(Bm, Cm, self.bc_norm.weight, self.b_bias, self.c_bias, ang, self.Hs,
                                             1e-6)
            xh = x.reshape(B, S, self.Hs, self.P)
            if self.mimo_x_up is not None:
                xh = self.mimo_x_up(xh)
            from ..ops.ssd_tc import mamba3_tc_skip_coef
            # the shifted-state diagonal correction rides on the fused D skip
            y = mamba3_tc_skip_coef(xh, dtv, loga, gp, cshift, bro, cro, self.D, bcdot)
            return self._finish(y, xh, gate, h, resid, B, S, skipped=True)
        lam = torch.sigmoid(self.lambda_proj(h).float())
        dtv = _softplus_dt(dt, self.dt_bias)
        Bm = Bm.reshape(B, S, self.g, self.N)
        Cm = Cm.reshape(B, S, self.g, self.N)
        rep = self.Hs // self.g
        if rep > 1:
            Bm = Bm.repeat_interleave(rep, 2)
            Cm = Cm.repeat_interleave(rep, 2)
        w = self.bc_norm.weight
        Bm = api.rmsnorm(Bm.contiguous(), w, 1e-6).float() + self.b_bias.float()
        Cm = api.rmsnorm(Cm.contiguous(), w, 1e-6).float() + self.c_bias.float()
        if self.complex_rope:
            theta = self.theta_proj(h).float().reshape(B, S, self.Hs, self.N // 2)
            ang = torch.cumsum(theta * dtv[..., None], 1)
            from ..ops import reference as R
            Bm = R.mamba3_rotate(Bm, ang)
            Cm = R.mamba3_rotate(Cm, ang)
        xh = x.reshape(B, S, self.Hs, self.P)
        if self.mimo_x_up is not None:
            xh = self.mimo_x_up(xh)
        y = ssm.mamba3_scan(xh, dtv, self.A(), Bm, Cm, lam, self.chunk, compat=self.compat)
        return self._finish(y, xh, gate, h, resid, B, S)

    def _fused_ok(self, h, x, S) -> bool:
        if self.compat or not h.is_cuda or self.conv1d is not None:
            return False
        from ..ops.ssd_tc import m3_bc_ok, tc_ok
        width = self.P * (self.R if self.mimo_x_up is not None else 1)
        probe = x.new_empty(1, 1, 1, width)
        return m3_bc_ok(x, self.N, self.Hs, self.g) and tc_ok(probe, self.N, S)

    def _finish(self, y, xh, gate, h, resid, B, S, skipped=False):
        """y + D x (unless ``skipped``: already added), mimo down, gated norm, out_proj."""
        if not skipped:
            y = y.float() + xh.float() * self.D.float()[:, None]
        y = y.to(h.dtype)
        if self.mimo_x_down is not None:
            y = self.mimo_x_down(y)
        y = y.reshape(B, S, self.I)
        y = api.gated_rmsnorm(y.contiguous(), gate.contiguous(), self.norm.weight, 1e-6)
        return self.out_proj(y, resid=resid)


class Mamba3Block(RefModule):
    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        self.norm = NormW(cfg.hidden_size, bias=True, device=device, dtype=dtype)
        self.mixer = Mamba3Mixer(cfg, device, dtype)

    def reset_parameters(self, std, gen=None):
        self.norm.reset_parameters()
        self.mixer.reset_parameters(std, gen)

    def forward(self, x):
        h, x = api.layernorm_resid(x, self.norm.weight, self.norm.bias, 1e-6)
        return self.mixer(h, x), None
