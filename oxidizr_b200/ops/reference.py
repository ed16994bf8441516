"""Pure-PyTorch statement of every op's math.

These functions are the CPU implementation of the op library and, run in
float64, the oracle every CUDA kernel is tested against.  Each cites the
upstream code whose math it restates.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


# ------------------------------------------------------------------ norms
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """model.rs:22-31: f32 internal ``x / sqrt(mean(x^2) + eps)``, cast back, then ``* weight``."""
    xf = x.float() if x.dtype != torch.float64 else x
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y.to(x.dtype) * w.to(x.dtype)


def layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """candle_nn::LayerNorm as used by Mamba2/3 blocks (mamba2.rs:768, eps 1e-6)."""
    xf = x.float() if x.dtype != torch.float64 else x
    y = F.layer_norm(xf, (x.shape[-1],), w.to(xf.dtype), b.to(xf.dtype), eps)
    return y.to(x.dtype)


def gated_rmsnorm(y: torch.Tensor, gate: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """MambaRMSNormGated (mamba2.rs:196-216): ``rmsnorm(y * silu(gate)) * w`` in f32."""
    dt = torch.float64 if y.dtype == torch.float64 else torch.float32
    h = y.to(dt) * F.silu(gate.to(dt))
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return (h * w.to(dt)).to(y.dtype)


# ------------------------------------------------------------------ RoPE
def rope_tables(dim: int, seq: int, theta: float, device=None, dtype=torch.float32) -> Tuple[torch.Tensor, torch.Tensor]:
    """model.rs:43-66: ``inv_freq_i = theta^(-2i/dim)``; returns cos/sin of shape [seq, dim/2]."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64, device=device) / dim))
    t = torch.arange(seq, dtype=torch.float64, device=device)
    f = t[:, None] * inv[None]
    return f.cos().to(dtype), f.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE (model.rs:68-117) on x [..., S, D] with half tables [S, D/2]."""
    d = x.shape[-1]
    c = torch.cat([cos, cos], -1).to(x.dtype)
    s = torch.cat([sin, sin], -1).to(x.dtype)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = torch.cat([-x2, x1], -1)
    return x * c + rot * s


# ------------------------------------------------------------- attention
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool = True) -> torch.Tensor:
    """Materialised causal attention (model.rs:362-377) on [B, H, S, D]; k/v may have
    fewer heads (GQA ``repeat_kv``, model.rs:388-399)."""
    hq, hk = q.shape[1], k.shape[1]
    if hk != hq:
        k = k.repeat_interleave(hq // hk, dim=1)
        v = v.repeat_interleave(hq // hk, dim=1)
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    if causal:
        S, T = q.shape[-2], k.shape[-2]
        mask = torch.ones(S, T, dtype=torch.bool, device=q.device).triu(T - S + 1)
        s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s.float() if s.dtype != torch.float64 else s, -1).to(v.dtype)
    return torch.matmul(p, v)


# --------------------------------------------------------- cross entropy
def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """candle_nn::loss::cross_entropy mean over tokens (trainer.rs:166-171)."""
    lf = logits.float() if logits.dtype != torch.float64 else logits
    return F.cross_entropy(lf.reshape(-1, lf.shape[-1]), targets.reshape(-1))


# ----------------------------------------------------------------- conv1d
def causal_conv1d(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], act: bool = True) -> torch.Tensor:
    """Depthwise causal conv (pad k-1 left, crop to S) + optional SiLU
    (mamba2.rs:344-352).  x [B, S, C] (channels last), w [C, 1, k] or [C, k]."""
    B, S, C = x.shape
    w2 = w.reshape(C, 1, -1)
    k = w2.shape[-1]
    y = F.conv1d(x.transpose(1, 2), w2.to(x.dtype), None if b is None else b.to(x.dtype), padding=k - 1, groups=C)
    y = y[..., :S].transpose(1, 2)
    return F.silu(y) if act else y


# --------------------------------------------------------------- Mamba2 SSD
def segsum(a: torch.Tensor) -> torch.Tensor:
    """L[i, j] = sum_{j < t <= i} a_t for j <= i, -inf above the diagonal."""
    T = a.shape[-1]
    cs = torch.cumsum(a, -1)
    d = cs[..., :, None] - cs[..., None, :]
    mask = torch.ones(T, T, dtype=torch.bool, device=a.device).tril()
    return d.masked_fill(~mask, float("-inf"))


def ssd_chunked(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, Bm: torch.Tensor, Cm: torch.Tensor,
                chunk: int, diag_only_g: bool = False) -> torch.Tensor:
    """Chunked SSD (mamba2.rs:381-482), the core without the D skip.

    x [B, S, H, P] (already multiplied by nothing; dt applied here), dt [B, S, H]
    (post softplus/clamp), A [H] (negative), B/C [B, S, H, N] (groups already
    expanded).  ``diag_only_g`` reproduces the upstream ``compute_g`` which uses
    ``C_l . B_l`` for every column (mamba2.rs:523-536).
    Returns y [B, S, H, P].
    """
    b, S, H, P = x.shape
    pad = (chunk - S % chunk) % chunk
    xd = x * dt[..., None]
    a = A[None, None, :] * dt
    if pad:
        xd = F.pad(xd, (0, 0, 0, 0, 0, pad))
        a = F.pad(a, (0, 0, 0, pad))
        Bm = F.pad(Bm, (0, 0, 0, 0, 0, pad))
        Cm = F.pad(Cm, (0, 0, 0, 0, 0, pad))
    L_ = S + pad
    nc = L_ // chunk
    xc = xd.reshape(b, nc, chunk, H, P)
    Bc = Bm.reshape(b, nc, chunk, H, -1)
    Cc = Cm.reshape(b, nc, chunk, H, -1)
    ac = a.reshape(b, nc, chunk, H).permute(0, 3, 1, 2)  # [b, H, nc, l]
    acs = torch.cumsum(ac, -1)
    Lm = torch.exp(segsum(ac))  # [b, H, nc, l, l]
    if diag_only_g:
        g = (Cc * Bc).sum(-1)  # [b, nc, l, H]
        G = g.permute(0, 3, 1, 2)[..., :, None].expand(-1, -1, -1, -1, chunk)
    else:
        G = torch.einsum("bclhn,bcshn->bhcls", Cc, Bc)
    y_diag = torch.einsum("bhcls,bcshp->bclhp", G * Lm, xc)
    decay_states = torch.exp(acs[..., -1:] - acs)  # [b, H, nc, l]
    states = torch.einsum("bclhn,bhcl,bclhp->bchpn", Bc, decay_states, xc)
    init = torch.zeros_like(states[:, :1])
    states = torch.cat([init, states], 1)
    decay_chunk = torch.exp(segsum(F.pad(acs[..., -1], (1, 0))))  # [b, H, nc+1, nc+1]
    new_states = torch.einsum("bhzc,bchpn->bzhpn", decay_chunk, states)
    states = new_states[:, :-1]
    y_off = torch.einsum("bclhn,bchpn,bhcl->bclhp", Cc, states, torch.exp(acs))
    y = (y_diag + y_off).reshape(b, L_, H, P)
    return y[:, :S]


def ssd_sequential(x, dt, A, Bm, Cm) -> torch.Tensor:
    """Ground-truth recurrence h_t = exp(dt A) h_{t-1} + dt B_t x_t^T; y_t = C_t h_t."""
    b, S, H, P = x.shape
    N = Bm.shape[-1]
    h = torch.zeros(b, H, P, N, dtype=x.dtype, device=x.device)
    ys = []
    for t in range(S):
        dA = torch.exp(dt[:, t] * A[None])  # [b, H]
        h = h * dA[..., None, None] + (dt[:, t, :, None, None] * x[:, t, :, :, None] * Bm[:, t, :, None, :])
        ys.append(torch.einsum("bhpn,bhn->bhp", h, Cm[:, t]))
    return torch.stack(ys, 1)


def mamba3_scan(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, Bm: torch.Tensor, Cm: torch.Tensor,
                lam: torch.Tensor, chunk: int, compat: bool = False) -> torch.Tensor:
    """Trapezoidal two-term scan (mamba3.rs:638-752) without the D skip.

    h_t = a_t h_{t-1} + gamma_t B_t x_t^T + beta_t B_{t-1} x_{t-1}^T,  y_t = C_t h_t
    with a_t = exp(dt_t A), gamma_t = lam_t dt_t, beta_t = (1 - lam_t) dt_t a_t.
    ``compat=True`` reproduces the upstream inter-chunk state, which pairs the
    beta term with B_t instead of B_{t-1} (mamba3.rs:709-712).
    x [B, S, H, P]; dt, lam [B, S, H]; B/C [B, S, H, N].
    """
    b, S, H, P = x.shape
    a = A[None, None] * dt
    gamma = lam * dt
    beta = (1 - lam) * dt * torch.exp(a)
    x_prev = F.pad(x[:, :-1], (0, 0, 0, 0, 1, 0))
    B_prev = F.pad(Bm[:, :-1], (0, 0, 0, 0, 1, 0))
    xg = x * gamma[..., None]
    xb = x_prev * beta[..., None]
    pad = (chunk - S % chunk) % chunk
    if pad:
        xg = F.pad(xg, (0, 0, 0, 0, 0, pad))
        xb = F.pad(xb, (0, 0, 0, 0, 0, pad))
        a = F.pad(a, (0, 0, 0, pad))
        Bm = F.pad(Bm, (0, 0, 0, 0, 0, pad))
        B_prev = F.pad(B_prev, (0, 0, 0, 0, 0, pad))
        Cm = F.pad(Cm, (0, 0, 0, 0, 0, pad))
    L_ = S + pad
    nc = L_ // chunk
    r = lambda t: t.reshape(b, nc, chunk, H, -1)
    xgc, xbc, Bc, Bpc, Cc = r(xg), r(xb), r(Bm), r(B_prev), r(Cm)
    ac = a.reshape(b, nc, chunk, H).permute(0, 3, 1, 2)
    acs = torch.cumsum(ac, -1)
    Lm = torch.exp(segsum(ac))
    G1 = torch.einsum("bclhn,bcshn->bhcls", Cc, Bc)
    G2 = torch.einsum("bclhn,bcshn->bhcls", Cc, Bpc)
    y_diag = torch.einsum("bhcls,bcshp->bclhp", G1 * Lm, xgc) + torch.einsum("bhcls,bcshp->bclhp", G2 * Lm, xbc)
    decay_states = torch.exp(acs[..., -1:] - acs)
    if compat:
        states = torch.einsum("bclhn,bhcl,bclhp->bchpn", Bc, decay_states, xgc + xbc)
    else:
        states = (torch.einsum("bclhn,bhcl,bclhp->bchpn", Bc, decay_states, xgc)
                  + torch.einsum("bclhn,bhcl,bclhp->bchpn", Bpc, decay_states, xbc))
    states = torch.cat([torch.zeros_like(states[:, :1]), states], 1)
    decay_chunk = torch.exp(segsum(F.pad(acs[..., -1], (1, 0))))
    states = torch.einsum("bhzc,bchpn->bzhpn", decay_chunk, states)[:, :-1]
    y_off = torch.einsum("bclhn,bchpn,bhcl->bclhp", Cc, states, torch.exp(acs))
    return (y_diag + y_off).reshape(b, L_, H, P)[:, :S]


def mamba3_sequential(x, dt, A, Bm, Cm, lam) -> torch.Tensor:
    b, S, H, P = x.shape
    N = Bm.shape[-1]
    h = torch.zeros(b, H, P, N, dtype=x.dtype, device=x.device)
    ys = []
    for t in range(S):
        at = torch.exp(dt[:, t] * A[None])
        g = lam[:, t] * dt[:, t]
        be = (1 - lam[:, t]) * dt[:, t] * at
        h = h * at[..., None, None] + g[..., None, None] * x[:, t, :, :, None] * Bm[:, t, :, None, :]
        if t > 0:
            h = h + be[..., None, None] * x[:, t - 1, :, :, None] * Bm[:, t - 1, :, None, :]
        ys.append(torch.einsum("bhpn,bhn->bhp", h, Cm[:, t]))
    return torch.stack(ys, 1)


def mamba3_rotate(t: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
    """Complex RoPE on interleaved (re, im) pairs of the state dim (mamba3.rs:581-612).
    t [B, S, H, N], angles [B, S, H, N/2]."""
    re, im = t[..., 0::2], t[..., 1::2]
    c, s = angles.cos(), angles.sin()
    out = torch.stack([re * c - im * s, re * s + im * c], -1)
    return out.reshape(t.shape)


# ------------------------------------------------------------ Mamba1 scan
def selective_scan(u, delta, A, Bm, Cm, clamp: Optional[float] = None) -> torch.Tensor:
    """Mamba1 scan (mamba.rs:212-291): h_t = exp(delta_t A) h_{t-1} + delta_t u_t B_t;
    y_t = h_t C_t.  u, delta [B, S, D]; A [D, N]; B, C [B, S, N].  ``clamp``
    reproduces the upstream +-30 state clamp."""
    b, S, D = u.shape
    h = torch.zeros(b, D, A.shape[1], dtype=u.dtype, device=u.device)
    ys = []
    for t in range(S):
        dA = torch.exp(delta[:, t, :, None] * A[None])
        h = dA * h + delta[:, t, :, None] * u[:, t, :, None] * Bm[:, t, None, :]
        if clamp is not None:
            h = h.clamp(-clamp, clamp)
        ys.append(torch.einsum("bdn,bn->bd", h, Cm[:, t]))
    return torch.stack(ys, 1)


# ------------------------------------------------------------------- AdamW
def adamw_step(p, g, m, v, step: int, lr: float, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01, grad_scale: float = 1.0):
    """optimizer.rs:126-192: ``p -= lr * m_hat / (sqrt(v_hat) + eps) + lr * wd * p``
    (decoupled weight decay on the pre-update parameter)."""
    g = g * grad_scale
    m.mul_(beta1).add_(g, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    upd = (m / bc1) / ((v / bc2).sqrt() + eps)
    p.sub_(lr * upd + lr * wd * p)
    return p
