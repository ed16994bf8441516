"""State-space-model ops: causal depthwise conv1d, Mamba2 chunked SSD,
Mamba3 trapezoidal scan and the Mamba1 selective scan.

bf16 CUDA tensors use the sm_100a kernels in ``csrc/ssm*.cu`` when the
extension provides them; everything else runs the float32 statement in
``ops.reference`` under autograd.

Upstream: conv1d mamba2.rs:344-352; ``ssd_forward`` mamba2.rs:381-482 (``segment_sum``
mamba2.rs:116-180); ``ssd_forward_trapezoidal`` mamba3.rs:638-752; ``selective_scan_sequential``
mamba.rs:212-291.
"""
from __future__ import annotations

import torch

from . import reference as R


def _ext_has(name: str) -> bool:
    from ._C import ext
    return hasattr(ext(), name)


def causal_conv1d_cuda(x, w, b, act: bool = True):
    if _ext_has("conv1d_fwd"):
        from .ssm_kernels import CausalConv1d
        return CausalConv1d.apply(x, w, b, act)
    return R.causal_conv1d(x.float(), w.float(), None if b is None else b.float(), act).to(x.dtype)


def _expand_heads(t, H):
    G = t.shape[2]
    return t if G == H else t.repeat_interleave(H // G, dim=2)


def _scan_ok(x, N):
    return x.is_cuda and _ext_has("ssm_scan_fwd") and N % 32 == 0 and x.shape[-1] % 8 == 0 and \
        (N // 32) in (1, 2, 4) and (x.shape[-1] // 8) in (1, 2, 4, 8, 16, 32)


def ssd(x, dt, A, Bm, Cm, chunk: int, diag_only_g: bool = False):
    """Mamba2 SSD core (no D skip), f32 result.  x [B,S,H,P], dt [B,S,H],
    A [H], B/C [B,S,G,N] with G dividing H (grouped B/C are shared by heads)."""
    H, N = x.shape[2], Bm.shape[-1]
    if not diag_only_g:
        from .ssd_tc import ssd_tc, tc_ok
        if tc_ok(x, N, x.shape[1]):
            return ssd_tc(x, dt, A, Bm, Cm)
    if not diag_only_g and _scan_ok(x, N):
        from .ssm_kernels import SSMScan
        dtf = dt.float()
        return SSMScan.apply(x, Bm, Cm, A.float()[None, None, :] * dtf, dtf, None)
    f = lambda t: t.float()
    return R.ssd_chunked(f(x), f(dt), f(A), f(_expand_heads(Bm, H)), f(_expand_heads(Cm, H)), chunk, diag_only_g)


def ssd_skip(x, dt, A, Bm, Cm, D, chunk: int, diag_only_g: bool = False):
    """``ssd(...) + D x`` (per-head D); bf16 from the fused tensor-core epilogue, else f32."""
    if not diag_only_g:
        from .ssd_tc import ssd_tc, tc_ok
        if tc_ok(x, Bm.shape[-1], x.shape[1]):
            return ssd_tc(x, dt, A, Bm, Cm, D)
    y = ssd(x, dt, A, Bm, Cm, chunk, diag_only_g)
    return y.float() + x.float() * D.float()[:, None]


def mamba3_scan(x, dt, A, Bm, Cm, lam, chunk: int, compat: bool = False):
    """Trapezoidal two-term scan (no D skip), f32 result.  B/C [B,S,H,N] per head."""
    N = Bm.shape[-1]
    if not compat:
        from .ssd_tc import mamba3_tc, tc_ok
        if tc_ok(x, N, x.shape[1]):
            return mamba3_tc(x, dt, A, Bm, Cm, lam)
    if not compat and _scan_ok(x, N):
        from .ssm_kernels import SSMScan
        dtf, lamf = dt.float(), lam.float()
        loga = A.float()[None, None, :] * dtf
        beta = (1 - lamf) * dtf * torch.exp(loga)
        return SSMScan.apply(x, Bm, Cm, loga, lamf * dtf, beta)
    f = lambda t: t.float()
    return R.mamba3_scan(f(x), f(dt), f(A), f(Bm), f(Cm), f(lam), chunk, compat)


def selective_scan(u, delta, A, Bm, Cm, clamp=None):
    """Mamba1 scan, f32 result."""
    if u.is_cuda and _ext_has("mamba1_scan_fwd") and A.shape[-1] == 16:
        from .ssm_kernels import Mamba1Scan
        return Mamba1Scan.apply(u, delta, A, Bm, Cm, clamp)
    f = lambda t: t.float()
    return R.selective_scan(f(u), f(delta), f(A), f(Bm), f(Cm), clamp)
