"""State-space-model ops: causal depthwise conv1d, Mamba2 chunked SSD,
Mamba3 trapezoidal scan and the Mamba1 selective scan.

bf16 CUDA tensors use the sm_100a kernels in ``csrc/ssm*.cu`` when the
extension provides them; everything else runs the float32 statement in
``ops.reference`` under autograd.
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


def ssd(x, dt, A, Bm, Cm, chunk: int, diag_only_g: bool = False):
    """Mamba2 SSD core (no D skip).  x [B,S,H,P], dt [B,S,H], A [H], B/C [B,S,H,N]."""
    if x.is_cuda and not diag_only_g and _ext_has("ssd_fwd"):
        from .ssm_kernels import SSD
        return SSD.apply(x, dt, A, Bm, Cm, chunk)
    f = lambda t: t.float()
    return R.ssd_chunked(f(x), f(dt), f(A), f(Bm), f(Cm), chunk, diag_only_g).to(x.dtype)


def mamba3_scan(x, dt, A, Bm, Cm, lam, chunk: int, compat: bool = False):
    if x.is_cuda and not compat and _ext_has("ssd_fwd"):
        from .ssm_kernels import Mamba3Scan
        return Mamba3Scan.apply(x, dt, A, Bm, Cm, lam, chunk)
    f = lambda t: t.float()
    return R.mamba3_scan(f(x), f(dt), f(A), f(Bm), f(Cm), f(lam), chunk, compat).to(x.dtype)


def selective_scan(u, delta, A, Bm, Cm, clamp=None):
    if u.is_cuda and _ext_has("selective_scan_fwd"):
        from .ssm_kernels import SelectiveScan
        return SelectiveScan.apply(u, delta, A, Bm, Cm, clamp)
    f = lambda t: t.float()
    return R.selective_scan(f(u), f(delta), f(A), f(Bm), f(Cm), clamp).to(u.dtype)
