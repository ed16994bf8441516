"""tcgen05 GEMM entry points (CUDA) with PyTorch equivalents on CPU.

All functions compute ``A @ B^T`` in the "both operands K-major" convention of
a linear layer and accept the transposed storage of either operand, so the
three GEMMs of ``y = x W^T`` (forward, dX, dW) run without transposes:

* forward  ``y  = x  @ W^T``   : A = x  [T, K] (K-major),  B = W [N, K] (K-major)
* dX       ``dx = dy @ W``     : A = dy [T, N] (K-major),  B = W stored [N, K] = [K', N'] (MN-major)
* dW       ``dW = dy^T @ x``   : A = dy stored [T, N] (MN-major), B = x stored [T, K] (MN-major)

Upstream: every ``Linear`` / ``matmul`` of the reference (Candle on cuBLAS), e.g. model.rs:238,248,
model.rs:367,377 and mamba2.rs:563,611,673,732.
"""
from __future__ import annotations

from typing import Optional

import torch

from ._C import ext, status


def mm(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = False,
       out: Optional[torch.Tensor] = None, out_dtype=torch.bfloat16, resid: Optional[torch.Tensor] = None,
       beta: float = 0.0, alpha: float = 1.0, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out = alpha * op(a) @ op(b)^T (+ bias) (+ resid) (+ beta * out)``; ``bias`` [N] for bf16 output.

    ``op(a) = a`` ([M, K]) when ``a_t`` is False, else ``a^T`` with ``a`` stored [K, M].
    ``op(b) = b`` ([N, K]) when ``b_t`` is False, else ``b^T`` with ``b`` stored [K, N].
    """
    M = a.shape[1] if a_t else a.shape[0]
    N = b.shape[1] if b_t else b.shape[0]
    if not a.is_cuda or not (_tma_ok(a) and _tma_ok(b)):
        # CPU, or rows that are not 16-byte aligned for the TMA descriptors (a
        # projection to a few per-head scalars): plain fp32-accumulated matmul
        A = a.t() if a_t else a
        B = b.t() if b_t else b
        r = alpha * (A.float() @ B.float().t())
        if bias is not None:
            r = r + bias.float()
        if resid is not None:
            r = r + resid.float()
        if out is not None:
            if beta != 0.0:
                r = r + beta * out.float()
            out.copy_(r.to(out.dtype))
            return out
        return r.to(out_dtype)
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
    ext().gemm(a, a_t, b, b_t, out, resid, float(beta), float(alpha), status(a.device), bias)
    return out


def _tma_ok(t: torch.Tensor) -> bool:
    """Rows 16-byte aligned for the TMA descriptors (bf16, unit inner stride)."""
    return t.dim() == 2 and t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0


def linear_fwd(x2d: torch.Tensor, w: torch.Tensor, resid: Optional[torch.Tensor] = None) -> torch.Tensor:
    return mm(x2d, w, resid=resid)


def linear_dx(dy2d: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return mm(dy2d, w, b_t=True)


def linear_dw(dy2d: torch.Tensor, x2d: torch.Tensor, out: Optional[torch.Tensor] = None, beta: float = 0.0,
              out_dtype=torch.float32) -> torch.Tensor:
    return mm(dy2d, x2d, a_t=True, b_t=True, out=out, beta=beta, out_dtype=out_dtype)
