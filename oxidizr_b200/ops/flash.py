"""Autograd wrappers of the sm_100a flash-attention kernels (csrc/flash_attn.cu).

``FlashAttentionQKV`` takes the fused ``[B, S, (Hq + 2 Hk) * D]`` projection
output (q | k | v heads, the layout the QKV GEMM writes) and returns the
attention output ``[B, S, Hq * D]``; its backward writes the fused gradient
``dqkv`` in the same layout, so no per-slice gradient assembly is needed.
``FlashAttention`` takes separate q, k ``[B, S, H, Dqk]`` and v ``[B, S, Hk, Dv]``
views; Dqk > Dv is the multi-head latent attention case (a RoPE part
concatenated to q and k, model.rs:226-236).
"""
from __future__ import annotations

import torch

from ._C import ext, status


def _fwd(q2, k2, v2, B, S, Hq, Hk, D, scale, causal, Dv=None):
    Dv = D if Dv is None else Dv
    o = torch.empty(B * S, Hq * Dv, dtype=q2.dtype, device=q2.device)
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device=q2.device)
    ext().flash_fwd(q2, k2, v2, o, lse, B, S, Hq, Hk, D, Dv, scale, causal, status(q2.device))
    return o, lse


def _bwd(q2, k2, v2, o, lse, do2, dq, dk, dv, B, S, Hq, Hk, D, scale, causal, Dv=None, rope=None):
    """rope = (cos, sin) tables: q and k were rotate-half RoPE outputs and dq / dk come
    back as the gradients of the unrotated q and k."""
    Dv = D if Dv is None else Dv
    delta = torch.empty(B, Hq, S, dtype=torch.float32, device=q2.device)
    dq_acc = torch.empty(B * S, Hq * D, dtype=torch.float32, device=q2.device)
    cos, sin = rope if rope is not None else (None, None)
    ext().flash_bwd(q2, k2, v2, o, do2, lse, delta, dq_acc, dq, dk, dv, B, S, Hq, Hk, D, Dv, scale, causal,
                    status(q2.device), cos, sin)


class FlashAttentionQKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, Hq: int, Hk: int, D: int, scale: float, causal: bool = True):
        B, S, N = qkv.shape
        qkv2 = qkv.reshape(B * S, N)
        if not qkv2.is_contiguous():
            qkv2 = qkv2.contiguous()
        q2, k2, v2 = qkv2[:, :Hq * D], qkv2[:, Hq * D:(Hq + Hk) * D], qkv2[:, (Hq + Hk) * D:]
        o, lse = _fwd(q2, k2, v2, B, S, Hq, Hk, D, scale, causal)
        ctx.save_for_backward(qkv2, o, lse)
        ctx.cfg = (B, S, Hq, Hk, D, scale, causal)
        return o.view(B, S, Hq * D)

    @staticmethod
    def backward(ctx, do):
        qkv2, o, lse = ctx.saved_tensors
        B, S, Hq, Hk, D, scale, causal = ctx.cfg
        do2 = do.reshape(B * S, Hq * D)
        if not do2.is_contiguous():
            do2 = do2.contiguous()
        dqkv = torch.empty_like(qkv2)
        q2, k2, v2 = qkv2[:, :Hq * D], qkv2[:, Hq * D:(Hq + Hk) * D], qkv2[:, (Hq + Hk) * D:]
        _bwd(q2, k2, v2, o, lse, do2, dqkv[:, :Hq * D], dqkv[:, Hq * D:(Hq + Hk) * D], dqkv[:, (Hq + Hk) * D:],
             B, S, Hq, Hk, D, scale, causal)
        return dqkv.view(B, S, -1), None, None, None, None, None


class FlashAttention(torch.autograd.Function):
    """q [B, S, Hq, Dqk], k [B, S, Hk, Dqk], v [B, S, Hk, Dv] (rows with unit inner stride)."""

    @staticmethod
    def forward(ctx, q, k, v, scale: float, causal: bool = True):
        B, S, Hq, D = q.shape
        Hk, Dv = k.shape[2], v.shape[3]
        q2 = q.reshape(B * S, Hq * D)
        k2 = k.reshape(B * S, Hk * D)
        v2 = v.reshape(B * S, Hk * Dv)
        o, lse = _fwd(q2, k2, v2, B, S, Hq, Hk, D, scale, causal, Dv)
        ctx.save_for_backward(q2, k2, v2, o, lse)
        ctx.cfg = (B, S, Hq, Hk, D, Dv, scale, causal)
        return o.view(B, S, Hq, Dv)

    @staticmethod
    def backward(ctx, do):
        q2, k2, v2, o, lse = ctx.saved_tensors
        B, S, Hq, Hk, D, Dv, scale, causal = ctx.cfg
        do2 = do.reshape(B * S, Hq * Dv).contiguous()
        dq = torch.empty(B * S, Hq * D, dtype=q2.dtype, device=q2.device)
        dk = torch.empty(B * S, Hk * D, dtype=q2.dtype, device=q2.device)
        dv = torch.empty(B * S, Hk * Dv, dtype=q2.dtype, device=q2.device)
        _bwd(q2, k2, v2, o, lse, do2, dq, dk, dv, B, S, Hq, Hk, D, scale, causal, Dv)
        return dq.view(B, S, Hq, D), dk.view(B, S, Hk, D), dv.view(B, S, Hk, Dv), None, None
