"""Causal attention entry points.

CUDA: the sm_100a flash-attention kernels (``csrc/flash_attn.cu``) when built;
CPU: the materialised reference (model.rs:362-377).
Layout: q/k [B, S, H, Dqk], v [B, S, Hk, Dv] (GQA when Hk < Hq; Dqk > Dv for
multi-head latent attention), output [B, S, Hq, Dv].
"""
from __future__ import annotations

import torch

from . import reference as R


def _has_native_fa() -> bool:
    from ._C import ext
    e = ext()
    return hasattr(e, "flash_fwd") and hasattr(e, "flash_bwd")


def native_ok(D: int, Dv: int = None) -> bool:
    """A flash kernel (forward and backward) exists for head dims (qk D, v Dv)."""
    if not _has_native_fa():
        return False
    from ._C import ext
    e = ext()
    Dv = D if Dv is None else Dv
    if hasattr(e, "flash_supported"):
        return bool(e.flash_supported(D, Dv, True))
    return Dv == D and D in (64, 128)


def attention_qkv(qkv, Hq: int, Hk: int, D: int, scale: float, causal: bool = True):
    """Attention over the fused [B, S, (Hq + 2 Hk) * D] projection; returns [B, S, Hq * D]."""
    if qkv.is_cuda and qkv.dtype == torch.bfloat16 and native_ok(D):
        from .flash import FlashAttentionQKV
        return FlashAttentionQKV.apply(qkv, Hq, Hk, D, scale, causal)
    B, S, _ = qkv.shape
    q = qkv[..., :Hq * D].view(B, S, Hq, D)
    k = qkv[..., Hq * D:(Hq + Hk) * D].view(B, S, Hk, D)
    v = qkv[..., (Hq + Hk) * D:].view(B, S, Hk, D)
    return attention(q, k, v, scale, causal).reshape(B, S, Hq * D)


def attention_cuda(q, k, v, scale: float, causal: bool = True):
    if native_ok(q.shape[-1], v.shape[-1]) and q.dtype == torch.bfloat16:
        from .flash import FlashAttention
        return FlashAttention.apply(q, k, v, scale, causal)
    # library attention, used only until the native kernel is present
    out = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=causal, scale=scale,
        enable_gqa=k.shape[2] != q.shape[2])
    return out.transpose(1, 2)


def attention(q, k, v, scale: float, causal: bool = True):
    if q.is_cuda:
        return attention_cuda(q, k, v, scale, causal)
    o = R.attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale, causal)
    return o.transpose(1, 2)
