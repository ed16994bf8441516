"""Causal attention entry points.

CUDA: the sm_100a flash-attention kernels (``csrc/flash_attn.cu``) when built;
CPU: the materialised reference (model.rs:362-377).
Layout: q [B, S, Hq, D], k/v [B, S, Hk, D] (GQA when Hk < Hq), output
[B, S, Hq, D].
"""
from __future__ import annotations

import torch

from . import reference as R


def _has_native_fa() -> bool:
    from ._C import ext
    return hasattr(ext(), "flash_fwd")


def attention_cuda(q, k, v, scale: float, causal: bool = True):
    if _has_native_fa():
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
