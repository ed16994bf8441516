"""Device-dispatching op API used by the models.

bf16 CUDA tensors run the sm_100a kernels (``ops.fused`` and friends); CPU
tensors (and non-bf16 CUDA tensors, e.g. an f32 model moved to the GPU) run
the PyTorch statement of the same math from ``ops.reference`` under autograd.

Upstream: RMSNorm model.rs:9-32, gated RMSNorm mamba2.rs:185-217, Mamba2 LayerNorm
mamba2.rs:768, RoPE model.rs:68-117, SwiGLU model.rs:430-455, attention model.rs:333-386 and
model.rs:196-256, lm_head model.rs:1002.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import reference as R


def _native(t: torch.Tensor) -> bool:
    return t.is_cuda and t.dtype == torch.bfloat16


def embedding(ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if _native(w):
        from .fused import Embedding
        return Embedding.apply(ids, w)
    return F.embedding(ids, w)


def rmsnorm(x, w, eps: float = 1e-5):
    if _native(x):
        from .fused import Norm
        return Norm.apply(x, None, w, None, 0, eps)
    return R.rmsnorm(x, w, eps)


def rmsnorm_resid(x, w, eps: float = 1e-5):
    """(rmsnorm(x, w), x) where the second output is the residual stream to add back after
    the sublayer: on the GPU its gradient is added inside the norm backward kernel."""
    if _native(x):
        from .fused import NormResid
        return NormResid.apply(x, w, None, 0, eps)
    return rmsnorm(x, w, eps), x


def layernorm_resid(x, w, b, eps: float = 1e-6):
    """(layernorm(x, w, b), x), the residual stream passing through like rmsnorm_resid."""
    if _native(x):
        from .fused import NormResid
        return NormResid.apply(x, w, b, 1, eps)
    return layernorm(x, w, b, eps), x


def layernorm(x, w, b, eps: float = 1e-6):
    if _native(x):
        from .fused import Norm
        return Norm.apply(x, None, w, b, 1, eps)
    return R.layernorm(x, w, b, eps)


def gated_rmsnorm(y, gate, w, eps: float = 1e-6):
    if _native(y):
        from .fused import Norm
        return Norm.apply(y, gate, w, None, 2, eps)
    return R.gated_rmsnorm(y, gate, w, eps)


class _SplitCols(torch.autograd.Function):
    """Column blocks of a projection output as views; the backward writes the block
    gradients into ONE buffer (a single concatenation) instead of the per-slice
    zero-fill + copy + sum that autograd does for plain slicing."""

    @staticmethod
    def forward(ctx, p, sizes):
        ctx.sizes, ctx.shape, ctx.dtype = sizes, p.shape, p.dtype
        outs, o = [], 0
        for n in sizes:
            outs.append(p.narrow(-1, o, n))
            o += n
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        lead = ctx.shape[:-1]
        parts = [torch.zeros(*lead, n, dtype=ctx.dtype, device=grads[0].device if grads[0] is not None else None)
                 if g is None else g.to(ctx.dtype) for g, n in zip(grads, ctx.sizes)]
        return torch.cat(parts, -1), None


def split_cols(p, sizes):
    """``p[..., a:b]`` blocks of widths ``sizes`` (summing to p's last dim)."""
    assert sum(sizes) == p.shape[-1], (sizes, p.shape)
    if p.requires_grad and torch.is_grad_enabled():
        return _SplitCols.apply(p, tuple(sizes))
    outs, o = [], 0
    for n in sizes:
        outs.append(p[..., o:o + n])
        o += n
    return tuple(outs)


def linear(x, w, bias=None, resid=None):
    if _native(x):
        from .fused import Linear
        return Linear.apply(x, w, bias, resid)
    y = F.linear(x, w.to(x.dtype), None if bias is None else bias.to(x.dtype))
    return y if resid is None else resid + y


def qkv_rope(x, w_qkv, cos, sin, hd: int, q_cols: int, k_cols: int):
    """x W_qkv^T with rotate-half RoPE applied to the q and k heads.
    cos/sin are [S, hd/2] f32 tables; token rows are [B*S] in sequence order."""
    if _native(x) and hd in (64, 128):
        from .fused import LinearRope
        return LinearRope.apply(x, w_qkv, cos, sin, hd, q_cols, k_cols)
    y = F.linear(x, w_qkv.to(x.dtype))
    B, S = x.shape[0], x.shape[1]
    q = y[..., :q_cols].reshape(B, S, -1, hd).transpose(1, 2)
    k = y[..., q_cols:q_cols + k_cols].reshape(B, S, -1, hd).transpose(1, 2)
    q = R.apply_rope(q, cos[:S], sin[:S]).transpose(1, 2).reshape(B, S, q_cols)
    k = R.apply_rope(k, cos[:S], sin[:S]).transpose(1, 2).reshape(B, S, k_cols)
    return torch.cat([q, k, y[..., q_cols + k_cols:]], -1)


def attention_rope(x, w_qkv, cos, sin, nh: int, kvh: int, hd: int, scale: float):
    """Causal GQA attention from the block input: qkv_rope + attention_qkv in one autograd
    node whose backward un-rotates dq / dk inside the flash backward."""
    from .attention import native_ok
    S = x.shape[1]
    if _native(x) and hd in (64, 128) and native_ok(hd) and cos.shape[0] >= S and x.shape[-1] % 8 == 0:
        from .fused import AttentionQKVRope
        return AttentionQKVRope.apply(x, w_qkv, cos, sin, nh, kvh, hd, scale)
    qkv = qkv_rope(x, w_qkv, cos, sin, hd, nh * hd, kvh * hd)
    return attention_qkv(qkv, nh, kvh, hd, scale, causal=True)


def mla_qkv(qc, kv, rp, cos, sin, nh: int, hd: int, dr: int):
    """MLA attention operands (model.rs:196-256): q = [q_c, rope(q_rope)], k = [k_c, rope(k_rope)]
    with the one k_rope of a token shared by every head, and v, from q_c [B, S, nh*hd],
    kv [B, S, 2*nh*hd] (k | v) and the rope block rp [B, S, dr + nh*dr] (k_rope | q_rope).
    Returns q, k [B, S, nh, hd + dr] and v [B, S, nh, hd]."""
    B, S = qc.shape[0], qc.shape[1]
    if _native(qc) and hd % 8 == 0 and dr % 2 == 0 and dr <= 64:
        from .mla import MlaPack
        return MlaPack.apply(qc, kv, rp, cos, sin, nh, hd, dr)
    k_r = rp[..., :dr].reshape(B, S, 1, dr)
    q_r = rp[..., dr:].reshape(B, S, nh, dr)
    q_r = R.apply_rope(q_r.transpose(1, 2), cos[:S], sin[:S]).transpose(1, 2)
    k_r = R.apply_rope(k_r.transpose(1, 2), cos[:S], sin[:S]).transpose(1, 2)
    q = torch.cat([qc.view(B, S, nh, hd), q_r.to(qc.dtype)], -1)
    k = torch.cat([kv[..., :nh * hd].view(B, S, nh, hd), k_r.to(kv.dtype).expand(B, S, nh, dr)], -1)
    return q, k, kv[..., nh * hd:].view(B, S, nh, hd)


def swiglu_mlp(x, w_gu, w_down, resid=None):
    """resid + down(silu(gate x) * up x); w_gu rows interleaved [g 128 | u 128]..."""
    I = w_gu.shape[0] // 2
    if _native(x) and I % 128 == 0:
        from .fused import SwiGLUMLP
        return SwiGLUMLP.apply(x, w_gu, w_down, resid)
    gu = F.linear(x, w_gu.to(x.dtype))
    nb = I // 128 if I % 128 == 0 else None
    if nb:
        gu = gu.reshape(*gu.shape[:-1], nb, 2, 128)
        g, u = gu[..., 0, :].reshape(*x.shape[:-1], I), gu[..., 1, :].reshape(*x.shape[:-1], I)
    else:
        g, u = gu[..., :I], gu[..., I:]
    y = F.linear(F.silu(g) * u, w_down.to(x.dtype))
    return y if resid is None else resid + y


def attention(q, k, v, scale: float, causal: bool = True):
    from .attention import attention as _att
    return _att(q, k, v, scale, causal)


def attention_qkv(qkv, Hq: int, Hk: int, D: int, scale: float, causal: bool = True):
    from .attention import attention_qkv as _aq
    return _aq(qkv, Hq, Hk, D, scale, causal)


def linear_cross_entropy(x, w, targets, ignore_index: int = -100):
    if _native(x):
        from .fused import LinearCrossEntropy
        return LinearCrossEntropy.apply(x, w, targets, ignore_index)
    logits = F.linear(x, w.to(x.dtype))
    return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1).long(),
                           ignore_index=ignore_index)


def causal_conv1d(x, w, b, act: bool = True):
    """x [B, S, C] channels-last; w [C, 1, k]; b [C]."""
    if _native(x):
        from .ssm import causal_conv1d_cuda
        return causal_conv1d_cuda(x, w, b, act)
    return R.causal_conv1d(x, w, b, act)
