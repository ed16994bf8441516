"""Autograd functions over the sm_100a kernels (CUDA, bf16 activations).

Weight gradients: when a parameter carries a ``main_grad`` attribute (a view
into the flat f32 gradient buffer of :mod:`oxidizr_b200.optim`), backward
accumulates its gradient there with a fused GEMM epilogue (``C += A B^T``) or
an atomic scatter, then calls ``param._oxi_grad_ready()`` if present (the DDP
bucket hook), and returns ``None`` to autograd.  Without ``main_grad`` the
gradient is returned normally.

Upstream: RMSNorm model.rs:9-32, RoPE model.rs:68-117, GQA projections model.rs:320-323,
SwiGLU MLP model.rs:430-455, embedding / lm_head model.rs:964-1002, cross-entropy trainer.rs:166-171.
"""
from __future__ import annotations

import math
from typing import Optional

import os

import torch

from ._C import ext, status
from .gemm import mm


# SwiGLU backward: the down projection's dX GEMM with a plain epilogue followed by
# one element-wise kernel (split, default), or with the SwiGLU-backward epilogue
# fused into the GEMM (OXI_SWIGLU_BWD=fused).  The fused epilogue has to load the
# saved gate / up rows and evaluate the sigmoid per element while the MMAs of the
# next tile wait on its accumulator; at the Llama shape it ran at about 490
# TFLOP/s, against about 1.2 PFLOP/s for the plain GEMM plus a memory-bound pass.
SWIGLU_BWD_SPLIT = os.environ.get("OXI_SWIGLU_BWD", "split") != "fused"


def _ready(p):
    cb = getattr(p, "_oxi_grad_ready", None)
    if cb is not None:
        cb()


def _wgrad_gemm(p: torch.nn.Parameter, dy2: torch.Tensor, x2: torch.Tensor):
    """dW = dy^T @ x ([N, K]) accumulated into p.main_grad, else returned."""
    mg = getattr(p, "main_grad", None)
    if mg is not None:
        mm(dy2, x2, a_t=True, b_t=True, out=mg.view(dy2.shape[1], x2.shape[1]), beta=1.0)
        _ready(p)
        return None
    g = mm(dy2, x2, a_t=True, b_t=True, out_dtype=torch.float32)
    return g.to(p.dtype)


def _vec_grad(p: torch.nn.Parameter, g32: torch.Tensor):
    mg = getattr(p, "main_grad", None)
    if mg is not None:
        mg.view(-1).add_(g32.view(-1))
        _ready(p)
        return None
    return g32.to(p.dtype).view(p.shape)


def _bias_grad(p: torch.nn.Parameter, dy2: torch.Tensor):
    """Column sums of dy2 [T, N] (bf16) accumulated straight into the bias's main_grad."""
    mg = getattr(p, "main_grad", None)
    if dy2.is_cuda and dy2.dtype == torch.bfloat16 and dy2.stride(1) == 1:
        if mg is not None and mg.is_contiguous():
            ext().colsum_add(dy2, mg.view(-1))
            _ready(p)
            return None
        g32 = torch.zeros(dy2.shape[1], dtype=torch.float32, device=dy2.device)
        ext().colsum_add(dy2, g32)
        return _vec_grad(p, g32)
    return _vec_grad(p, dy2.sum(0, dtype=torch.float32))


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------- embedding
class Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w):
        ids_f = _c(ids.reshape(-1))
        out = torch.empty(ids_f.numel(), w.shape[1], dtype=w.dtype, device=w.device)
        ext().embed_fwd(ids_f, w, out)
        ctx.save_for_backward(ids_f)
        ctx.w = w
        return out.view(*ids.shape, w.shape[1])

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        w = ctx.w
        dy = _c(dy.reshape(-1, w.shape[1]))
        mg = getattr(w, "main_grad", None)
        if mg is not None:
            ext().embed_bwd(ids, dy, mg.view(w.shape))
            _ready(w)
            return None, None
        g = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        ext().embed_bwd(ids, dy, g)
        return None, g.to(w.dtype)


# ------------------------------------------------------------------- norms
class Norm(torch.autograd.Function):
    """mode 0 RMSNorm(x)*w, 1 LayerNorm(x)*w+b, 2 RMSNorm(x*silu(gate))*w."""

    @staticmethod
    def forward(ctx, x, gate, w, b, mode: int, eps: float):
        xc = _c(x)
        H = x.shape[-1]
        rows = xc.numel() // H
        y = torch.empty_like(xc)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        mean = torch.empty(rows, dtype=torch.float32, device=x.device) if mode == 1 else None
        gc = _c(gate) if gate is not None else None
        ext().norm_fwd(mode, xc, gc, w, b, y, rstd, mean, eps)
        ctx.save_for_backward(xc, gc, rstd, mean)
        ctx.w, ctx.b, ctx.mode = w, b, mode
        return y

    @staticmethod
    def backward(ctx, dy):
        dx, dgate, gw, gb = _norm_bwd(ctx, dy, None)
        return dx, dgate, gw, gb, None, None


def _grad_target(p, H: int, device):
    """(f32 [H] buffer the norm kernel adds its weight gradient into, whether it is p.main_grad)."""
    mg = getattr(p, "main_grad", None) if p is not None else None
    if mg is not None and mg.dtype == torch.float32 and mg.is_contiguous() and mg.numel() == H:
        return mg.view(-1), True
    return torch.zeros(H, dtype=torch.float32, device=device), False


def _norm_bwd(ctx, dy, dres):
    """Norm backward; dres (the gradient of a residual stream that passed through) is added
    to dx inside the kernel.  Weight gradients accumulate straight into main_grad (the kernel
    adds with atomics), so no zero fill or separate add runs."""
    xc, gc, rstd, mean = ctx.saved_tensors
    w, b, mode = ctx.w, ctx.b, ctx.mode
    H = xc.shape[-1]
    dyc = _c(dy)
    dx = torch.empty_like(xc)
    dgate = torch.empty_like(gc) if mode == 2 else None
    dw, w_direct = _grad_target(w, H, xc.device)
    db, b_direct = _grad_target(b, H, xc.device) if mode == 1 else (None, False)
    dr = _c(dres.reshape(xc.shape)) if dres is not None else None
    ext().norm_bwd(mode, dyc, xc, gc, w, rstd, mean, dr, dx, dgate, dw, db)
    if w_direct:
        _ready(w)
        gw = None
    else:
        gw = _vec_grad(w, dw)
    if mode != 1:
        gb = None
    elif b_direct:
        _ready(b)
        gb = None
    else:
        gb = _vec_grad(b, db)
    return dx, dgate, gw, gb


class NormResid(torch.autograd.Function):
    """(norm(x), x) for mode 0 (RMSNorm(x) w) or 1 (LayerNorm(x) w + b): the residual stream
    x passes through this node, so the gradient that comes back for it is added to the
    norm's input gradient inside the norm backward kernel (no separate add of the two
    gradient branches).  Upstream: the pre-norm blocks x + f(norm(x)) of model.rs:874-939."""

    @staticmethod
    def forward(ctx, x, w, b, mode: int, eps: float):
        xc = _c(x)
        H = x.shape[-1]
        rows = xc.numel() // H
        y = torch.empty_like(xc)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        mean = torch.empty(rows, dtype=torch.float32, device=x.device) if mode == 1 else None
        ext().norm_fwd(mode, xc, None, w, b, y, rstd, mean, eps)
        ctx.save_for_backward(xc, None, rstd, mean)
        ctx.w, ctx.b, ctx.mode = w, b, mode
        return y, x

    @staticmethod
    def backward(ctx, dy, dres):
        dx, _, gw, gb = _norm_bwd(ctx, dy, dres)
        return dx, gw, gb, None, None


# ----------------------------------------------------------------- linears
class Linear(torch.autograd.Function):
    """y = x W^T (+ bias) (+ resid).  x [..., K], W [N, K]."""

    @staticmethod
    def forward(ctx, x, w, bias, resid):
        K = x.shape[-1]
        x2 = _c(x.reshape(-1, K))
        r2 = _c(resid.reshape(-1, w.shape[0])) if resid is not None else None
        y = mm(x2, w, resid=r2, bias=bias)
        ctx.save_for_backward(x2)
        ctx.w, ctx.has_bias, ctx.has_resid, ctx.bias = w, bias is not None, resid is not None, bias
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        (x2,) = ctx.saved_tensors
        w = ctx.w
        dy2 = _c(dy.reshape(-1, w.shape[0]))
        dx = mm(dy2, w, b_t=True).view(*dy.shape[:-1], w.shape[1]) if ctx.needs_input_grad[0] else None
        gw = _wgrad_gemm(w, dy2, x2)
        gb = _bias_grad(ctx.bias, dy2) if ctx.has_bias else None
        dres = dy if ctx.has_resid else None
        return dx, gw, gb, dres


class LinearRope(torch.autograd.Function):
    """qkv = rope(x W^T) with RoPE on the first q_cols + k_cols columns."""

    @staticmethod
    def forward(ctx, x, w, cos, sin, hd: int, q_cols: int, k_cols: int):
        K = x.shape[-1]
        x2 = _c(x.reshape(-1, K))
        out = torch.empty(x2.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        ext().gemm_rope(x2, w, out, cos, sin, hd, q_cols, k_cols, status(x.device))
        ctx.save_for_backward(x2, cos, sin)
        ctx.w, ctx.hd, ctx.rot = w, hd, q_cols + k_cols
        return out.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, cos, sin = ctx.saved_tensors
        w = ctx.w
        d = dy.reshape(-1, w.shape[0])
        if d.stride(1) == 1 and d.stride(0) % 8 == 0 and d.data_ptr() % 16 == 0 and w.shape[0] % 8 == 0:
            dy2 = ext().rope_bwd_to(d, ctx.rot, ctx.hd, cos, sin)  # one pass, no copy first
        else:
            dy2 = d.contiguous().clone()
            ext().rope_bwd(dy2, ctx.rot, ctx.hd, cos, sin)
        dx = mm(dy2, w, b_t=True).view(*dy.shape[:-1], w.shape[1])
        gw = _wgrad_gemm(w, dy2, x2)
        return dx, gw, None, None, None, None, None


class AttentionQKVRope(torch.autograd.Function):
    """Causal GQA attention of one block from its input: qkv = rope(x W_qkv^T) (RoPE in the
    GEMM epilogue), o = flash(q, k, v).  The backward takes the inverse rotation inside
    the flash backward (dK epilogue, dQ conversion), so the QKV projection's dX / dW GEMMs
    read the unrotated gradient with no separate RoPE pass.  Upstream: model.rs:333-386."""

    @staticmethod
    def forward(ctx, x, w, cos, sin, nh: int, kvh: int, hd: int, scale: float):
        from .flash import _fwd
        B, S, K = x.shape
        x2 = _c(x.reshape(-1, K))
        qc, kc = nh * hd, kvh * hd
        qkv = torch.empty(x2.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        ext().gemm_rope(x2, w, qkv, cos, sin, hd, qc, kc, status(x.device))
        o, lse = _fwd(qkv[:, :qc], qkv[:, qc:qc + kc], qkv[:, qc + kc:], B, S, nh, kvh, hd, scale, True)
        ctx.save_for_backward(x2, qkv, o, lse, cos, sin)
        ctx.w, ctx.cfg = w, (B, S, nh, kvh, hd, scale)
        return o.view(B, S, qc)

    @staticmethod
    def backward(ctx, do):
        from .flash import _bwd
        x2, qkv, o, lse, cos, sin = ctx.saved_tensors
        w = ctx.w
        B, S, nh, kvh, hd, scale = ctx.cfg
        qc, kc = nh * hd, kvh * hd
        do2 = _c(do.reshape(B * S, qc))
        dqkv = torch.empty_like(qkv)
        _bwd(qkv[:, :qc], qkv[:, qc:qc + kc], qkv[:, qc + kc:], o, lse, do2, dqkv[:, :qc], dqkv[:, qc:qc + kc],
             dqkv[:, qc + kc:], B, S, nh, kvh, hd, scale, True, rope=(cos, sin))
        dx = mm(dqkv, w, b_t=True).view(B, S, w.shape[1]) if ctx.needs_input_grad[0] else None
        gw = _wgrad_gemm(w, dqkv, x2)
        return dx, gw, None, None, None, None, None, None


class SwiGLUMLP(torch.autograd.Function):
    """y = resid + (silu(x Wg^T) * (x Wu^T)) Wd^T with W_gu interleaved in 128-row blocks."""

    @staticmethod
    def forward(ctx, x, w_gu, w_down, resid):
        K = x.shape[-1]
        x2 = _c(x.reshape(-1, K))
        M = x2.shape[0]
        I = w_gu.shape[0] // 2
        h = torch.empty(M, I, dtype=x.dtype, device=x.device)
        gu = torch.empty(M, 2 * I, dtype=x.dtype, device=x.device)
        ext().gemm_swiglu(x2, w_gu, h, gu, status(x.device))
        r2 = _c(resid.reshape(-1, w_down.shape[0])) if resid is not None else None
        y = mm(h, w_down, resid=r2)
        ctx.save_for_backward(x2, h, gu)
        ctx.w_gu, ctx.w_down, ctx.has_resid = w_gu, w_down, resid is not None
        return y.view(*x.shape[:-1], w_down.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, h, gu = ctx.saved_tensors
        w_gu, w_down = ctx.w_gu, ctx.w_down
        dy2 = _c(dy.reshape(-1, w_down.shape[0]))
        g_down = _wgrad_gemm(w_down, dy2, h)
        dgu = torch.empty_like(gu)
        if SWIGLU_BWD_SPLIT:
            # dH with the plain epilogue, then one element-wise pass for dG / dU
            dh = mm(dy2, w_down, b_t=True)
            ext().swiglu_bwd(dh, gu, dgu)
        else:
            ext().gemm_swiglu_bwd(dy2, w_down, gu, dgu, status(dy.device))
        g_gu = _wgrad_gemm(w_gu, dgu, x2)
        dx = mm(dgu, w_gu, b_t=True).view(*dy.shape[:-1], w_gu.shape[1])
        return dx, g_gu, g_down, (dy if ctx.has_resid else None)


# ------------------------------------------------------------- LM head + CE
# Logits larger than this (bytes of bf16 [T, V]) are never materialised: the
# backward recomputes them in column chunks instead (OXI_CE_MODE = full |
# chunked | auto overrides).  Materialising is faster when it fits (one GEMM
# fewer); the chunked path keeps only per-row log-sum-exp.
CE_LOGITS_BUDGET = int(float(os.environ.get("OXI_CE_LOGITS_BUDGET", 16e9)))
CE_CHUNK = int(os.environ.get("OXI_CE_CHUNK", 8192))


def ce_mode(M: int, V: int) -> str:
    mode = os.environ.get("OXI_CE_MODE", "auto")
    if mode in ("full", "chunked"):
        return mode
    return "chunked" if M * V * 2 > CE_LOGITS_BUDGET else "full"


class LinearCrossEntropy(torch.autograd.Function):
    """Mean token cross-entropy of logits = x W^T without a separate softmax pass.

    Forward: one GEMM whose epilogue writes per-(row, 256-column tile) max and
    sum-of-exp partials and the target logit (and, in ``full`` mode, the bf16
    logits); a small kernel combines the partials into log-sum-exp and per-row
    loss.
    Backward, ``full``: softmax-minus-one-hot in place on the saved logits, then
    the dX and dW GEMMs read it directly.  ``chunked`` (logit-free): per column
    chunk of ``CE_CHUNK`` vocabulary rows, recompute that chunk's logits, form
    softmax-minus-one-hot from the saved log-sum-exp, accumulate dX (f32) and
    write that chunk's rows of dW; no [T, V] buffer exists at any point.
    """

    @staticmethod
    def forward(ctx, x, w, targets, ignore_index: int = -100):
        K = x.shape[-1]
        x2 = _c(x.reshape(-1, K))
        M, V = x2.shape[0], w.shape[0]
        tg = _c(targets.reshape(-1)).long()
        if ignore_index != -1:
            tg = torch.where(tg == ignore_index, torch.full_like(tg, -1), tg)
        nt = (V + 255) // 256
        mode = ce_mode(M, V)
        logits = None
        if mode == "full":
            ldl = (V + 7) // 8 * 8
            logits = torch.empty(M, ldl, dtype=x.dtype, device=x.device)
        pm = torch.empty(M, nt, dtype=torch.float32, device=x.device)
        ps = torch.empty_like(pm)
        tl = torch.zeros(M, dtype=torch.float32, device=x.device)
        ext().gemm_ce(x2, w, tg, pm, ps, tl, logits, 1.0, status(x.device))
        lse = torch.empty(M, dtype=torch.float32, device=x.device)
        loss = torch.empty(M, dtype=torch.float32, device=x.device)
        ext().ce_finish(pm, ps, tl, tg, lse, loss)
        count = (tg >= 0).sum().clamp_min(1)
        if logits is None:
            ctx.save_for_backward(x2, lse, tg, count)
        else:
            ctx.save_for_backward(x2, logits, lse, tg, count)
        ctx.w, ctx.V, ctx.xshape, ctx.mode = w, V, x.shape, mode
        return loss.sum() / count

    @staticmethod
    def backward(ctx, dloss):
        w, V = ctx.w, ctx.V
        if ctx.mode == "full":
            x2, logits, lse, tg, count = ctx.saved_tensors
            gscale = (dloss.float() / count.float()).reshape(1).contiguous()
            ext().ce_bwd(logits, V, lse, tg, gscale, 1.0)
            dl = logits[:, :V]
            dx = mm(dl, w, b_t=True)
            gw = _wgrad_gemm(w, dl, x2)
            return dx.view(ctx.xshape), gw, None, None
        x2, lse, tg, count = ctx.saved_tensors
        gscale = (dloss.float() / count.float()).reshape(1).contiguous()
        M, K = x2.shape
        C = max(8, min(CE_CHUNK, V) // 8 * 8)
        buf = torch.empty(M, C, dtype=x2.dtype, device=x2.device)  # one chunk of logits, reused
        dx32 = torch.empty(M, K, dtype=torch.float32, device=x2.device)
        mg = getattr(w, "main_grad", None)
        gw = None if mg is not None else torch.zeros(V, K, dtype=torch.float32, device=x2.device)
        for c0 in range(0, V, C):
            n = min(C, V - c0)
            wc = w[c0:c0 + n]
            lc = buf[:, :n]
            mm(x2, wc, out=lc)
            ext().ce_bwd(lc, n, lse, tg, gscale, 1.0, c0)
            mm(lc, wc, b_t=True, out=dx32, beta=0.0 if c0 == 0 else 1.0)
            dst = (mg.view(V, K) if mg is not None else gw)[c0:c0 + n]
            mm(lc, x2, a_t=True, b_t=True, out=dst, beta=1.0)
        if mg is not None:
            _ready(w)
        return dx32.to(x2.dtype).view(ctx.xshape), (gw.to(w.dtype) if gw is not None else None), None, None


# -------------------------------------------------------------- attention
def flash_attention(q, k, v, scale: float, causal: bool = True):
    """q [B, S, Hq, D], k/v [B, S, Hk, D] -> [B, S, Hq, D]."""
    from .attention import attention_cuda
    return attention_cuda(q, k, v, scale, causal)
