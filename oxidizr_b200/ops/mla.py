"""Multi-head latent attention operands (model.rs:196-256) in one kernel each way
(csrc/mla.cu).

``MlaPack``: from q_c = W_uq c_q [B, S, nh*hd], kv = W_ukv c_kv [B, S, 2*nh*hd]
(k | v) and the rope block of the down projection rp [B, S, dr + nh*dr]
(k_rope | q_rope) it returns q = [q_c, rope(q_rope)] and k = [k_c, rope(k_rope)]
as [B, S, nh, hd + dr] (the single k_rope row of a token rotated once and stored
to every head) and v packed [B, S, nh, hd].  The backward writes the three
input gradients in one pass: the head sum of dk_rope and dq_rope rotated back.
"""
from __future__ import annotations

import torch

from ._C import ext


class MlaPack(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qc, kv, rp, cos, sin, nh: int, hd: int, dr: int):
        B, S = qc.shape[0], qc.shape[1]
        T = B * S
        qc2 = qc.reshape(T, nh * hd)
        kv2 = kv.reshape(T, 2 * nh * hd)
        rp2 = rp.reshape(T, dr + nh * dr)
        q, k, v = ext().mla_pack_fwd(qc2, kv2, rp2, cos, sin, S, nh, hd, dr)
        ctx.save_for_backward(cos, sin)
        ctx.dims = (B, S, nh, hd, dr)
        return q.view(B, S, nh, hd + dr), k.view(B, S, nh, hd + dr), v.view(B, S, nh, hd)

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin = ctx.saved_tensors
        B, S, nh, hd, dr = ctx.dims
        T = B * S
        z = lambda g, n: torch.zeros(T, n, dtype=torch.bfloat16, device=cos.device) if g is None else g.reshape(T, n)
        dq2 = z(dq, nh * (hd + dr)).contiguous()
        dk2 = z(dk, nh * (hd + dr)).contiguous()
        dv2 = z(dv, nh * hd).contiguous()
        dqc, dkv, drp = ext().mla_pack_bwd(dq2, dk2, dv2, cos, sin, S, nh, hd, dr)
        return (dqc.view(B, S, nh * hd), dkv.view(B, S, 2 * nh * hd), drp.view(B, S, dr + nh * dr),
                None, None, None, None, None)
