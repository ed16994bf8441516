"""Attention blocks: Llama-style GQA (model.rs:290-426) and MLA with decoupled
RoPE (model.rs:124-286), plus the dense SwiGLU MLP (model.rs:430-455)."""
from __future__ import annotations

import math

import torch
from torch import nn

from ..ops import api
from .common import RefModule, RopeCache, _assign, interleave_gu, normal_, split_gu, take


class GQAAttention(RefModule):
    """q/k/v/o projections without bias, rotate-half RoPE over the full head
    dim, causal softmax attention with scale 1/sqrt(head_dim).

    Kernel layout: one fused ``w_qkv`` [(nh + 2 kvh) * hd, H]; the QKV GEMM
    applies RoPE in its epilogue; the output projection adds the residual in
    its epilogue.
    """

    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        H = cfg.hidden_size
        self.nh = cfg.num_heads
        self.kvh = cfg.kv_heads if cfg.kv_heads is not None else cfg.num_heads
        self.hd = H // self.nh
        self.theta = cfg.rope_theta
        self.max_seq = cfg.max_seq_len
        self.scale = 1.0 / math.sqrt(self.hd)
        n_qkv = (self.nh + 2 * self.kvh) * self.hd
        self.w_qkv = nn.Parameter(torch.empty(n_qkv, H, device=device, dtype=dtype))
        self.o_proj = nn.Parameter(torch.empty(H, self.nh * self.hd, device=device, dtype=dtype))

    def reset_parameters(self, std: float, gen=None):
        normal_(self.w_qkv, std, gen)
        normal_(self.o_proj, std, gen)

    def forward(self, h: torch.Tensor, resid: torch.Tensor) -> torch.Tensor:
        B, S, _ = h.shape
        cos, sin = RopeCache.get(self.hd, S, self.theta, h.device)
        o = api.attention_rope(h, self.w_qkv, cos, sin, self.nh, self.kvh, self.hd, self.scale)
        return api.linear(o, self.o_proj, resid=resid)

    def export_ref(self, prefix, out):
        qc, kc = self.nh * self.hd, self.kvh * self.hd
        w = self.w_qkv.detach()
        out[prefix + "q_proj.weight"] = w[:qc]
        out[prefix + "k_proj.weight"] = w[qc:qc + kc]
        out[prefix + "v_proj.weight"] = w[qc + kc:]
        out[prefix + "o_proj.weight"] = self.o_proj.detach()

    def import_ref(self, prefix, sd):
        w = torch.cat([take(sd, prefix + "q_proj.weight"), take(sd, prefix + "k_proj.weight"),
                       take(sd, prefix + "v_proj.weight")], 0)
        _assign(self.w_qkv, sd, prefix + "q_proj.weight", w)
        _assign(self.o_proj, sd, prefix + "o_proj.weight")


class MLAAttention(RefModule):
    """Multi-head latent attention with decoupled RoPE (model.rs:196-256).

    c_kv = W_dkv x, c_q = W_dq x, q_rope = W_qr x (per head), k_rope = W_kr x
    (one, shared by all heads), q = W_uq c_q, k = W_uk c_kv, v = W_uv c_kv,
    Q = [q, rope(q_rope)], K = [k, rope(k_rope)], scale 1/sqrt(hd + d_rope).
    Kernel layout: the four projections of x are one GEMM (``w_down``), and
    W_uk/W_uv one GEMM (``w_ukv``).
    """

    def __init__(self, cfg, device=None, dtype=None):
        super().__init__()
        H = cfg.hidden_size
        self.nh = cfg.num_heads
        self.hd = H // self.nh
        self.dr = cfg.d_rope
        self.kvl = cfg.kv_latent_dim
        self.ql = cfg.q_latent_dim
        self.theta = cfg.rope_theta
        self.scale = 1.0 / math.sqrt(self.hd + self.dr)
        self.n_down = self.kvl + self.ql + self.dr + self.nh * self.dr
        self.w_down = nn.Parameter(torch.empty(self.n_down, H, device=device, dtype=dtype))
        self.w_uq = nn.Parameter(torch.empty(self.nh * self.hd, self.ql, device=device, dtype=dtype))
        self.w_ukv = nn.Parameter(torch.empty(2 * self.nh * self.hd, self.kvl, device=device, dtype=dtype))
        self.o_proj = nn.Parameter(torch.empty(H, self.nh * self.hd, device=device, dtype=dtype))

    def reset_parameters(self, std, gen=None):
        for p in (self.w_down, self.w_uq, self.w_ukv, self.o_proj):
            normal_(p, std, gen)

    def forward(self, h, resid):
        B, S, _ = h.shape
        nh, hd, dr = self.nh, self.hd, self.dr
        d = api.linear(h, self.w_down)
        # c_kv | c_q | k_rope | q_rope blocks as views; one gradient buffer in the backward
        c_kv, c_q, rp = api.split_cols(d, [self.kvl, self.ql, dr + nh * dr])
        q_c = api.linear(c_q, self.w_uq)
        kv = api.linear(c_kv, self.w_ukv)
        cos, sin = RopeCache.get(dr, S, self.theta, h.device)
        # RoPE on the rope parts and the shared k_rope broadcast to every head, in one kernel
        q, k, v = api.mla_qkv(q_c, kv, rp, cos, sin, nh, hd, dr)
        o = api.attention(q, k, v, self.scale, causal=True).reshape(B, S, nh * hd)
        return api.linear(o, self.o_proj, resid=resid)

    def _splits(self):
        a = self.kvl
        b = a + self.ql
        c = b + self.dr
        return a, b, c

    def export_ref(self, prefix, out):
        a, b, c = self._splits()
        w = self.w_down.detach()
        out[prefix + "w_dkv.weight"] = w[:a]
        out[prefix + "w_dq.weight"] = w[a:b]
        out[prefix + "w_kr.weight"] = w[b:c]
        out[prefix + "w_qr.weight"] = w[c:]
        out[prefix + "w_uq.weight"] = self.w_uq.detach()
        n = self.nh * self.hd
        out[prefix + "w_uk.weight"] = self.w_ukv.detach()[:n]
        out[prefix + "w_uv.weight"] = self.w_ukv.detach()[n:]
        out[prefix + "o_proj.weight"] = self.o_proj.detach()

    def import_ref(self, prefix, sd):
        w = torch.cat([take(sd, prefix + k) for k in ("w_dkv.weight", "w_dq.weight", "w_kr.weight", "w_qr.weight")],
                      0)
        _assign(self.w_down, sd, prefix + "w_dkv.weight", w)
        _assign(self.w_uq, sd, prefix + "w_uq.weight")
        _assign(self.w_ukv, sd, prefix + "w_uk.weight",
                torch.cat([take(sd, prefix + "w_uk.weight"), take(sd, prefix + "w_uv.weight")], 0))
        _assign(self.o_proj, sd, prefix + "o_proj.weight")


class SwiGLU(RefModule):
    """down(silu(gate x) * up x), no bias; gate/up fused and row-interleaved."""

    def __init__(self, H: int, I: int, device=None, dtype=None):
        super().__init__()
        self.H, self.I = H, I
        self.w_gu = nn.Parameter(torch.empty(2 * I, H, device=device, dtype=dtype))
        self.w_down = nn.Parameter(torch.empty(H, I, device=device, dtype=dtype))

    def reset_parameters(self, std, gen=None):
        normal_(self.w_gu, std, gen)
        normal_(self.w_down, std, gen)

    def forward(self, h, resid=None):
        return api.swiglu_mlp(h, self.w_gu, self.w_down, resid)

    def export_ref(self, prefix, out):
        g, u = split_gu(self.w_gu.detach())
        out[prefix + "gate_proj.weight"] = g
        out[prefix + "up_proj.weight"] = u
        out[prefix + "down_proj.weight"] = self.w_down.detach()

    def import_ref(self, prefix, sd):
        w = interleave_gu(take(sd, prefix + "gate_proj.weight"), take(sd, prefix + "up_proj.weight"))
        _assign(self.w_gu, sd, prefix + "gate_proj.weight", w)
        _assign(self.w_down, sd, prefix + "down_proj.weight")
