"""Model FLOPs per trained token (forward + backward), for MFU and roofline.

Convention: every matmul costs 2 FLOPs per multiply-add in the forward and
twice that in the backward (6 x active matmul parameters per token); causal
attention adds 3 x S x heads x (d_qk + d_v) per token (half of the S x S
scores, fwd + bwd); a chunked SSD scan adds 3 x its per-token tensor work
(intra-chunk C B^T and (L o C B^T) X over half a chunk, state update and
readout), once for Mamba3 as well (its two-term update is computed as one scan).  MoE layers count the routed top-k experts plus the shared ones, and
the router.
"""
from __future__ import annotations


def _attn_gqa(cfg):
    H = cfg.hidden_size
    nh = cfg.num_heads
    hd = H // nh
    kv = (cfg.kv_heads or nh) * hd
    params = H * (nh * hd + 2 * kv) + nh * hd * H
    scores = 3.0 * cfg.max_seq_len * nh * (hd + hd)
    return params, scores


def _attn_mla(cfg):
    H = cfg.hidden_size
    nh = cfg.num_heads
    hd = H // nh
    dr = cfg.d_rope
    kvl, ql = cfg.kv_latent_dim, cfg.q_latent_dim
    params = H * (kvl + ql + dr + nh * dr) + ql * nh * hd + kvl * 2 * nh * hd + nh * hd * H
    scores = 3.0 * cfg.max_seq_len * nh * ((hd + dr) + hd)
    return params, scores


def _mlp(cfg):
    return 3 * cfg.hidden_size * (cfg.intermediate_size or 4 * cfg.hidden_size)


def _moe(cfg):
    H, I = cfg.hidden_size, cfg.intermediate_size or 4 * cfg.hidden_size
    n_shared = cfg.n_shared_experts
    return cfg.num_experts * H + (cfg.experts_per_tok + n_shared) * 3 * H * I


def _mamba2(cfg, mamba3: bool):
    H = cfg.hidden_size
    hs, P, N = cfg.mamba2_num_heads, cfg.mamba2_head_dim, cfg.mamba2_state_size
    g = cfg.mamba2_n_groups or 1
    I = hs * P
    C = cfg.mamba2_chunk_size
    if mamba3:
        R = cfg.mamba3_mimo_rank or 1
        # in_proj (x, z, B, C, dt), lambda, theta, out_proj; MIMO up/down per head
        params = H * (2 * I + 2 * g * N + hs) + H * hs + H * hs * (N // 2) + I * H
        if (cfg.mamba3_mimo_rank or 0) > 1:
            params += 2 * hs * P * P * R
        width = P * R
        # the trapezoidal update runs as ONE scan over the shifted state (the second term
        # folds into the input coefficient and the D skip), so one SSD term is counted
        terms = 1
    else:
        params = H * (2 * I + 2 * g * N + hs) + I * H
        width = P
        terms = 1
    scan = 3.0 * terms * hs * (C * (N + width) + 4 * N * width)
    return params, scan


def _mamba1(cfg):
    H = cfg.hidden_size
    di = 2 * H
    N = 16
    r = max(1, -(-H // 16))
    params = H * 2 * di + di * (r + 2 * N) + r * di + di * H
    scan = 3.0 * 6 * di * N
    return params, scan


def flops_per_token(cfg) -> float:
    """Training FLOPs per token of a :class:`~oxidizr_b200.config.ModelConfig`."""
    total_params = cfg.vocab_size * cfg.hidden_size  # lm_head (the embedding is a gather)
    extra = 0.0
    for i in range(cfg.num_layers):
        kind = cfg.layer_kind(i)
        if kind == "gqa_mlp":
            p, s = _attn_gqa(cfg)
            total_params += p + _mlp(cfg)
            extra += s
        elif kind == "gqa_moe":
            p, s = _attn_gqa(cfg)
            total_params += p + _moe(cfg)
            extra += s
        elif kind == "mla_moe":
            p, s = _attn_mla(cfg)
            total_params += p + _moe(cfg)
            extra += s
        elif kind in ("mamba2", "mamba3"):
            p, s = _mamba2(cfg, kind == "mamba3")
            total_params += p
            extra += s
        else:
            p, s = _mamba1(cfg)
            total_params += p
            extra += s
    return 6.0 * total_params + extra
