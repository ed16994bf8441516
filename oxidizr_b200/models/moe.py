"""Fine-grained mixture of experts (model.rs:461-752), computed sparsely.

Router ``Linear(H, E)`` without bias; routing probabilities are the softmax of
the router logits; each token picks its top-k experts by logit and weights
them with the softmax over those k logits (model.rs:541-556).  Shared experts
are always on (model.rs:574-576).  Upstream runs every expert densely on every
token and weighs the outputs with a dense [T, E] matrix; running each expert
only on its routed tokens gives the same output for the same routing.

Auxiliary load-balancing loss:
* ``mean_sq`` (default, upstream formula model.rs:585-590):
  ``mean_e((mean_t p_te)^2)`` -- differentiable here (upstream detaches it);
* ``switch``: ``E * sum_e f_e * P_e`` with f_e the routed-token fraction.

Expert weights are stored stacked ([E, 2I, H] gate|up interleaved, [E, H, I])
so a grouped GEMM can address them; ``export_ref`` writes the upstream
per-expert names ``experts.{e}.{gate,up,down}_proj.weight``.  Several shared
experts are one SwiGLU of width ``num_shared_experts * I`` (the sum of SwiGLU
experts equals one SwiGLU over the concatenated intermediate dimension).

With expert parallelism (``ep_group`` set) each rank holds E/ep experts and the
token dispatch/combine goes through :mod:`oxidizr_b200.parallel.ep`.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import api
from .attention import SwiGLU
from .common import RefModule, _assign, interleave_gu, normal_, split_gu, take


def _grouped_ok(x, w_gu) -> bool:
    if not x.is_cuda:
        return False
    from ..ops.moe_kernels import grouped_ok
    return grouped_ok(x, w_gu)


def route(logits: torch.Tensor, k: int):
    """Top-k routing: returns (probs [T,E] f32, top_idx [T,k] int64, top_w [T,k] f32)."""
    lf = logits.float()
    probs = torch.softmax(lf, -1)
    topv, topi = torch.topk(lf, k, dim=-1)
    topw = torch.softmax(topv, -1)
    return probs, topi, topw


def aux_loss(probs: torch.Tensor, topi: torch.Tensor, E: int, kind: str = "mean_sq") -> torch.Tensor:
    return aux_from_usage(probs.mean(0), torch.bincount(topi.reshape(-1), minlength=E), topi.numel(), E, kind)


def aux_from_usage(usage: torch.Tensor, counts: torch.Tensor, n_sel: int, E: int, kind: str) -> torch.Tensor:
    """Load-balancing loss from the mean routing probability per expert."""
    if kind == "switch":
        f = counts.float() / n_sel
        return E * (f.detach() * usage).sum()
    return usage.pow(2).mean()


def route_with_aux(logits: torch.Tensor, k: int, E: int, kind: str):
    """(top_idx, top_w, aux, counts): the fused router kernel on CUDA, torch ops elsewhere."""
    if logits.is_cuda:
        from ..ops.moe_kernels import RouterTopK, router_ok
        if router_ok(logits, k):
            topi, topw, usage, counts = RouterTopK.apply(logits, k)
            return topi, topw, aux_from_usage(usage, counts, topi.numel(), E, kind), counts
    probs, topi, topw = route(logits, k)
    return topi, topw, aux_loss(probs, topi, E, kind), None


class MoE(RefModule):
    def __init__(self, cfg, device=None, dtype=None, ep_group=None):
        super().__init__()
        H = cfg.hidden_size
        self.E = cfg.num_experts
        self.k = cfg.experts_per_tok
        self.I = cfg.intermediate_size
        self.H = H
        self.aux_kind = cfg.moe_aux_loss or "mean_sq"
        self.ep_group = ep_group
        if ep_group is not None:
            import torch.distributed as dist
            self.ep_size = dist.get_world_size(ep_group)
            self.ep_rank = dist.get_rank(ep_group)
        else:
            self.ep_size, self.ep_rank = 1, 0
        assert self.E % self.ep_size == 0, "num_experts must be divisible by the expert-parallel size"
        self.E_local = self.E // self.ep_size
        self.router = nn.Parameter(torch.empty(self.E, H, device=device, dtype=dtype))
        self.w_gu = nn.Parameter(torch.empty(self.E_local, 2 * self.I, H, device=device, dtype=dtype))
        self.w_down = nn.Parameter(torch.empty(self.E_local, H, self.I, device=device, dtype=dtype))
        self.n_shared = cfg.n_shared_experts
        self.shared = SwiGLU(H, self.n_shared * self.I, device, dtype) if self.n_shared > 0 else None
        # under expert parallelism the expert weights are shards, not replicas:
        # the data-parallel optimizers keep them out of the gradient all-reduce
        if self.ep_size > 1:
            self.w_gu._oxi_ep_local = True
            self.w_down._oxi_ep_local = True

    def reset_parameters(self, std, gen=None):
        normal_(self.router, std, gen)
        if self.ep_size > 1:
            # draw every expert (same stream of numbers as one process holding all
            # of them) and keep this rank's slice
            lo = self.ep_rank * self.E_local
            for p in (self.w_gu, self.w_down):
                full = torch.empty((self.E,) + tuple(p.shape[1:]), device=p.device, dtype=p.dtype)
                normal_(full, std, gen)
                with torch.no_grad():
                    p.copy_(full[lo:lo + self.E_local])
                del full
        else:
            normal_(self.w_gu, std, gen)
            normal_(self.w_down, std, gen)
        if self.shared is not None:
            self.shared.reset_parameters(std, gen)

    # ------------------------------------------------------------ compute
    def _experts_local(self, xs: torch.Tensor, counts) -> torch.Tensor:
        """Run local expert e on rows [off_e, off_e + counts[e]) of xs."""
        ys = torch.empty_like(xs)
        off = 0
        for e, c in enumerate(counts):
            if c:
                ys[off:off + c] = api.swiglu_mlp(xs[off:off + c], self.w_gu[e], self.w_down[e])
            off += c
        return ys

    def forward(self, h: torch.Tensor, resid: torch.Tensor):
        B, S, H = h.shape
        x = h.reshape(-1, H)
        logits = api.linear(x, self.router)
        topi, topw, aux, counts = route_with_aux(logits, self.k, self.E, self.aux_kind)
        if self.ep_size > 1:
            from ..parallel import ep
            if counts is not None and ep.nvlink_ok(self, x):
                y = ep.ep_moe_nvlink(self, x, topi, topw, counts, resid.reshape(-1, H)).view(B, S, H)
                return (self.shared(h, y) if self.shared is not None else y), aux
            y = ep.ep_moe(self, x, topi, topw)
        elif _grouped_ok(x, self.w_gu):
            from ..ops.moe_kernels import GroupedExperts
            r = resid.reshape(-1, H)
            if self.shared is not None:
                y = GroupedExperts.apply(x, topi, topw, self.w_gu, self.w_down, r).view(B, S, H)
                return self.shared(h, y), aux
            return GroupedExperts.apply(x, topi, topw, self.w_gu, self.w_down, r).view(B, S, H), aux
        else:
            flat_e = topi.reshape(-1)
            order = torch.argsort(flat_e, stable=True)
            tok = order // self.k
            counts = torch.bincount(flat_e, minlength=self.E).tolist()
            xs = x.index_select(0, tok)
            ys = self._experts_local(xs, counts)
            wts = topw.reshape(-1).index_select(0, order).to(ys.dtype)
            y = torch.zeros_like(x).index_add_(0, tok, ys * wts[:, None])
        y = y.view(B, S, H)
        if self.shared is not None:
            return self.shared(h, resid + y), aux
        return resid + y, aux

    # ------------------------------------------------------------ names
    def export_ref(self, prefix, out):
        out[prefix + "router.gate.weight"] = self.router.detach()
        base = self.ep_rank * self.E_local
        for e in range(self.E_local):
            g, u = split_gu(self.w_gu.detach()[e])
            p = f"{prefix}experts.{base + e}."
            out[p + "gate_proj.weight"] = g
            out[p + "up_proj.weight"] = u
            out[p + "down_proj.weight"] = self.w_down.detach()[e]
        if self.shared is not None:
            self.shared.export_ref(prefix + "shared_expert.", out)

    def import_ref(self, prefix, sd):
        _assign(self.router, sd, prefix + "router.gate.weight")
        base = self.ep_rank * self.E_local
        with torch.no_grad():
            for e in range(self.E_local):
                p = f"{prefix}experts.{base + e}."
                w = interleave_gu(take(sd, p + "gate_proj.weight"), take(sd, p + "up_proj.weight"))
                self.w_gu[e].copy_(w.to(self.w_gu.dtype))
                self.w_down[e].copy_(take(sd, p + "down_proj.weight").to(self.w_down.dtype))
        if self.shared is not None:
            self.shared.import_ref(prefix + "shared_expert.", sd)
