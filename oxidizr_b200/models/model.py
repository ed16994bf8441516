"""Block dispatcher and the top-level causal LM (model.rs:764-1006).

``LitGPT``: embedding -> blocks -> final RMSNorm -> untied ``lm_head``.
Per-layer block type follows ``ModelConfig.layer_kind`` (model.rs:795-870):
Mamba3 / Mamba2 / Mamba1 for layers in ``mamba_layers``; otherwise MLA+MoE when
``kv_latent_dim`` is set, GQA+MoE when ``num_experts`` is set without MLA (an
extension), else GQA+SwiGLU.

``forward(ids, targets)`` returns ``(ce_loss, aux_losses)`` using the fused
lm_head + cross-entropy kernel (the logits are never returned);
``logits(ids)`` returns them for inference and tests.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import List, Optional, Tuple

import torch
from torch import nn

from ..config import ModelConfig, torch_dtype
from ..ops import api
from .attention import GQAAttention, MLAAttention, SwiGLU
from .common import RefModule, _assign, normal_
from .mamba import Mamba1Block, Mamba2Block, Mamba3Block, NormW
from .moe import MoE


class AttnBlock(RefModule):
    """Pre-norm attention + FFN block (model.rs:904-939)."""

    def __init__(self, cfg: ModelConfig, kind: str, device=None, dtype=None, ep_group=None):
        super().__init__()
        H = cfg.hidden_size
        self.kind = kind
        self.self_attn = MLAAttention(cfg, device, dtype) if kind == "mla_moe" else GQAAttention(cfg, device, dtype)
        if kind in ("mla_moe", "gqa_moe"):
            self.moe = MoE(cfg, device, dtype, ep_group=ep_group)
            self.mlp = None
        else:
            I = cfg.intermediate_size if cfg.intermediate_size is not None else 4 * H
            self.mlp = SwiGLU(H, I, device, dtype)
            self.moe = None
        self.input_layernorm = NormW(H, device=device, dtype=dtype)
        self.post_attention_layernorm = NormW(H, device=device, dtype=dtype)

    def reset_parameters(self, std, gen=None):
        self.self_attn.reset_parameters(std, gen)
        (self.moe or self.mlp).reset_parameters(std, gen)
        self.input_layernorm.reset_parameters()
        self.post_attention_layernorm.reset_parameters()

    def forward(self, x):
        h, x = api.rmsnorm_resid(x, self.input_layernorm.weight, 1e-5)
        x = self.self_attn(h, x)
        h, x = api.rmsnorm_resid(x, self.post_attention_layernorm.weight, 1e-5)
        if self.moe is not None:
            return self.moe(h, x)
        return self.mlp(h, x), None


def make_block(cfg: ModelConfig, i: int, device=None, dtype=None, ep_group=None) -> RefModule:
    kind = cfg.layer_kind(i)
    if kind == "mamba3":
        return Mamba3Block(cfg, device, dtype)
    if kind == "mamba2":
        return Mamba2Block(cfg, device, dtype)
    if kind == "mamba1":
        return Mamba1Block(cfg, device, dtype)
    return AttnBlock(cfg, kind, device, dtype, ep_group=ep_group)


# names of the block containers in the upstream checkpoint
_BLOCK_PREFIX = {"mamba3": "mamba3.", "mamba2": "mamba2.", "mamba1": ""}


class LitGPT(RefModule):
    def __init__(self, cfg: ModelConfig, device=None, dtype=None, ep_group=None):
        super().__init__()
        self.cfg = cfg
        dtype = dtype or torch_dtype(cfg.dtype)
        H, V = cfg.hidden_size, cfg.vocab_size
        self.embed_tokens = nn.Parameter(torch.empty(V, H, device=device, dtype=dtype))
        self.layers = nn.ModuleList([make_block(cfg, i, device, dtype, ep_group) for i in range(cfg.num_layers)])
        self.norm = NormW(H, device=device, dtype=dtype)
        self.lm_head = nn.Parameter(torch.empty(V, H, device=device, dtype=dtype))
        # Optional callable given the parameters a part of the forward is about to
        # use; a sharded data-parallel optimizer sets it so that the forward waits
        # for each parameter bucket's all-gather only when it first needs it.
        self._param_gate = None

    def reset_parameters(self, seed: Optional[int] = None):
        gen = None
        if seed is not None:
            gen = torch.Generator(device=self.embed_tokens.device)
            gen.manual_seed(seed)
        std = self.cfg.std
        normal_(self.embed_tokens, std, gen)
        normal_(self.lm_head, std, gen)
        self.norm.reset_parameters()
        for layer in self.layers:
            layer.reset_parameters(std, gen)
        return self

    # ------------------------------------------------------------ forward
    def hidden(self, ids: torch.Tensor) -> Tuple[torch.Tensor, List[torch.Tensor]]:
        gate = self._param_gate
        if gate is not None:
            gate((self.embed_tokens,))
        x = api.embedding(ids, self.embed_tokens)
        aux = []
        for layer in self.layers:
            if gate is not None:
                gate(layer.parameters())
            x, a = layer(x)
            if a is not None:
                aux.append(a)
        if gate is not None:
            gate((self.norm.weight, self.lm_head))
        x = api.rmsnorm(x, self.norm.weight, 1e-5)
        return x, aux

    def forward(self, ids: torch.Tensor, targets: torch.Tensor):
        x, aux = self.hidden(ids)
        loss = api.linear_cross_entropy(x, self.lm_head, targets)
        return loss, aux

    def logits(self, ids: torch.Tensor) -> torch.Tensor:
        x, _ = self.hidden(ids)
        return torch.nn.functional.linear(x.float(), self.lm_head.float())

    # ------------------------------------------------------------ checkpoint names
    def export_ref(self, prefix: str = "", out: Optional[dict] = None) -> "OrderedDict[str, torch.Tensor]":
        out = OrderedDict() if out is None else out
        out[prefix + "embed_tokens.weight"] = self.embed_tokens.detach()
        for i, layer in enumerate(self.layers):
            kind = self.cfg.layer_kind(i)
            base = f"{prefix}layers.{i}."
            if kind in ("mamba3", "mamba2"):
                layer.export_ref(base + _BLOCK_PREFIX[kind], out)
            else:
                layer.export_ref(base, out)
        out[prefix + "norm.weight"] = self.norm.weight.detach()
        out[prefix + "lm_head.weight"] = self.lm_head.detach()
        return out

    def _ep_group(self):
        for m in self.modules():
            if isinstance(m, MoE) and m.ep_size > 1:
                return m.ep_group
        return None

    def export_ref_gathered(self, dst: int = 0) -> Optional["OrderedDict[str, torch.Tensor]"]:
        """``export_ref`` with the expert shards of expert-parallel layers gathered
        to rank ``dst`` (collective over the expert-parallel group; other ranks
        get None).  Without expert parallelism it is plain ``export_ref``."""
        sd = self.export_ref()
        g = self._ep_group()
        if g is None:
            return sd
        import torch.distributed as dist
        mine = {k: v.cpu() for k, v in sd.items() if ".experts." in k}
        rank = dist.get_rank(g)
        parts = [None] * dist.get_world_size(g) if rank == dst else None
        dist.gather_object(mine, parts, dst=dist.get_global_rank(g, dst), group=g)
        if rank != dst:
            return None
        out = OrderedDict((k, v) for k, v in sd.items() if ".experts." not in k)
        for part in parts:
            out.update(part)
        return out

    def import_ref(self, sd: dict, prefix: str = "") -> None:
        _assign(self.embed_tokens, sd, prefix + "embed_tokens.weight")
        for i, layer in enumerate(self.layers):
            kind = self.cfg.layer_kind(i)
            base = f"{prefix}layers.{i}."
            if kind in ("mamba3", "mamba2"):
                layer.import_ref(base + _BLOCK_PREFIX[kind], sd)
            else:
                layer.import_ref(base, sd)
        _assign(self.norm.weight, sd, prefix + "norm.weight")
        _assign(self.lm_head, sd, prefix + "lm_head.weight")


def build_model(cfg: ModelConfig, device="cpu", seed: Optional[int] = None, ep_group=None,
                dtype=None) -> LitGPT:
    m = LitGPT(cfg, device=device, dtype=dtype, ep_group=ep_group)
    m.reset_parameters(seed if seed is not None else (cfg.seed if cfg.seed is not None else 0))
    return m
