"""Shared model utilities: initialisation, RoPE tables, reference-name export.

Modules in this package keep some parameters fused for the kernels (q|k|v,
gate|up interleaved in 128-row blocks, MLA down projections, stacked experts)
and translate to/from the upstream per-tensor names (``model.rs``,
``mamba*.rs`` ``vb.pp(...)`` prefixes) in ``export_ref`` / ``import_ref``.

Upstream: weight names from ``VarBuilder`` prefixes (model.rs:320-323,442-444,517-530,856-866,
model.rs:964-972; mamba.rs:71-97; mamba2.rs:263-300; mamba3.rs:303-378); RoPE tables model.rs:43-66.
"""
from __future__ import annotations

import math
from typing import Dict

import torch
from torch import nn

from ..ops import reference as R

BLOCK = 128  # row interleave granularity of fused gate/up weights


def normal_(t: torch.Tensor, std: float, gen: torch.Generator = None) -> torch.Tensor:
    """In-place normal(0, std) init drawn in f32 on the generator's device."""
    with torch.no_grad():
        dev = gen.device if gen is not None else t.device
        v = torch.empty(t.shape, dtype=torch.float32, device=dev).normal_(0.0, std, generator=gen)
        t.copy_(v)
    return t


def interleave_gu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """[I, H] gate and up -> [2I, H] with rows [g0:128, u0:128, g128:256, ...].
    Falls back to plain concatenation when I is not a multiple of 128."""
    I = g.shape[0]
    if I % BLOCK:
        return torch.cat([g, u], 0)
    return torch.stack([g.reshape(I // BLOCK, BLOCK, -1), u.reshape(I // BLOCK, BLOCK, -1)], 1).reshape(2 * I, -1)


def split_gu(gu: torch.Tensor):
    I = gu.shape[0] // 2
    if I % BLOCK:
        return gu[:I], gu[I:]
    v = gu.reshape(I // BLOCK, 2, BLOCK, -1)
    return v[:, 0].reshape(I, -1), v[:, 1].reshape(I, -1)


class RopeCache:
    """f32 cos/sin half tables [S, dim/2] per (dim, seq, theta, device)."""
    _cache: Dict = {}

    @classmethod
    def get(cls, dim: int, seq: int, theta: float, device):
        key = (dim, seq, float(theta), str(device))
        t = cls._cache.get(key)
        if t is None:
            c, s = R.rope_tables(dim, seq, theta, device=device, dtype=torch.float32)
            t = (c.contiguous(), s.contiguous())
            cls._cache[key] = t
        return t


class RefModule(nn.Module):
    """Mixin: map fused parameters to upstream names."""

    def export_ref(self, prefix: str, out: dict) -> None:  # pragma: no cover - overridden
        for n, p in self.named_parameters(recurse=False):
            out[prefix + n] = p.detach()
        for n, m in self.named_children():
            if isinstance(m, RefModule):
                m.export_ref(prefix + n + ".", out)

    def import_ref(self, prefix: str, sd: dict) -> None:
        for n, p in self.named_parameters(recurse=False):
            _assign(p, sd, prefix + n)
        for n, m in self.named_children():
            if isinstance(m, RefModule):
                m.import_ref(prefix + n + ".", sd)


def _assign(p: torch.Tensor, sd: dict, key: str, value: torch.Tensor = None) -> None:
    if value is None:
        if key not in sd:
            raise KeyError(f"missing tensor in checkpoint: {key}")
        value = sd[key]
    if tuple(value.shape) != tuple(p.shape):
        raise ValueError(f"shape mismatch for {key}: checkpoint {tuple(value.shape)} vs model {tuple(p.shape)}")
    with torch.no_grad():
        p.copy_(value.to(device=p.device, dtype=p.dtype))


def take(sd: dict, key: str) -> torch.Tensor:
    if key not in sd:
        raise KeyError(f"missing tensor in checkpoint: {key}")
    return sd[key]
