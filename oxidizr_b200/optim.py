"""Flat-buffer AdamW with f32 master weights and on-device global-norm clipping.

Upstream: candle ``AdamW`` with ``ParamsAdamW{lr, ..Default}`` (trainer.rs:60-64,
beta (0.9, 0.999), eps 1e-8, weight decay 0.01, decoupled) and
``DistributedAdamW::step`` (distributed/optimizer.rs:126-192).  Upstream
"clipping" only measures the norm and pre-scales the next step's loss
(trainer.rs:131-141); here the gradient is clipped to ``max_grad_norm`` on the
device, with no host synchronisation.

Layout: all parameters of a dtype live in one flat buffer (their ``.data`` is
re-pointed into it), with an f32 master copy, f32 moments and an f32 gradient
buffer whose per-parameter views are exposed as ``param.main_grad``.  The fused
autograd functions accumulate weight gradients straight into those views; one
kernel launch then updates every parameter.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

ALIGN = 64  # elements; keeps every parameter view 256-byte aligned in f32


def _ep_skip_word(device):
    """Device word set when an expert-parallel layer ran over its receive capacity
    this step (the update is then skipped), or None (see parallel/ep.py)."""
    from .parallel.ep import ep_skip_word
    return ep_skip_word(device)


def _ep_step_end(device) -> None:
    from .parallel.ep import ep_step_end
    ep_step_end(device)


@dataclass
class AdamWConfig:
    lr: float = 3e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.01
    max_grad_norm: float = 1.0

    @staticmethod
    def with_lr(lr: float) -> "AdamWConfig":
        return AdamWConfig(lr=lr)


def _round(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


class FlatParams:
    """Owns the flat parameter/gradient/master/moment buffers of a param list."""

    def __init__(self, named_params: Sequence[Tuple[str, torch.nn.Parameter]], device, pad_to: int = ALIGN):
        self.names = [n for n, _ in named_params]
        self.params = [p for _, p in named_params]
        assert self.params, "no parameters"
        self.dtype = self.params[0].dtype
        assert all(p.dtype == self.dtype for p in self.params), "mixed parameter dtypes"
        self.device = torch.device(device)
        offs, o = [], 0
        for p in self.params:
            offs.append(o)
            o += _round(p.numel())
        self.numel = _round(o, pad_to)
        self.offsets = offs
        self.flat = torch.zeros(self.numel, dtype=self.dtype, device=self.device)
        self.grad = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        with torch.no_grad():
            for p, off in zip(self.params, offs):
                n = p.numel()
                self.flat[off:off + n].copy_(p.data.reshape(-1))
                p.data = self.flat[off:off + n].view(p.shape)
                p.main_grad = self.grad[off:off + n].view(p.shape)
        self.master = self.flat.float() if self.dtype != torch.float32 else self.flat

    def view(self, buf: torch.Tensor, i: int) -> torch.Tensor:
        p = self.params[i]
        off = self.offsets[i]
        return buf[off:off + p.numel()].view(p.shape)

    def fold_autograd_grads(self) -> None:
        """Add gradients that arrived through plain autograd (``.grad``) into main_grad."""
        for p in self.params:
            if p.grad is not None:
                p.main_grad.add_(p.grad.to(torch.float32))
                p.grad = None

    def zero_grad(self) -> None:
        self.grad.zero_()
        for p in self.params:
            p.grad = None


def split_local(named_params):
    """(replicated, local): local = expert-parallel shards (``param._oxi_ep_local``)."""
    rep = [(n, p) for n, p in named_params if not getattr(p, "_oxi_ep_local", False)]
    loc = [(n, p) for n, p in named_params if getattr(p, "_oxi_ep_local", False)]
    return rep, loc


class LocalAdamW:
    """AdamW over parameters that each data-parallel rank holds alone (expert
    shards).  Their gradients are sums over every rank's tokens, so the same
    device coefficient (clip x 1/world) as the all-reduced gradients applies."""

    def __init__(self, named_params, cfg: "AdamWConfig", device):
        self.flat = FlatParams(named_params, device)
        self.cfg = cfg
        self.m = torch.zeros_like(self.flat.master)
        self.v = torch.zeros_like(self.flat.master)

    def sq_into(self, buf: torch.Tensor) -> None:
        """buf += sum(g^2) over the local gradients (device)."""
        self.flat.fold_autograd_grads()
        if self.flat.device.type == "cuda":
            from .ops._C import ext
            ext().sqsum(self.flat.grad, buf)
        else:
            buf.add_(self.flat.grad.pow(2).sum())

    def update(self, coef: torch.Tensor, step: int) -> None:
        c, f = self.cfg, self.flat
        bc1, bc2 = 1.0 - c.beta1 ** step, 1.0 - c.beta2 ** step
        if f.device.type == "cuda":
            from .ops._C import ext
            ext().adamw(f.master, f.flat if f.flat is not f.master else None, f.grad, self.m, self.v, c.lr, c.beta1,
                        c.beta2, c.eps, c.weight_decay, bc1, bc2, coef)
        else:
            g = f.grad * coef
            self.m.mul_(c.beta1).add_(g, alpha=1 - c.beta1)
            self.v.mul_(c.beta2).addcmul_(g, g, value=1 - c.beta2)
            p = f.master
            p.sub_(c.lr * (self.m / bc1) / ((self.v / bc2).sqrt() + c.eps) + c.lr * c.weight_decay * p)
            if f.flat is not f.master:
                f.flat.copy_(p)
        f.zero_grad()

    def state_tensors(self) -> Dict[str, torch.Tensor]:
        return {"master": self.flat.master, "exp_avg": self.m, "exp_avg_sq": self.v}

    def sync_master_from_params(self) -> None:
        if self.flat.master is not self.flat.flat:
            with torch.no_grad():
                self.flat.master.copy_(self.flat.flat.float())


class AdamW:
    """Single-process optimizer over a :class:`FlatParams`.

    ``local`` (optional :class:`LocalAdamW`) holds parameters that are not
    replicated; ``_local_sq`` lets a data-parallel subclass reduce their
    squared norm across ranks before the clip coefficient is formed.
    """

    local: Optional["LocalAdamW"] = None

    def _local_sq(self, buf: torch.Tensor) -> None:
        self.local.sq_into(buf)

    def __init__(self, flat: FlatParams, cfg: AdamWConfig):
        self.flat, self.cfg = flat, cfg
        self.m = torch.zeros_like(flat.master)
        self.v = torch.zeros_like(flat.master)
        self.step_count = 0
        dev = flat.device
        self._sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self._coef = torch.ones(1, dtype=torch.float32, device=dev)
        self._norm = torch.zeros(1, dtype=torch.float32, device=dev)
        # [t, 1 - b1^t, 1 - b2^t] advanced on the device, so a captured step (CUDA
        # graph) gets the right bias correction on every replay
        self._step_state = torch.zeros(3, dtype=torch.float32, device=dev)

    @property
    def lr(self) -> float:
        return self.cfg.lr

    def grad_norm_tensor(self) -> torch.Tensor:
        return self._norm

    def step(self, grad_scale: float = 1.0) -> torch.Tensor:
        """One update; returns the pre-clip global grad norm as a device scalar."""
        f, c = self.flat, self.cfg
        f.fold_autograd_grads()
        self.step_count += 1
        t = self.step_count
        bc1 = 1.0 - c.beta1 ** t
        bc2 = 1.0 - c.beta2 ** t
        if f.device.type == "cuda":
            from .ops._C import ext
            e = ext()
            self._sq.zero_()
            e.sqsum(f.grad, self._sq)
            if self.local is not None:
                self._local_sq(self._sq)
            skip = _ep_skip_word(f.device) if self.local is not None else None
            e.clip_coef(self._sq, float(c.max_grad_norm or 0.0), float(grad_scale), self._coef, self._norm,
                        self._step_state, c.beta1, c.beta2, skip)
            e.adamw(f.master, f.flat if f.flat is not f.master else None, f.grad, self.m, self.v, c.lr, c.beta1,
                    c.beta2, c.eps, c.weight_decay, bc1, bc2, self._coef, self._step_state[1:])
            if self.local is not None:
                self.local.update(self._coef, t)
                _ep_step_end(f.device)
        else:
            g = f.grad * grad_scale
            sq = g.pow(2).sum()
            if self.local is not None:
                lsq = torch.zeros(1, dtype=torch.float32)
                self._local_sq(lsq)
                sq = sq + lsq[0] * grad_scale * grad_scale
            nrm = sq.sqrt()
            self._norm.copy_(nrm.reshape(1))
            if not bool(torch.isfinite(nrm)):
                # as on the device: a non-finite gradient norm skips the update
                f.zero_grad()
                if self.local is not None:
                    self.local.flat.zero_grad()
                return self._norm
            coef = 1.0
            if c.max_grad_norm and nrm.item() > c.max_grad_norm:
                coef = c.max_grad_norm / (nrm.item() + 1e-6)
            g = g * coef
            if self.local is not None:
                self.local.update(torch.tensor(coef * grad_scale, dtype=torch.float32), t)
            self.m.mul_(c.beta1).add_(g, alpha=1 - c.beta1)
            self.v.mul_(c.beta2).addcmul_(g, g, value=1 - c.beta2)
            upd = (self.m / bc1) / ((self.v / bc2).sqrt() + c.eps)
            p = f.master
            p.sub_(c.lr * upd + c.lr * c.weight_decay * p)
            if f.flat is not f.master:
                f.flat.copy_(p)
        f.zero_grad()
        return self._norm

    # ------------------------------------------------------------ state
    def sync_master_from_params(self) -> None:
        """Re-derive the f32 master weights after the parameters were loaded."""
        f = self.flat
        if f.master is not f.flat:
            with torch.no_grad():
                f.master.copy_(f.flat.float())
        if self.local is not None:
            self.local.sync_master_from_params()

    def state_tensors(self) -> Dict[str, torch.Tensor]:
        return {"master": self.flat.master, "exp_avg": self.m, "exp_avg_sq": self.v}

    def load_state_tensors(self, d: Dict[str, torch.Tensor], step: int) -> None:
        with torch.no_grad():
            self.flat.master.copy_(d["master"].to(self.flat.master.device))
            if self.flat.flat is not self.flat.master:
                self.flat.flat.copy_(self.flat.master)
            self.m.copy_(d["exp_avg"].to(self.m.device))
            self.v.copy_(d["exp_avg_sq"].to(self.v.device))
            self._step_state.fill_(0.0)
            self._step_state[0] = float(step)
        self.step_count = int(step)
