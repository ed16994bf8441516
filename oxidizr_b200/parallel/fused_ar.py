"""Fused NVLink data parallelism: bucketed bf16 reduce-scatter during backward,
cross-rank clip, sharded AdamW and a P2P parameter all-gather (csrc/comm.cu).

This replaces the upstream NCCL synchroniser (distributed/nccl.rs:153-184,
which stages every parameter through host memory and all-reduces on rank 0's
communicator only) with one process per GPU and peer-to-peer NVLink traffic
issued from our own kernels:

* buckets of parameters (reverse order of use) are reduced as soon as
  backward has produced all their gradients, on a side stream, so the
  transfers overlap the rest of backward: each rank casts its gradient to
  bf16 in its send buffer, and the owner of each shard reads the W slices
  over NVLink and sums them in f32 (``OXI_RS_MODE=push``: NVLink stores into
  the owners' receive slots, then a local sum);
* each rank keeps f32 master weights and AdamW moments for its 1/W shard of
  every bucket only (optimizer state sharded W ways);
* after backward: one tiny kernel exchanges partial norms (global-norm clip),
  then one kernel updates the owned shards and writes the new bf16 parameters
  straight into every peer's parameter buffer.

NCCL (through torch.distributed) is used only to exchange IPC handles at
start-up and for checkpoint gathers.
"""
from __future__ import annotations

import os
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..ops._C import ext, status
from ..optim import AdamWConfig, LocalAdamW, split_local

ALIGN = 64


def _roundup(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class SymmetricBuffer:
    """A device buffer of the same size on every rank, mapped by all peers."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        self.device = device
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.local, handle = ext().ipc_alloc(int(nbytes), device.index)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        self._opened = []
        for i, h in enumerate(handles):
            if i == self.rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                p = ext().ipc_open(h, device.index)
                self.ptrs.append(p)
                self._opened.append(p)
        self.ptr_table = torch.tensor(self.ptrs, dtype=torch.int64, device=device)

    def close(self):
        for p in self._opened:
            ext().ipc_close(p, self.device.index)
        self._opened = []


class FusedDDPAdamW:
    """Drop-in optimizer for data-parallel training over NVLink (sync backend ``fused``)."""

    collective_state = True  # state_tensors() gathers the shards: every rank calls it

    def __init__(self, named_params: Sequence[Tuple[str, torch.nn.Parameter]], cfg: AdamWConfig, device,
                 group=None, bucket_bytes: int = 32 << 20, rs_ctas: Optional[int] = None,
                 peer_timeout_s: float = 30.0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        self.rank = dist.get_rank(group)
        self.W = dist.get_world_size(group)
        # CTAs per reduce-scatter kernel (they share SMs with the backward GEMMs)
        self.rs_ctas = int(rs_ctas if rs_ctas is not None else os.environ.get("OXI_RS_CTAS", 64))
        # a peer that has not posted its flag within this time is reported as failed
        self.wait_ns = int(peer_timeout_s * 1e9)
        named_params, local = split_local(list(named_params))
        # expert-parallel shards: updated locally with the same clip coefficient
        self.local = LocalAdamW(local, cfg, device) if local else None
        self.names = [n for n, _ in named_params]
        self.params = [p for _, p in named_params]
        assert all(p.dtype == torch.bfloat16 for p in self.params), "fused DDP needs bf16 parameters"
        W = self.W
        # ---- layout: buckets in reverse parameter order, each padded to W * ALIGN
        per = max(bucket_bytes // 2, 1)
        order = list(range(len(self.params)))[::-1]
        groups, cur, cur_n = [], [], 0
        for i in order:
            cur.append(i)
            cur_n += _roundup(self.params[i].numel(), ALIGN)
            if cur_n >= per:
                groups.append(cur)
                cur, cur_n = [], 0
        if cur:
            groups.append(cur)
        assert len(groups) <= 512, "too many buckets; raise bucket_bytes"
        self.offsets = [0] * len(self.params)
        self.buckets = []  # (lo, len, shard_off, param indices)
        o = 0
        shard_off = 0
        for g in groups:
            lo = o
            for i in g:
                self.offsets[i] = o
                o += _roundup(self.params[i].numel(), ALIGN)
            ln = _roundup(o - lo, W * ALIGN)
            o = lo + ln
            self.buckets.append([lo, ln, shard_off, g])
            shard_off += ln // W
        self.N = o
        self.shard_numel = shard_off
        # ---- buffers
        dev = self.device
        # bf16 gradient exchange buffer: this rank's send buffer (pull mode) or
        # the receive slots of its shards (push mode)
        self.xfer = SymmetricBuffer(self.N * 2, dev, group)
        self.rs_mode = 1 if os.environ.get("OXI_RS_MODE", "pull") == "push" else 0
        self.param = SymmetricBuffer(self.N * 2, dev, group)
        self.pad = SymmetricBuffer(ext().pad_words() * 4, dev, group)
        self.flat = self.param.local.view(torch.bfloat16)
        self.pad_local = self.pad.local.view(torch.int32)
        self.grad = torch.zeros(self.N, dtype=torch.float32, device=dev)
        with torch.no_grad():
            for p, off in zip(self.params, self.offsets):
                n = p.numel()
                self.flat[off:off + n].copy_(p.data.reshape(-1))
                p.data = self.flat[off:off + n].view(p.shape)
                p.main_grad = self.grad[off:off + n].view(p.shape)
            # identical replicas: take rank 0's initial parameters
            dist.broadcast(self.flat, src=0, group=group)
        self.rgrad = torch.zeros(self.shard_numel, dtype=torch.float32, device=dev)
        self.master = torch.empty(self.shard_numel, dtype=torch.float32, device=dev)
        for lo, ln, so, _ in self.buckets:
            sh = ln // W
            self.master[so:so + sh].copy_(self.flat[lo + self.rank * sh: lo + (self.rank + 1) * sh].float())
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.bucket_table = torch.tensor([[b[0], b[1], b[2]] for b in self.buckets], dtype=torch.int64, device=dev)
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self._coef = torch.zeros(1, dtype=torch.float32, device=dev)
        self._norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self._done = torch.zeros(1, dtype=torch.int32, device=dev)
        self._push_done = torch.zeros(512, dtype=torch.int32, device=dev)
        self.comm_stream = torch.cuda.Stream(device=dev)
        self.epoch = 1
        self.step_count = 0
        self.accumulating = False
        self._pending = [len(b[3]) for b in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._sumsq_zeroed = False
        for bi, b in enumerate(self.buckets):
            for i in b[3]:
                self.params[i]._oxi_grad_ready = (lambda k=bi: self._on_ready(k))
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    @property
    def lr(self) -> float:
        return self.cfg.lr

    # ------------------------------------------------------------ backward hooks
    def _on_ready(self, bi: int):
        if self.accumulating:
            return
        self._pending[bi] -= 1
        if self._pending[bi] == 0:
            self._launch(bi)

    def _launch(self, bi: int):
        if self._launched[bi]:
            return
        self._launched[bi] = True
        lo, ln, so, _ = self.buckets[bi]
        e = ext()
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            if not self._sumsq_zeroed:
                self._sumsq.zero_()
                self._sumsq_zeroed = True
            e.rs_bucket(self.rs_mode, self.grad, self.xfer.ptr_table, self.xfer.local, self.pad.ptr_table,
                        self.pad_local, self._push_done, self.rank, self.W, bi, self.epoch, lo, ln,
                        self.rgrad[so:so + ln // self.W], self._sumsq, self.rs_ctas, status(self.device), self.wait_ns)

    # ------------------------------------------------------------ step
    def step(self, grad_scale: float = 1.0) -> torch.Tensor:
        for p in self.params:  # gradients that came through plain autograd
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None
        for bi in range(len(self.buckets)):
            self._launch(bi)
        cur = torch.cuda.current_stream(self.device)
        cur.wait_stream(self.comm_stream)
        c = self.cfg
        e = ext()
        self.step_count += 1
        t = self.step_count
        if self.local is not None:
            self.local.sq_into(self._sumsq)  # joins this rank's partial of the global norm
        e.norm_exchange(self.pad.ptr_table, self.pad_local, self.rank, self.W, self.epoch, self._sumsq,
                        float(c.max_grad_norm or 0.0), self._coef, self._norm, status(self.device),
                        self.wait_ns)
        if grad_scale != 1.0:
            self._coef.mul_(grad_scale)
        e.adamw_allgather(self.bucket_table, self.rank, self.W, self.rgrad, self.master, self.m, self.v,
                          self.param.ptr_table, self.pad.ptr_table, self.pad_local, self.epoch, c.lr, c.beta1,
                          c.beta2, c.eps, c.weight_decay, 1.0 - c.beta1 ** t, 1.0 - c.beta2 ** t, self._coef,
                          self._done, status(self.device), self.wait_ns)
        if self.local is not None:
            self.local.update(self._coef, t)
        self.grad.zero_()
        self.epoch += 1
        self._pending = [len(b[3]) for b in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._sumsq_zeroed = False
        return self._norm

    # ------------------------------------------------------------ state (collective)
    def _gather_full(self, shard: torch.Tensor) -> torch.Tensor:
        parts = [torch.empty_like(shard) for _ in range(self.W)]
        dist.all_gather(parts, shard, group=self.group)
        full = torch.zeros(self.N, dtype=shard.dtype, device=shard.device)
        for lo, ln, so, _ in self.buckets:
            sh = ln // self.W
            for r in range(self.W):
                full[lo + r * sh: lo + (r + 1) * sh].copy_(parts[r][so:so + sh])
        return full

    def state_tensors(self):
        """Full master / moments in flat layout (collective: every rank must call)."""
        return {"master": self._gather_full(self.master), "exp_avg": self._gather_full(self.m),
                "exp_avg_sq": self._gather_full(self.v)}

    def sync_master_from_params(self) -> None:
        """Re-derive this rank's f32 master shards after the parameters were loaded."""
        with torch.no_grad():
            for lo, ln, so, _ in self.buckets:
                sh = ln // self.W
                self.master[so:so + sh].copy_(self.flat[lo + self.rank * sh: lo + (self.rank + 1) * sh].float())
        if self.local is not None:
            self.local.sync_master_from_params()

    def load_state_tensors(self, d, step: int):
        with torch.no_grad():
            for key, dst in (("master", self.master), ("exp_avg", self.m), ("exp_avg_sq", self.v)):
                full = d[key].to(self.device)
                for lo, ln, so, _ in self.buckets:
                    sh = ln // self.W
                    dst[so:so + sh].copy_(full[lo + self.rank * sh: lo + (self.rank + 1) * sh])
            # parameters follow the master weights
            full = d["master"].to(self.device)
            self.flat.copy_(full[: self.N].to(torch.bfloat16))
        self.step_count = int(step)

    def close(self):
        torch.cuda.synchronize(self.device)
        for b in (self.xfer, self.param, self.pad):
            b.close()
