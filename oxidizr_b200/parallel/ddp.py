"""Data-parallel gradient synchronisation + optimizer step.

Upstream's ``GradientSynchronizer`` (distributed/sync.rs:101-140) with backends
``single | cpustaging | nccl`` runs in one process and never reduces across
real replicas (distributed/nccl.rs:153-184 calls all_reduce on rank 0's
communicator only).  Here every rank is its own process and gradients are
really reduced:

* ``cpustaging`` -- gloo all-reduce of the flat f32 gradient (CPU tensors or
  host-staged GPU tensors); used by the CPU multi-process tests;
* ``nccl``       -- bucketed NCCL all-reduce, each bucket launched on a side
  stream as soon as backward has produced all of its gradients (baseline);
* ``nccl_sharded`` -- the sharded algorithm of the product path (bucketed
  bf16 reduce-scatter overlapped with backward, sharded AdamW, bucketed bf16
  all-gather overlapped with the next forward) with NCCL as the transport:
  the like-for-like baseline of ``fused``;
* ``fused``      -- the sm_100a NVLink reduce-scatter + clip + AdamW +
  all-gather kernels of :mod:`oxidizr_b200.parallel.fused_ar` (product path).

Gradients are averaged (scale 1/world) before clipping; every rank applies the
same update, so replicas stay bit-identical.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from ..optim import AdamW, AdamWConfig, FlatParams, LocalAdamW, split_local


class Bucket:
    def __init__(self, lo: int, hi: int, params: List[torch.nn.Parameter]):
        self.lo, self.hi = lo, hi
        self.params = params
        self.pending = len(params)
        self.handle = None


class DDPAdamW(AdamW):
    """AdamW over a FlatParams whose gradient is all-reduced across the group."""

    def __init__(self, flat: FlatParams, cfg: AdamWConfig, backend: str = "nccl", group=None,
                 bucket_bytes: int = 64 << 20, overlap: bool = True, local: Optional[LocalAdamW] = None):
        super().__init__(flat, cfg)
        self.local = local
        self.group = group
        self.world = dist.get_world_size(group)
        self.backend = backend
        self.overlap = overlap and backend == "nccl" and flat.device.type == "cuda"
        self.buckets: List[Bucket] = []
        self.accumulating = False  # set by the trainer on all but the last micro-batch
        if self.overlap:
            self._build_buckets(bucket_bytes)
            self.comm_stream = torch.cuda.Stream(device=flat.device)

    # buckets cover contiguous ranges of the flat buffer, in reverse parameter
    # order (the order backward produces gradients)
    def _build_buckets(self, bucket_bytes: int):
        f = self.flat
        per = max(bucket_bytes // 4, 1)
        order = list(range(len(f.params)))[::-1]
        cur: List[int] = []
        cur_n = 0
        groups = []
        for i in order:
            cur.append(i)
            cur_n += f.params[i].numel()
            if cur_n >= per:
                groups.append(cur)
                cur, cur_n = [], 0
        if cur:
            groups.append(cur)
        for g in groups:
            lo = min(f.offsets[i] for i in g)
            hi = max(f.offsets[i] + f.params[i].numel() for i in g)
            b = Bucket(lo, hi, [f.params[i] for i in g])
            self.buckets.append(b)
            for i in g:
                f.params[i]._oxi_grad_ready = (lambda bb=b: self._on_ready(bb))

    def _local_sq(self, buf: torch.Tensor) -> None:
        """Squared norm of the expert shards, summed over the group (each rank holds different ones)."""
        tmp = torch.zeros_like(buf)
        self.local.sq_into(tmp)
        dist.all_reduce(tmp, group=self.group)
        buf.add_(tmp)

    def _on_ready(self, b: Bucket):
        if self.accumulating:
            return
        b.pending -= 1
        if b.pending == 0:
            self._launch(b)

    def _launch(self, b: Bucket):
        cur = torch.cuda.current_stream(self.flat.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            b.handle = dist.all_reduce(self.flat.grad[b.lo:b.hi], group=self.group, async_op=True)

    def step(self, grad_scale: float = 1.0) -> torch.Tensor:
        f = self.flat
        f.fold_autograd_grads()
        if self.overlap:
            # buckets whose params never reported (e.g. unused) are launched now
            for b in self.buckets:
                if b.handle is None:
                    self._launch(b)
            for b in self.buckets:
                b.handle.wait()
                b.handle = None
                b.pending = len(b.params)
            torch.cuda.current_stream(f.device).wait_stream(self.comm_stream)
        elif self.backend == "cpustaging" and f.device.type == "cuda":
            g = f.grad.cpu()
            dist.all_reduce(g, group=self.group)
            f.grad.copy_(g)
        else:
            dist.all_reduce(f.grad, group=self.group)
        return super().step(grad_scale / self.world)


def make_ddp_optimizer(named_params, cfg: AdamWConfig, device, backend: str, group=None, model=None, **kw):
    """Data-parallel AdamW over a model's parameters for ``backend`` in
    ``cpustaging | nccl | nccl_sharded | fused``.  Expert-parallel shards
    (``_oxi_ep_local``) are updated locally; everything else is averaged over
    the group.  With ``model`` (a LitGPT) the sharded backends overlap their
    parameter all-gather with the model's next forward."""
    named_params = list(named_params)
    if backend in ("fused", "nccl_sharded"):
        from .fused_ar import FusedDDPAdamW, NcclShardedAdamW
        cls = FusedDDPAdamW if backend == "fused" else NcclShardedAdamW
        opt = cls(named_params, cfg, device, group=group, **kw)
        if model is not None:
            opt.attach(model)
        return opt
    rep, loc = split_local(named_params)
    local = LocalAdamW(loc, cfg, device) if loc else None
    return DDPAdamW(FlatParams(rep, device), cfg, backend=backend, group=group, local=local, **kw)
