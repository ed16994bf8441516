"""Sharded data parallelism over NVLink: bucketed bf16 reduce-scatter during
backward, cross-rank clip, sharded AdamW and a bucketed parameter all-gather
that overlaps the next forward (csrc/comm.cu).

This replaces the upstream NCCL synchroniser (distributed/nccl.rs:153-184,
which stages every parameter through host memory and all-reduces on rank 0's
communicator only) with one process per GPU and NVLink traffic issued from our
own kernels:

* buckets of parameters (reverse order of use) are reduced as soon as
  backward has produced all their gradients, on a side stream, so the
  transfers overlap the rest of backward.  Each rank casts its gradient to
  bf16 in its send buffer (clearing the f32 gradient in the same pass) and the
  owner of each shard sums the W copies in f32: by reading the W slices over
  NVLink (``pull``, the default for W < 4), by having the senders store into
  its receive slots (``push``), or through NVSwitch with one
  ``multimem.ld_reduce`` per 16 bytes on a multicast object (``nvls``, the
  default for W >= 4 when the GPUs support multicast);
* each rank keeps f32 master weights and AdamW moments for its 1/W shard of
  every bucket only (optimizer state sharded W ways);
* after backward one tiny kernel exchanges partial norms (global-norm clip);
  then, per bucket on the communication stream, one kernel updates the owned
  shard and sends the new bf16 parameters to every rank (bulk stores into the
  peers' parameter buffers, or one ``multimem.st`` with NVLS).  The next
  forward waits for a bucket only when it first uses it (``attach(model)``),
  so the all-gather of later layers overlaps the forward of earlier ones.

``NcclShardedAdamW`` is the same algorithm (same buckets, cast, sharded AdamW
kernel and overlap) with NCCL's bf16 reduce-scatter and all-gather as the
transport: the like-for-like baseline of the NVLink kernels.

Set-up uses torch.distributed: CUDA-IPC handles are exchanged with
``all_gather_object``; the NVLS multicast object is created and bound by
torch's symmetric-memory allocator.  The data movement is ours.
"""
from __future__ import annotations

import os
from typing import Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..ops._C import ext, status
from ..optim import AdamWConfig, LocalAdamW, split_local

ALIGN = 64
RS_MODES = {"pull": 0, "push": 1, "nvls": 2}


def _roundup(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class SymmetricBuffer:
    """A device buffer of the same size on every rank, mapped by all peers (CUDA IPC)."""

    multicast_ptr = 0

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


class MulticastBuffer:
    """A symmetric buffer with an NVLS multicast address (torch symmetric memory).

    ``ptrs`` are the peers' unicast addresses, ``multicast_ptr`` the address
    whose loads reduce over (``multimem.ld_reduce``) and whose stores go to
    (``multimem.st``) every rank's copy through NVSwitch."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.device = device
        group = group or dist.group.WORLD
        try:
            symm_mem.enable_symm_mem_for_group(group.group_name)
        except Exception:
            pass  # newer releases need no opt-in
        self.local = symm_mem.empty(int(nbytes), dtype=torch.uint8, device=device)
        self.handle = symm_mem.rendezvous(self.local, group)
        self.multicast_ptr = int(self.handle.multicast_ptr)
        if not self.multicast_ptr:
            raise RuntimeError("symmetric memory has no multicast address on this device")
        self.local.zero_()
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.ptr_table = torch.tensor(self.ptrs, dtype=torch.int64, device=device)

    def close(self):
        pass  # unmapped with the tensor, after every rank has stopped using it


def multicast_supported(device: torch.device) -> bool:
    try:
        from torch._C._distributed_c10d import _SymmetricMemory
        return bool(_SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, device.index))
    except Exception:
        return False


class _NoStream:
    """Stand-in for a CUDA stream on the CPU (everything is ordered there)."""

    def wait_stream(self, other):
        pass


class ShardedDDPAdamW:
    """Bucket layout, sharded optimizer state and the overlap logic shared by
    the NVLink transport (:class:`FusedDDPAdamW`) and the NCCL one (and, on the
    CPU, a gloo transport used by the host-logic tests)."""

    collective_state = True  # state_tensors() gathers the shards: every rank calls it

    def __init__(self, named_params: Sequence[Tuple[str, torch.nn.Parameter]], cfg: AdamWConfig, device,
                 group=None, bucket_bytes: int = 32 << 20, rs_ctas: Optional[int] = None,
                 ag_ctas: Optional[int] = None, peer_timeout_s: float = 30.0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        self.rank = dist.get_rank(group)
        self.W = dist.get_world_size(group)
        # CTAs per reduce-scatter (128 threads each) / all-gather (256 threads each) kernel;
        # both are small enough to sit on an SM beside the GEMM CTA they overlap
        self.rs_ctas = int(rs_ctas if rs_ctas is not None else os.environ.get("OXI_RS_CTAS", 256))
        self.ag_ctas = int(ag_ctas if ag_ctas is not None else os.environ.get("OXI_AG_CTAS", 148))
        # a peer that has not posted its flag within this time is reported as failed
        self.wait_ns = int(peer_timeout_s * 1e9)
        named_params, local = split_local(list(named_params))
        # expert-parallel shards: updated locally with the same clip coefficient
        self.local = LocalAdamW(local, cfg, device) if local else None
        self.names = [n for n, _ in named_params]
        self.params = [p for _, p in named_params]
        assert all(p.dtype == torch.bfloat16 for p in self.params), "sharded DDP needs bf16 parameters"
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
        self._bucket_of = {}
        o = 0
        shard_off = 0
        for bi, g in enumerate(groups):
            lo = o
            for i in g:
                self.offsets[i] = o
                o += _roundup(self.params[i].numel(), ALIGN)
                self._bucket_of[id(self.params[i])] = bi
            ln = _roundup(o - lo, W * ALIGN)
            o = lo + ln
            self.buckets.append([lo, ln, shard_off, g])
            shard_off += ln // W
        self.N = o
        self.shard_numel = shard_off
        self._alloc_transport()
        dev = self.device
        self.flat = self.param_local.view(torch.bfloat16)
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
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self._coef = torch.zeros(1, dtype=torch.float32, device=dev)
        self._norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self._done = torch.zeros(1, dtype=torch.int32, device=dev)
        self._push_done = torch.zeros(512, dtype=torch.int32, device=dev)
        self._cuda = dev.type == "cuda"
        self.comm_stream = torch.cuda.Stream(device=dev) if self._cuda else _NoStream()
        self.epoch = 1
        self.step_count = 0
        self.accumulating = False
        self._pending = [len(b[3]) for b in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._sumsq_zeroed = False
        # all-gather in flight: its epoch, and the buckets the compute stream has waited for
        self._ag_epoch: Optional[int] = None
        self._waited = set()
        self.overlap_allgather = False  # set by attach(model)
        for bi, b in enumerate(self.buckets):
            for i in b[3]:
                self.params[i]._oxi_grad_ready = (lambda k=bi: self._on_ready(k))
        self._sync()
        dist.barrier(group=group)

    # ------------------------------------------------------------ streams (no-ops on the CPU)
    def _cur(self):
        return torch.cuda.current_stream(self.device) if self._cuda else _NoStream()

    def _on_comm(self):
        import contextlib
        return torch.cuda.stream(self.comm_stream) if self._cuda else contextlib.nullcontext()

    def _sync(self):
        if self._cuda:
            torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------ transport hooks
    def _alloc_transport(self):
        raise NotImplementedError

    def _rs(self, bi: int):
        """Reduce-scatter bucket bi into rgrad (f32) + sumsq, on the current (comm) stream."""
        raise NotImplementedError

    def _norm_coef(self, max_norm: float):
        """Global clip coefficient (1/W included) into self._coef, norm into self._norm."""
        raise NotImplementedError

    def _ag(self, bi: int, lr, bc1, bc2):
        """AdamW on the owned shard of bucket bi + all-gather, on the current (comm) stream."""
        raise NotImplementedError

    def _wait_bucket(self, bi: int, epoch: int):
        """Make the current stream wait until bucket bi's parameters of `epoch` are in place."""
        raise NotImplementedError

    @property
    def lr(self) -> float:
        return self.cfg.lr

    def _skip_word(self):
        """Expert-parallel over-capacity flag of this step (skips the update), if any."""
        if self.local is None:
            return None
        from .ep import ep_skip_word
        return ep_skip_word(self.device)

    # ------------------------------------------------------------ overlap with the forward
    def attach(self, model) -> None:
        """Let ``model`` (a LitGPT) wait for each bucket's parameters just before
        it first uses them, so the all-gather overlaps the forward."""
        model._param_gate = self.wait_params_of
        self.overlap_allgather = True

    def wait_params_of(self, params: Iterable[torch.Tensor]) -> None:
        if self._ag_epoch is None:
            return
        for p in params:
            bi = self._bucket_of.get(id(p))
            if bi is not None and bi not in self._waited:
                self._waited.add(bi)
                self._wait_bucket(bi, self._ag_epoch)

    def sync_params(self) -> None:
        """Make the current stream wait for every bucket of the last all-gather
        (call before reading parameters outside the forward)."""
        if self._ag_epoch is None:
            return
        for bi in range(len(self.buckets)):
            if bi not in self._waited:
                self._waited.add(bi)
                self._wait_bucket(bi, self._ag_epoch)
        self._ag_epoch = None
        self._waited = set()

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
        # this step's casts overwrite buffers the previous all-gather's peers
        # have finished with only once every bucket of it has landed here
        self.sync_params()
        self._launched[bi] = True
        cur = self._cur()
        self.comm_stream.wait_stream(cur)
        with self._on_comm():
            if not self._sumsq_zeroed:
                self._sumsq.zero_()
                self._sumsq_zeroed = True
            self._rs(bi)

    # ------------------------------------------------------------ step
    def step(self, grad_scale: float = 1.0) -> torch.Tensor:
        for p in self.params:  # gradients that came through plain autograd
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None
        for bi in range(len(self.buckets)):
            self._launch(bi)
        cur = self._cur()
        cur.wait_stream(self.comm_stream)
        c = self.cfg
        self.step_count += 1
        t = self.step_count
        if self.local is not None:
            self.local.sq_into(self._sumsq)  # joins this rank's partial of the global norm
        self._norm_coef(float(c.max_grad_norm or 0.0))
        if grad_scale != 1.0:
            self._coef.mul_(grad_scale)
        bc1, bc2 = 1.0 - c.beta1 ** t, 1.0 - c.beta2 ** t
        self.comm_stream.wait_stream(cur)
        with self._on_comm():
            # the forward uses the last buckets first (reverse parameter order)
            for bi in reversed(range(len(self.buckets))):
                self._ag(bi, c.lr, bc1, bc2)
        if self.local is not None:
            self.local.update(self._coef, t)
            from .ep import ep_step_end
            ep_step_end(self.device)
        self._ag_epoch = self.epoch
        self._waited = set()
        self.epoch += 1
        self._pending = [len(b[3]) for b in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._sumsq_zeroed = False
        if not self.overlap_allgather:
            self.sync_params()
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
        self.sync_params()
        self._cur().wait_stream(self.comm_stream)
        return {"master": self._gather_full(self.master), "exp_avg": self._gather_full(self.m),
                "exp_avg_sq": self._gather_full(self.v)}

    def sync_master_from_params(self) -> None:
        """Re-derive this rank's f32 master shards after the parameters were loaded."""
        self.sync_params()
        with torch.no_grad():
            for lo, ln, so, _ in self.buckets:
                sh = ln // self.W
                self.master[so:so + sh].copy_(self.flat[lo + self.rank * sh: lo + (self.rank + 1) * sh].float())
        if self.local is not None:
            self.local.sync_master_from_params()

    def load_state_tensors(self, d, step: int):
        self.sync_params()
        self._cur().wait_stream(self.comm_stream)
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
        # every peer's writes into this rank's buffers must have landed before they are unmapped
        self.sync_params()
        self._sync()
        dist.barrier(group=self.group)


class FusedDDPAdamW(ShardedDDPAdamW):
    """Drop-in optimizer for data-parallel training over NVLink (sync backend ``fused``).

    ``mode``: ``pull`` / ``push`` (P2P over CUDA-IPC mappings) or ``nvls``
    (multicast object); default ``OXI_AR_MODE`` or ``auto`` = ``nvls`` for
    W >= 4 ranks when the GPUs support multicast, else ``pull``.  With W = 2
    every GPU already sends exactly its peer's half once in ``pull``; NVLS only
    cuts the bytes a GPU sends when W >= 4 (it sends its gradient once instead
    of (W-1)/W of it for each of the two phases)."""

    def __init__(self, *a, mode: Optional[str] = None, **kw):
        self._mode_req = (mode or os.environ.get("OXI_AR_MODE", "auto")).lower()
        super().__init__(*a, **kw)

    def _alloc_transport(self):
        dev, W = self.device, self.W
        mode = self._mode_req
        if mode == "auto":
            mode = "nvls" if W >= 4 and multicast_supported(dev) else "pull"
        if mode == "nvls":
            ok = torch.tensor([1], device=dev)
            try:
                xfer = MulticastBuffer(self.N * 2, dev, self.group)
                param = MulticastBuffer(self.N * 2, dev, self.group)
            except Exception:
                ok.zero_()
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)  # every rank takes the same path
            if int(ok.item()) == 1:
                self.xfer, self.param = xfer, param
            else:
                mode = "pull"
        if mode != "nvls":
            # bf16 gradient exchange buffer: this rank's send buffer (pull) or
            # the receive slots of its shards (push)
            self.xfer = SymmetricBuffer(self.N * 2, dev, self.group)
            self.param = SymmetricBuffer(self.N * 2, dev, self.group)
        self.mode = mode
        self.rs_mode = RS_MODES[mode]
        self.pad = SymmetricBuffer(ext().pad_words() * 4, dev, self.group)
        self.pad_local = self.pad.local.view(torch.int32)
        self.param_local = self.param.local

    def _rs(self, bi):
        lo, ln, so, _ = self.buckets[bi]
        ext().rs_bucket(self.rs_mode, self.grad, True, self.xfer.ptr_table, self.xfer.local,
                        self.xfer.multicast_ptr, self.pad.ptr_table, self.pad_local, self._push_done, self.rank,
                        self.W, bi, self.epoch, lo, ln, self.rgrad[so:so + ln // self.W], self._sumsq, self.rs_ctas,
                        status(self.device), self.wait_ns)

    def _norm_coef(self, max_norm):
        ext().norm_exchange(self.pad.ptr_table, self.pad_local, self.rank, self.W, self.epoch, self._sumsq, max_norm,
                            self._coef, self._norm, status(self.device), self.wait_ns, self._skip_word())

    def _ag(self, bi, lr, bc1, bc2):
        lo, ln, so, _ = self.buckets[bi]
        c = self.cfg
        ext().adamw_ag_bucket(self.rs_mode, lo, ln, so, self.W, self.rank, self.W, self.rgrad, self.master, self.m,
                              self.v, self.param.ptr_table, self.param.multicast_ptr, self.pad.ptr_table, bi,
                              self.epoch, lr, c.beta1, c.beta2, c.eps, c.weight_decay, bc1, bc2, self._coef,
                              self._done, status(self.device), self.ag_ctas)

    def _wait_bucket(self, bi, epoch):
        ext().ag_wait(self.pad_local, self.W, bi, epoch, status(self.device), self.wait_ns)

    def close(self):
        super().close()
        for b in (self.xfer, self.param, self.pad):
            b.close()


class NcclShardedAdamW(ShardedDDPAdamW):
    """The same sharded algorithm over NCCL (sync backend ``nccl_sharded``):
    bf16 ``reduce_scatter_tensor`` per bucket during backward, one f32
    all-reduce of the squared norm, the same sharded AdamW kernel, and an
    in-place bf16 ``all_gather_into_tensor`` per bucket that the next forward
    waits for bucket by bucket.  The like-for-like baseline of FusedDDPAdamW."""

    def _alloc_transport(self):
        dev = self.device
        self.send = torch.zeros(self.N, dtype=torch.bfloat16, device=dev)
        self.recv = torch.zeros(self.shard_numel, dtype=torch.bfloat16, device=dev)
        self.param_local = torch.zeros(self.N * 2, dtype=torch.uint8, device=dev)
        self._own_table = torch.tensor([self.param_local.data_ptr()], dtype=torch.int64, device=dev)
        self._events = {}

    def _rs(self, bi):
        lo, ln, so, _ = self.buckets[bi]
        sh = ln // self.W
        e = ext()
        e.grad_to_bf16(self.grad[lo:lo + ln], self.send[lo:lo + ln], True)
        dist.reduce_scatter_tensor(self.recv[so:so + sh], self.send[lo:lo + ln], group=self.group)
        e.bf16_to_f32_sumsq(self.recv[so:so + sh], self.rgrad[so:so + sh], self._sumsq)

    def _norm_coef(self, max_norm):
        dist.all_reduce(self._sumsq, group=self.group)
        ext().clip_coef(self._sumsq, max_norm, 1.0 / self.W, self._coef, self._norm, None, 0.0, 0.0,
                        self._skip_word())

    def _ag(self, bi, lr, bc1, bc2):
        lo, ln, so, _ = self.buckets[bi]
        sh = ln // self.W
        c = self.cfg
        ext().adamw_ag_bucket(0, lo, ln, so, self.W, self.rank, 1, self.rgrad, self.master, self.m, self.v,
                              self._own_table, 0, None, bi, self.epoch, lr, c.beta1, c.beta2, c.eps,
                              c.weight_decay, bc1, bc2, self._coef, self._done, status(self.device), self.ag_ctas)
        out = self.flat[lo:lo + ln]
        dist.all_gather_into_tensor(out, out[self.rank * sh:(self.rank + 1) * sh], group=self.group)
        ev = torch.cuda.Event()
        ev.record(self.comm_stream)
        self._events[bi] = ev

    def _wait_bucket(self, bi, epoch):
        ev = self._events.pop(bi, None)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)
