"""Expert parallelism for the MoE layer.

Upstream has no expert parallelism (every expert runs on every token in one
process, model.rs:561-565).  Here each of ``W`` ranks of an expert-parallel
group holds E/W experts, and every token row travels to the rank that owns
each of its top-k experts.  Two implementations of the same exchange:

* ``nvlink`` (default on CUDA, :class:`EPExperts`): the sm_100a kernels of
  ``csrc/ep.cu``.  The per-expert counts are all-gathered through NVLink signal
  pads; the dispatch kernel writes token rows straight into the owners'
  receive buffers (P2P stores, CUDA-IPC symmetric memory); the owners run the
  grouped tcgen05 expert GEMMs on their receive buffer; the combine kernel
  reads the k expert rows of each token back over NVLink and adds them,
  weighted, to the residual.  Backward pushes output gradients to the owners,
  which compute the routing-weight gradients and the expert backward GEMMs;
  the sources gather the input gradients.  Every wait is bounded.  No host
  synchronisation: receive buffers have a fixed capacity (2x the balanced
  load); the count kernel checks it on the device, and a layer whose routing
  would overflow any owner is skipped on every rank (all see the same counts)
  and flags the step, whose update the optimizer then skips.  The host reads
  that flag once per step, lazily, and regrows the buffers collectively before
  the next step's first MoE layer.
* ``nccl`` (baseline, and the CPU/gloo path, :func:`ep_moe`): NCCL/gloo
  all-to-all of the permuted rows (``torch.distributed.nn`` keeps it
  differentiable), split sizes read on the host.

Expert weight gradients are sums over the tokens of every rank; the
data-parallel optimizers scale them by 1/W like the averaged dense gradients
and keep them out of the all-reduce (``param._oxi_ep_local``).
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

# flag kinds of csrc/kernels_ep.h
K_DISPATCHED, K_YREADY, K_DYPUSHED, K_DXREADY = 1, 2, 3, 4


def _a2a(x: torch.Tensor, out_splits, in_splits, group):
    from torch.distributed.nn.functional import all_to_all_single
    out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
    return all_to_all_single(out, x, out_splits, in_splits, group=group)


def ep_moe(moe, x: torch.Tensor, topi: torch.Tensor, topw: torch.Tensor) -> torch.Tensor:
    """Routed-expert output (without residual / shared experts) for tokens x [T, H], over all-to-all."""
    group = moe.ep_group
    W, El = moe.ep_size, moe.E_local
    k = topi.shape[1]
    flat = topi.reshape(-1)
    order = torch.argsort(flat, stable=True)
    tok = order // k
    dest = flat.index_select(0, order) // El
    send_counts = torch.bincount(dest, minlength=W)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    s_split = send_counts.tolist()
    r_split = recv_counts.tolist()
    x_send = x.index_select(0, tok)
    local_ids = (flat.index_select(0, order) % El).to(torch.int64)
    ids_recv = torch.empty(sum(r_split), dtype=torch.int64, device=x.device)
    dist.all_to_all_single(ids_recv, local_ids, r_split, s_split, group=group)
    x_recv = _a2a(x_send, r_split, s_split, group)
    R = x_recv.shape[0]
    from ..models.moe import _grouped_ok
    if R > 0 and _grouped_ok(x_recv, moe.w_gu):
        from ..ops.moe_kernels import GroupedExperts
        ones = torch.ones(R, 1, dtype=torch.float32, device=x.device)
        y_recv = GroupedExperts.apply(x_recv, ids_recv[:, None], ones, moe.w_gu, moe.w_down, None)
    else:
        from ..ops import api
        # every expert joins the graph (with zero rows if unused) so all ranks see the same backward
        y_recv = torch.zeros_like(x_recv)
        for e in range(El):
            sel = (ids_recv == e).nonzero().squeeze(1)
            y_recv = y_recv.index_copy(0, sel, api.swiglu_mlp(x_recv.index_select(0, sel), moe.w_gu[e],
                                                              moe.w_down[e]))
    y_send = _a2a(y_recv, s_split, r_split, group)
    w_sorted = topw.reshape(-1).index_select(0, order).to(y_send.dtype)
    return torch.zeros_like(x).index_add(0, tok, y_send * w_sorted[:, None])


# ---------------------------------------------------------------------- NVLink
class EPGroup:
    """Signal pad and exchange counter shared by the MoE layers of one group."""

    _groups = {}

    @classmethod
    def get(cls, group, device) -> "EPGroup":
        key = (id(group), torch.device(device).index)
        if key not in cls._groups:
            cls._groups[key] = EPGroup(group, device)
        return cls._groups[key]

    def __init__(self, group, device, timeout_s: Optional[float] = None):
        from ..ops._C import ext
        from .fused_ar import SymmetricBuffer
        self.group = group
        self.device = torch.device(device)
        self.W = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.pad = SymmetricBuffer(ext().ep_pad_words() * 4, self.device, group)
        self.pad_local = self.pad.local.view(torch.int32)
        self.done = torch.zeros(4, dtype=torch.int32, device=self.device)  # last-CTA counters
        self.cursor = torch.zeros(256, dtype=torch.int32, device=self.device)
        t = timeout_s if timeout_s is not None else float(os.environ.get("OXI_PEER_TIMEOUT_S", 30.0))
        self.wait_ns = int(t * 1e9)
        self.seq = 0
        # gradient rows pushed to expert owners live only inside one layer's
        # backward, so every layer of the group shares one buffer
        self.dyrecv = None
        self.dyrecv_bytes = 0
        # [over-capacity flag of this step, most receive rows any layer needed]:
        # written by the count kernels, read by the optimizer's clip kernel (skip)
        # and, one step later, by the host (regrow)
        self.overflow = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._ovf_host = torch.zeros(2, dtype=torch.int32).pin_memory()
        self._ovf_event = None
        self.layers = []
        self.regrows = 0

    def shared_dyrecv(self, nbytes: int):
        """The group's gradient receive buffer, grown collectively to at least nbytes."""
        if nbytes > self.dyrecv_bytes:
            from .fused_ar import SymmetricBuffer
            torch.cuda.synchronize(self.device)
            if self.dyrecv is not None:
                self.dyrecv.close()
                dist.barrier(group=self.group)
            self.dyrecv = SymmetricBuffer(nbytes, self.device, self.group)
            self.dyrecv_bytes = nbytes
        return self.dyrecv

    def next_seq(self) -> int:
        self.seq += 1
        return self.seq

    def step_end(self) -> None:
        """After the optimizer has read this step's flag: copy it to the host
        (asynchronously) and clear it for the next step."""
        self._ovf_host.copy_(self.overflow, non_blocking=True)
        self._ovf_event = torch.cuda.Event()
        self._ovf_event.record()
        self.overflow.zero_()

    def check_regrow(self) -> None:
        """Before a step's first MoE layer: if the previous step ran over a receive
        capacity, grow every layer's buffers (collective; every rank saw the same
        flag).  Waits for the previous step's flag copy only."""
        ev, self._ovf_event = self._ovf_event, None
        if ev is None:
            return
        ev.synchronize()
        flag, need = int(self._ovf_host[0]), int(self._ovf_host[1])
        if flag:
            self.regrows += 1
            for buf in self.layers:
                buf.ensure(max(need, buf.cap + 1))


def _groups_on(device):
    idx = torch.device(device).index
    return [g for (gid, di), g in EPGroup._groups.items() if di == idx]


def ep_skip_word(device) -> Optional[torch.Tensor]:
    """The device word that makes an optimizer skip this step's update (an expert-
    parallel layer ran over its receive capacity), or None without expert parallelism."""
    gs = _groups_on(device)
    return gs[0].overflow[0:1] if gs else None


def ep_step_end(device) -> None:
    """Called by the optimizers after their update launches."""
    for g in _groups_on(device):
        g.step_end()


class EPLayerBuffers:
    """The symmetric receive/output buffers of one MoE layer (grown collectively)."""

    # receive-buffer growth is a collective (IPC handle exchange plus a device
    # sync), so it must be rare: the first size and every growth leave 2x room for
    # routing imbalance (routers drift while training; at 1.5x a 4-GPU run still
    # regrew five of sixteen layers in eight steps)
    HEADROOM = 2.0
    reallocs = 0  # class-wide count, reported by the benchmark

    def __init__(self, grp: EPGroup, H: int):
        self.grp, self.H = grp, H
        self.cap = 0
        self.bufs = None
        self.pairs = 0
        self.yret = None  # [T*k, H]: this rank's expert output rows, then their input gradients
        grp.layers.append(self)

    def ensure_pairs(self, pairs: int):
        """yret holds one row per (token, slot) of this rank; its size only changes with
        the batch shape, identically on every rank (collective)."""
        if pairs != self.pairs:
            from .fused_ar import SymmetricBuffer
            g = self.grp
            torch.cuda.synchronize(g.device)
            if self.yret is not None:
                self.yret.close()
                dist.barrier(group=g.group)
            self.yret = SymmetricBuffer(pairs * self.H * 2, g.device, g.group)
            self.pairs = pairs

    def ensure(self, rows: int, balanced_rows: int = 0, exact: bool = False):
        if rows <= self.cap and not (balanced_rows and self.cap == 0):
            return
        from .fused_ar import SymmetricBuffer
        g = self.grp
        if exact:
            cap = max(256, (rows + 255) // 256 * 256)
        else:
            want = max(rows * self.HEADROOM, balanced_rows * self.HEADROOM, self.cap * self.HEADROOM)
            cap = max(256, (int(want) + 1023) // 1024 * 1024)
        EPLayerBuffers.reallocs += 1
        torch.cuda.synchronize(g.device)
        if self.bufs is not None:
            for b in self.bufs.values():
                b.close()
            dist.barrier(group=g.group)
        H = self.H
        self.bufs = {
            "xrecv": SymmetricBuffer(cap * H * 2, g.device, g.group),
            "metaw": SymmetricBuffer(cap * 4, g.device, g.group),
            "srcidx": SymmetricBuffer(cap * 4, g.device, g.group),
        }
        g.shared_dyrecv(cap * H * 2)  # looked up at use time: a later growth replaces it
        self.cap = cap

    def _buf(self, name: str):
        return self.grp.dyrecv if name == "dyrecv" else self.bufs[name]

    def local(self, name: str, dtype, cols: int = 0) -> torch.Tensor:
        t = self._buf(name).local.view(dtype)
        if cols:
            return t[: self.cap * cols].view(self.cap, cols)
        return t[: self.cap] if dtype in (torch.float32, torch.int32) else t

    def table(self, name: str) -> torch.Tensor:
        return self._buf(name).ptr_table


def _mark(moe, name: str) -> None:
    """Record a CUDA event named ``name`` on the current stream when the layer carries a
    phase timer (``moe._ep_timer``, a list set by the expert-parallel microbenchmark)."""
    tm = getattr(moe, "_ep_timer", None)
    if tm is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        tm.append((name, ev))


class EPExperts(torch.autograd.Function):
    """resid + sum_j topw[t, j] * SwiGLU_{topi[t, j]}(x_t), experts spread over the group (NVLink).

    The combine is fused into the owners' down-projection GEMM: its epilogue stores
    every output row straight into the source rank's ``yret`` (P2P) as the tiles
    finish, and its last CTA posts the flag; the source then sums its k rows per
    token locally.  The backward does the same with the input-gradient rows."""

    @staticmethod
    def forward(ctx, x, topi, topw, counts, w_gu, w_down, resid, moe):
        from ..ops._C import ext, status
        e = ext()
        g: EPGroup = moe._ep
        buf: EPLayerBuffers = moe._ep_buf
        T, H = x.shape
        El, I2, _ = w_gu.shape
        I = I2 // 2
        k = topi.shape[1]
        W, rank = g.W, g.rank
        st = status(x.device)
        xc = x if x.stride(1) == 1 else x.contiguous()
        topi = topi.contiguous()
        tw = topw.float().contiguous()
        seq = g.next_seq()
        if buf.cap == 0:  # first use: 2x the balanced load plus every segment's alignment
            forced = int(os.environ.get("OXI_EP_INITIAL_ROWS", "0"))  # tests: start over capacity
            buf.ensure(forced, exact=True) if forced else buf.ensure(0, balanced_rows=T * k + El * 256)
        buf.ensure_pairs(T * k)
        _mark(moe, "fwd_start")
        # the counts kernel checks every owner's rows against the capacity on the
        # device (no host read); over capacity, the layer is skipped on every rank
        all_counts, seg, rc = e.ep_counts(counts.int().contiguous(), g.pad.ptr_table, g.pad_local, rank, W, seq,
                                          buf.cap, g.overflow, st, g.wait_ns)
        cap = buf.cap
        xr = buf.local("xrecv", torch.bfloat16, H)
        e.moe_zero_pad(seg, rc, xr)
        e.ep_mark_pad(seg, rc, buf.local("srcidx", torch.int32))
        pos = e.ep_dispatch(xc, topi, tw, all_counts, rank, W, g.cursor, buf.table("xrecv"), buf.table("metaw"),
                            buf.table("srcidx"), g.done[0:1], g.pad.ptr_table, seq, seg, st)
        e.ep_wait(g.pad_local, K_DISPATCHED, W, seq, st, g.wait_ns)
        _mark(moe, "dispatched")
        h = torch.empty(cap, I, dtype=x.dtype, device=x.device)
        gu = torch.empty(cap, I2, dtype=x.dtype, device=x.device)
        e.gemm_grouped(1, 2, xr, False, w_gu.view(El * I2, H), False, El, seg, I2, h, gu, None, st)
        _mark(moe, "gate_up")
        e.ep_expert_gemm_scatter(h, w_down.view(El * H, I), False, El, seg, H, buf.local("srcidx", torch.int32),
                                 buf.yret.ptr_table, T * k, g.done[2:3], g.pad.ptr_table, K_YREADY, rank, W, seq, st)
        yret = buf.yret.local.view(torch.bfloat16).view(T * k, H)
        y = e.ep_sum_pairs(yret, tw, T, k, resid.contiguous() if resid is not None else None, g.pad_local, K_YREADY,
                           W, seq, st, g.wait_ns)
        _mark(moe, "combined")
        ctx.save_for_backward(topi, tw, pos, h, gu, seg, rc)
        ctx.moe, ctx.w_gu, ctx.w_down, ctx.has_resid = moe, w_gu, w_down, resid is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops._C import ext, status
        from ..ops.moe_kernels import _wgrad_grouped, swiglu_bwd_grouped
        e = ext()
        topi, tw, pos, h, gu, seg, rc = ctx.saved_tensors
        moe = ctx.moe
        g: EPGroup = moe._ep
        buf: EPLayerBuffers = moe._ep_buf
        w_gu, w_down = ctx.w_gu, ctx.w_down
        El, I2, H = w_gu.shape
        I = I2 // 2
        T, k = topi.shape
        W, rank = g.W, g.rank
        st = status(dy.device)
        dy = dy.contiguous()
        seq = g.next_seq()
        _mark(moe, "bwd_start")
        xr = buf.local("xrecv", torch.bfloat16, H)
        dyr = buf.local("dyrecv", torch.bfloat16, H)
        yret = buf.yret.local.view(torch.bfloat16).view(T * k, H)
        # dy rows to the owners; d topw from this rank's copy of the expert outputs
        dtw = e.ep_push_dy(dy, topi, pos, El, buf.table("dyrecv"), yret, g.done[1:2], g.pad.ptr_table, rank, W, seq,
                           seg, st)
        e.ep_wait(g.pad_local, K_DYPUSHED, W, seq, st, g.wait_ns)
        _mark(moe, "dy_pushed")
        e.ep_scale_rows(dyr, buf.local("metaw", torch.float32), seg, rc, El)
        g_down = _wgrad_grouped(w_down, dyr, h, seg, El)
        dgu = torch.empty_like(gu)
        swiglu_bwd_grouped(dyr, w_down, gu, dgu, El, seg, st)
        g_gu = _wgrad_grouped(w_gu, dgu, xr, seg, El)
        _mark(moe, "expert_grads")
        # input-gradient rows straight into the sources' yret (their forward rows were
        # consumed by their push_dy, which finished before DYPUSHED)
        e.ep_expert_gemm_scatter(dgu, w_gu.view(El * I2, H), True, El, seg, I2, buf.local("srcidx", torch.int32),
                                 buf.yret.ptr_table, T * k, g.done[3:4], g.pad.ptr_table, K_DXREADY, rank, W, seq, st)
        dx = e.ep_sum_pairs(yret, None, T, k, None, g.pad_local, K_DXREADY, W, seq, st, g.wait_ns)
        _mark(moe, "dx_combined")
        return dx, None, dtw, None, g_gu, g_down, (dy if ctx.has_resid else None), None


def nvlink_ok(moe, x) -> bool:
    if not x.is_cuda or os.environ.get("OXI_EP_BACKEND", "nvlink") != "nvlink":
        return False
    from ..ops._C import ext
    from ..ops.moe_kernels import grouped_ok
    return hasattr(ext(), "ep_dispatch") and grouped_ok(x, moe.w_gu) and moe.k <= 16 and moe.E <= 256


def ep_moe_nvlink(moe, x, topi, topw, counts, resid):
    if getattr(moe, "_ep", None) is None:
        moe._ep = EPGroup.get(moe.ep_group, x.device)
        moe._ep_buf = EPLayerBuffers(moe._ep, x.shape[1])
    moe._ep.check_regrow()
    return EPExperts.apply(x, topi, topw, counts, moe.w_gu, moe.w_down, resid, moe)
