"""Host logic of the sharded data-parallel optimizer (parallel/fused_ar.py) on CPU
gloo ranks: bucket layout, the gradient clear folded into the reduce-scatter,
the global-norm clip, sharded AdamW, the per-bucket gating of the next
forward's waits and the collective state gather.  The transport here is a
torch-only stand-in over gloo (the GPU transports are tested against NCCL in
tests/test_ddp.py); everything else is the production class."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

W = 2
SIZES = [1000, 37, 4096, 130, 777, 64]
STEPS = 3
CFG = dict(lr=1e-2, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, max_grad_norm=1.0)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_cls():
    from oxidizr_b200.parallel.fused_ar import ShardedDDPAdamW

    class GlooSharded(ShardedDDPAdamW):
        """Reduce-scatter / all-gather with gloo collectives, AdamW in torch."""

        def _alloc_transport(self):
            self.param_local = torch.zeros(self.N * 2, dtype=torch.uint8)
            self.waits = []

        def _rs(self, bi):
            lo, ln, so, _ = self.buckets[bi]
            sh = ln // self.W
            g = self.grad[lo:lo + ln].to(torch.bfloat16).float()  # the bf16 wire format
            self.grad[lo:lo + ln].zero_()  # cleared as it is read, like the cast kernel
            dist.all_reduce(g, group=self.group)
            mine = g[self.rank * sh:(self.rank + 1) * sh]
            self.rgrad[so:so + sh].copy_(mine)
            self._sumsq += (mine * mine).sum()

        def _norm_coef(self, max_norm):
            t = self._sumsq.clone()
            dist.all_reduce(t, group=self.group)
            nrm = float(t.sqrt()) / self.W
            c = 1.0 / self.W
            if max_norm > 0 and nrm > max_norm:
                c *= max_norm / (nrm + 1e-6)
            self._norm.fill_(nrm)
            self._coef.fill_(c)

        def _ag(self, bi, lr, bc1, bc2):
            lo, ln, so, _ = self.buckets[bi]
            sh = ln // self.W
            c = self.cfg
            g = self.rgrad[so:so + sh] * self._coef
            m, v, p = self.m[so:so + sh], self.v[so:so + sh], self.master[so:so + sh]
            m.mul_(c.beta1).add_(g, alpha=1 - c.beta1)
            v.mul_(c.beta2).addcmul_(g, g, value=1 - c.beta2)
            p.sub_(lr * (m / bc1) / ((v / bc2).sqrt() + c.eps) + lr * c.weight_decay * p)
            parts = [torch.empty(sh, dtype=torch.bfloat16) for _ in range(self.W)]
            dist.all_gather(parts, p.to(torch.bfloat16), group=self.group)
            self.flat[lo:lo + ln].copy_(torch.cat(parts))

        def _wait_bucket(self, bi, epoch):
            self.waits.append((bi, epoch))

    return GlooSharded


def _worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=W)
    try:
        from oxidizr_b200.optim import AdamWConfig
        gen = torch.Generator().manual_seed(0)
        params = [torch.nn.Parameter((torch.randn(n, generator=gen) * 0.1).to(torch.bfloat16)) for n in SIZES]
        ref_master = [p.detach().float().clone() for p in params]
        ref_m = [torch.zeros_like(t) for t in ref_master]
        ref_v = [torch.zeros_like(t) for t in ref_master]
        cfg = AdamWConfig(**CFG)
        opt = _make_cls()([(f"p{i}", p) for i, p in enumerate(params)], cfg, "cpu", bucket_bytes=2048)
        opt.overlap_allgather = True  # what attach(model) sets: the forward waits bucket by bucket
        assert len(opt.buckets) > 2
        assert all(ln % (W * 64) == 0 for _, ln, _, _ in opt.buckets)
        rgen = torch.Generator().manual_seed(100 + rank)
        for step in range(1, STEPS + 1):
            grads = [torch.randn(n, generator=rgen) for n in SIZES]
            # backward: gradients land in main_grad, buckets launch as their parameters report
            for i in reversed(range(len(params))):
                params[i].main_grad.copy_(grads[i])
                params[i]._oxi_grad_ready()
            opt.step()
            # the clear is folded into the reduce-scatter: nothing is left for the next backward
            assert float(opt.grad.abs().sum()) == 0.0
            # the forward waits bucket by bucket: asking for one parameter waits for its bucket only
            n0 = len(opt.waits)
            opt.wait_params_of([params[0]])
            assert opt.waits[n0:] == [(opt._bucket_of[id(params[0])], opt.epoch - 1)]
            opt.wait_params_of([params[0]])  # once per step
            assert len(opt.waits) == n0 + 1
            opt.sync_params()
            assert {b for b, e in opt.waits if e == opt.epoch - 1} == set(range(len(opt.buckets)))
            # reference: mean of every rank's bf16-rounded gradient, global-norm clip, AdamW in f32
            allg = []
            for g in grads:
                parts = [torch.empty_like(g) for _ in range(W)]
                dist.all_gather(parts, g.to(torch.bfloat16).float())
                allg.append(torch.stack(parts).sum(0) / W)
            nrm = float(torch.sqrt(sum((g * g).sum() for g in allg)))
            clip = min(1.0, CFG["max_grad_norm"] / (nrm + 1e-6)) if nrm > CFG["max_grad_norm"] else 1.0
            bc1, bc2 = 1 - CFG["beta1"] ** step, 1 - CFG["beta2"] ** step
            for g, p, m, v in zip(allg, ref_master, ref_m, ref_v):
                g = g * clip
                m.mul_(CFG["beta1"]).add_(g, alpha=1 - CFG["beta1"])
                v.mul_(CFG["beta2"]).addcmul_(g, g, value=1 - CFG["beta2"])
                p.sub_(CFG["lr"] * (m / bc1) / ((v / bc2).sqrt() + CFG["eps"]) + CFG["lr"] * CFG["weight_decay"] * p)
            assert abs(float(opt._norm) - nrm) < 1e-4 * nrm
            for p, r in zip(params, ref_master):
                torch.testing.assert_close(p.detach().float(), r.to(torch.bfloat16).float(), atol=1e-2, rtol=0)
        st = opt.state_tensors()
        for i, r in enumerate(ref_master):
            off = opt.offsets[i]
            torch.testing.assert_close(st["master"][off:off + r.numel()], r, atol=2e-3, rtol=1e-3)
        opt.close()
        if rank == 0:
            torch.save({"ok": True, "buckets": len(opt.buckets)}, out)
    finally:
        dist.destroy_process_group()


def test_sharded_optimizer_host_logic_on_gloo(tmp_path):
    out = str(tmp_path / "res.pt")
    mp.spawn(_worker, args=(_port(), out), nprocs=W, join=True)
    res = torch.load(out)
    assert res["ok"] and res["buckets"] > 2
