"""Data-parallel gradient-sync microbenchmark (one process per GPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m oxidizr_b200.parallel.commbench --params 1280e6 [--iters 5]

Times, on the device with CUDA events (max over ranks), for a flat model of
``--params`` bf16 parameters split into 32 M-element tensors:

* ``fused``      -- the NVLink path of :class:`FusedDDPAdamW` after backward:
                    bf16 reduce-scatter of every bucket (NVLink push + local sum), norm
                    exchange + clip, sharded AdamW, P2P parameter all-gather;
* ``fused_rs``   -- the reduce-scatter part alone;
* ``nccl_ar``    -- NCCL all-reduce of the f32 gradient + full AdamW (the
                    ``nccl`` backend without overlap);
* ``nccl_rs_ag`` -- NCCL bf16 reduce-scatter + all-gather (transfer only).

The roofline of the fused step is the slower of the NVLink bytes (reduce-
scatter in + all-gather out, (W-1)/W of the bf16 gradient each way, at the
measured 770 GB/s per direction) and the HBM bytes of the sharded AdamW at the
measured copy bandwidth.  Rank 0 prints one JSON line.

Upstream path it replaces: distributed/nccl.rs:153-184 (per-parameter NCCL all-reduce
through host copies) and distributed/optimizer.rs:126-192 (AdamW).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


def _time(fn, iters, dev):
    fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = torch.tensor([e0.elapsed_time(e1) / iters], device=dev, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", type=float, default=1280e6)
    ap.add_argument("--chunk", type=float, default=32e6)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--bucket-mb", type=int, default=32)
    ap.add_argument("--rs-ctas", default="64",
                    help="comma list: CTA budgets of the reduce-scatter to sweep (the first is used for the full "
                         "fused step; 64 is the trainer's default)")
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    W, rank = dist.get_world_size(), dist.get_rank()
    from ..optim import AdamW, AdamWConfig, FlatParams
    from ..ops._C import check_status
    from .fused_ar import FusedDDPAdamW
    n_total, chunk = int(args.params), int(args.chunk)
    sizes = [chunk] * (n_total // chunk) + ([n_total % chunk] if n_total % chunk else [])
    gen = torch.Generator(device=dev).manual_seed(rank)
    params = [torch.nn.Parameter(torch.randn(n, device=dev, generator=gen).mul_(0.02).bfloat16()) for n in sizes]
    cfg = AdamWConfig(lr=1e-4)
    res = {"params": n_total, "world": W}

    sweep = [int(c) for c in str(args.rs_ctas).split(",")]
    opt = FusedDDPAdamW([(f"p{i}", p) for i, p in enumerate(params)], cfg, dev, bucket_bytes=args.bucket_mb << 20,
                        rs_ctas=sweep[0])
    opt.grad.normal_(generator=gen)

    def fused_step():
        opt.step()
        opt.grad.normal_(generator=gen)  # step() zeroes the gradient

    def grad_refill():
        opt.grad.normal_(generator=gen)

    ms_refill = _time(grad_refill, args.iters, dev)
    res["fused_ms"] = round(_time(fused_step, args.iters, dev) - ms_refill, 3)

    def fused_rs():
        opt._launched = [False] * len(opt.buckets)
        opt._sumsq_zeroed = False
        for bi in range(len(opt.buckets)):
            opt._launch(bi)
        torch.cuda.current_stream(dev).wait_stream(opt.comm_stream)
        opt.epoch += 1

    # the reduce-scatter alone: bump the epoch on every rank in lockstep
    res["fused_rs_ms"] = round(_time(fused_rs, args.iters, dev), 3)
    for c in sweep[1:]:
        opt.rs_ctas = c
        res[f"fused_rs_ms_ctas{c}"] = round(_time(fused_rs, args.iters, dev), 3)
    opt.rs_ctas = sweep[0]
    torch.cuda.synchronize(dev)
    check_status(dev)
    opt.close()
    del opt
    torch.cuda.empty_cache()

    flat = FlatParams([(f"p{i}", p) for i, p in enumerate(params)], dev)
    base = AdamW(flat, cfg)
    flat.grad.normal_(generator=gen)

    def nccl_ar():
        dist.all_reduce(flat.grad)
        base.step(1.0 / W)

    res["nccl_ar_ms"] = round(_time(nccl_ar, args.iters, dev), 3)
    g16 = torch.randn(n_total // (W * 8) * W * 8, device=dev, generator=gen).bfloat16()
    shard = torch.empty(g16.numel() // W, device=dev, dtype=torch.bfloat16)

    def nccl_rs_ag():
        dist.reduce_scatter_tensor(shard, g16)
        dist.all_gather_into_tensor(g16, shard)

    res["nccl_rs_ag_ms"] = round(_time(nccl_rs_ag, args.iters, dev), 3)
    # rooflines
    from ..utils.kbench import measured_peaks
    hbm = measured_peaks()["hbm_gbs"]
    nvl_bytes = (W - 1) / W * n_total * 2  # per direction per GPU, each phase
    rs_ms = nvl_bytes / (NVLINK_GBS * 1e9) * 1e3
    adam_bytes = n_total / W * (4 * 7) + n_total * 2 * 2  # shard f32 state r/w + bf16 grads/params
    adam_ms = adam_bytes / (hbm * 1e9) * 1e3
    res["roofline_rs_ms"] = round(rs_ms, 3)
    res["roofline_fused_ms"] = round(max(2 * rs_ms, adam_ms), 3)
    res["fused_rs_frac_of_roofline"] = round(rs_ms / res["fused_rs_ms"], 3)
    res["fused_frac_of_roofline"] = round(res["roofline_fused_ms"] / res["fused_ms"], 3)
    res["fused_rs_gbs_per_dir"] = round(nvl_bytes / (res["fused_rs_ms"] * 1e-3) / 1e9, 1)
    res["nccl_rs_ag_gbs_per_dir"] = round(2 * nvl_bytes / (res["nccl_rs_ag_ms"] * 1e-3) / 1e9, 1)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
