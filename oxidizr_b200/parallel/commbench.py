"""Data-parallel gradient-sync microbenchmark (one process per GPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m oxidizr_b200.parallel.commbench --params 1280e6 [--iters 5] [--modes pull,nvls]

Times, on the device with CUDA events (max over ranks), for a flat model of
``--params`` bf16 parameters split into 32 M-element tensors, the whole
synchronisation + optimizer step that follows backward (every bucket's
reduce-scatter, the clip-norm exchange, the sharded AdamW and the parameter
all-gather, waited for by the compute stream):

* ``fused_<mode>``  -- :class:`FusedDDPAdamW` over NVLink with our kernels
                       (``pull``/``push`` P2P, ``nvls`` multicast), at every
                       (reduce-scatter, all-gather) CTA budget of
                       ``--rs-ctas`` x ``--ag-ctas`` (the first pair is the
                       reported one, the fastest is ``best``);
* ``nccl_sharded``  -- the same algorithm with NCCL bf16 reduce-scatter and
                       all-gather as the transport (like-for-like baseline);
* ``nccl_ar``       -- NCCL f32 all-reduce + replicated AdamW (the ``nccl``
                       backend, upstream's algorithm), for reference.

Roofline of a step (per GPU): the slower of its NVLink bytes at the measured
770 GB/s per direction and its HBM bytes at the measured copy bandwidth.
With N parameters and W ranks: HBM = cast (read f32, write bf16, clear f32:
10N) + send buffer read by the owners (2N) + reduced shard (4N/W) + sharded
AdamW (28N/W) + parameters received (2N); NVLink out = 4N(W-1)/W for P2P
(each phase sends (W-1)/W of the bf16 gradient) or 2N + 2N/W for NVLS (the
switch reads the whole send buffer once, the all-gather multicasts the shard
once).  Rank 0 prints one JSON line.

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


def _time(fn, iters, dev, prep=None):
    """Max over ranks of the mean device time of fn() (prep() runs untimed before each call)."""
    if prep:
        prep()
    fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    tot = 0.0
    for _ in range(iters):
        if prep:
            prep()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize(dev)
        tot += e0.elapsed_time(e1)
    ms = torch.tensor([tot / iters], device=dev, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def roofline_ms(N: int, W: int, mode: str, hbm_gbs: float) -> dict:
    hbm = 10 * N + 2 * N + 4 * N / W + 28 * N / W + 2 * N
    nvl = (2 * N + 2 * N / W) if mode == "nvls" else 4 * N * (W - 1) / W
    t_h = hbm / (hbm_gbs * 1e9) * 1e3
    t_n = nvl / (NVLINK_GBS * 1e9) * 1e3
    return {"hbm_ms": round(t_h, 3), "nvlink_ms": round(t_n, 3), "roofline_ms": round(max(t_h, t_n), 3),
            "bound": "hbm" if t_h >= t_n else "nvlink"}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", type=float, default=1280e6)
    ap.add_argument("--chunk", type=float, default=32e6)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--bucket-mb", type=int, default=32)
    ap.add_argument("--modes", default="auto",
                    help="comma list of fused transports to time: pull, push, nvls (auto: pull, plus nvls "
                         "when the GPUs support multicast)")
    ap.add_argument("--rs-ctas", default="256",
                    help="comma list: CTA budgets of the reduce-scatter kernels (first: the training default)")
    ap.add_argument("--ag-ctas", default="148,296",
                    help="comma list: CTA budgets of the AdamW + all-gather kernels (first: the training "
                         "default, which leaves SMs to the forward it overlaps)")
    ap.add_argument("--no-nccl-ar", action="store_true")
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    W, rank = dist.get_world_size(), dist.get_rank()
    from ..optim import AdamW, AdamWConfig, FlatParams
    from ..ops._C import check_status
    from ..utils.kbench import measured_peaks
    from .fused_ar import FusedDDPAdamW, NcclShardedAdamW, multicast_supported
    hbm = measured_peaks()["hbm_gbs"]
    n_total, chunk = int(args.params), int(args.chunk)
    sizes = [chunk] * (n_total // chunk) + ([n_total % chunk] if n_total % chunk else [])
    gen = torch.Generator(device=dev).manual_seed(rank)
    params = [torch.nn.Parameter(torch.randn(n, device=dev, generator=gen).mul_(0.02).bfloat16()) for n in sizes]
    cfg = AdamWConfig(lr=1e-4)
    res = {"params": n_total, "world": W, "hbm_gbs": hbm, "nvlink_gbs": NVLINK_GBS,
           "multicast_supported": multicast_supported(dev)}
    modes = args.modes.split(",") if args.modes != "auto" else (["pull"] + (["nvls"] if res["multicast_supported"]
                                                                           else []))

    def time_sharded(opt):
        def refill():
            opt.grad.normal_(generator=gen)  # the casts clear the gradient as they read it
        return _time(opt.step, args.iters, dev, prep=refill)

    named = [(f"p{i}", p) for i, p in enumerate(params)]
    rs_list = [int(c) for c in args.rs_ctas.split(",")]
    ag_list = [int(c) for c in args.ag_ctas.split(",")]

    def sweep(opt, rf):
        """Time every (rs_ctas, ag_ctas) pair; the first pair is the reported one."""
        rows = []
        for rc in rs_list:
            for ac in ag_list:
                opt.rs_ctas, opt.ag_ctas = rc, ac
                ms = time_sharded(opt)
                rows.append({"rs_ctas": rc, "ag_ctas": ac, "ms": round(ms, 3),
                             "frac_of_roofline": round(rf["roofline_ms"] / ms, 3)})
        best = min(rows, key=lambda r: r["ms"])
        return {**rf, "ms": rows[0]["ms"], "frac_of_roofline": rows[0]["frac_of_roofline"],
                "rs_ctas": rows[0]["rs_ctas"], "ag_ctas": rows[0]["ag_ctas"], "best": best,
                "sweep": rows if len(rows) > 1 else None}

    for mode in modes:
        opt = FusedDDPAdamW(named, cfg, dev, bucket_bytes=args.bucket_mb << 20, mode=mode)
        key = f"fused_{opt.mode}"
        if opt.mode != mode:
            res[f"fused_{mode}_unavailable"] = f"fell back to {opt.mode}"
        res[key] = sweep(opt, roofline_ms(opt.N, W, opt.mode, hbm))
        torch.cuda.synchronize(dev)
        check_status(dev)
        opt.close()
        del opt
        torch.cuda.empty_cache()

    opt = NcclShardedAdamW(named, cfg, dev, bucket_bytes=args.bucket_mb << 20)
    res["nccl_sharded"] = sweep(opt, roofline_ms(opt.N, W, "pull", hbm))
    opt.close()
    del opt
    torch.cuda.empty_cache()
    best = min((v["best"]["ms"], k) for k, v in res.items() if k.startswith("fused_") and isinstance(v, dict))
    res["best_fused"] = best[1]
    res["speedup_vs_nccl_sharded"] = round(res["nccl_sharded"]["best"]["ms"] / best[0], 3)

    if not args.no_nccl_ar:
        flat = FlatParams(named, dev)
        base = AdamW(flat, cfg)
        flat.grad.normal_(generator=gen)

        def nccl_ar():
            dist.all_reduce(flat.grad)
            base.step(1.0 / W)

        res["nccl_ar_ms"] = round(_time(nccl_ar, args.iters, dev), 3)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
