"""Where a training step of a ``bench.py`` model spends its device time
(torch.profiler, CUDA activity only).

    python -m oxidizr_b200.utils.stepprof --model mamba3 [--steps 2] [--rows 40] [--cuda-graph]
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m oxidizr_b200.utils.stepprof --model llama --backend fused --timeline

Prints the total device time per step and the top kernels with their share and
launch count per step.  ``--timeline`` adds, per CUDA stream, its busy time
within the profiled steps, and for the compute stream (the one with the most
kernel time) the idle gaps between its kernels, largest first, with the
kernels on either side and what the other streams ran meanwhile: the exposed
part of the data-parallel communication.  Runs three untimed warm-up steps
first.  One GPU, or one process per GPU (rank 0 prints) with ``--backend``.
"""
from __future__ import annotations

import argparse
import collections
import datetime
import json
import os
import sys
import tempfile


def _timeline(trace_path: str, steps: int, rows: int) -> None:
    ev = json.load(open(trace_path))
    ev = ev["traceEvents"] if isinstance(ev, dict) else ev
    kern = [e for e in ev if e.get("ph") == "X" and e.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset")]
    if not kern:
        print("timeline: no device events")
        return
    by_stream = collections.defaultdict(list)
    for e in kern:
        by_stream[e.get("args", {}).get("stream", e.get("tid"))].append(e)
    t0 = min(e["ts"] for e in kern)
    t1 = max(e["ts"] + e["dur"] for e in kern)
    span = (t1 - t0) / steps
    busy = {s: sum(e["dur"] for e in es) / steps for s, es in by_stream.items()}
    main = max(busy, key=busy.get)
    print(f"timeline: {span / 1000:.2f} ms per step from first to last kernel; per stream busy time:")
    for s, b in sorted(busy.items(), key=lambda kv: -kv[1]):
        print(f"  stream {s}: {b / 1000:8.3f} ms busy ({len(by_stream[s]) // steps} kernels / step)"
              + ("  <- compute" if s == main else ""))
    es = sorted(by_stream[main], key=lambda e: e["ts"])
    gaps = []
    for a, b in zip(es, es[1:]):
        g = b["ts"] - (a["ts"] + a["dur"])
        if g > 5:
            gaps.append((g, a, b))
    tot_gap = sum(g for g, _, _ in gaps) / steps
    print(f"compute stream idle: {tot_gap / 1000:.3f} ms per step in {len(gaps) // steps} gaps > 5 us; largest:")
    others = [e for s, v in by_stream.items() if s != main for e in v]
    for g, a, b in sorted(gaps, key=lambda x: -x[0])[:rows]:
        lo, hi = a["ts"] + a["dur"], b["ts"]
        during = collections.Counter(e["name"][:48] for e in others if e["ts"] < hi and e["ts"] + e["dur"] > lo)
        print(f"  {g / 1000:7.3f} ms  after {a['name'][:56]!r}  before {b['name'][:56]!r}  "
              f"others: {dict(during.most_common(3))}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--rows", type=int, default=40)
    ap.add_argument("--cuda-graph", action="store_true")
    ap.add_argument("--backend", default=None,
                    help="data-parallel backend under torch.distributed.run (fused, nccl_sharded, nccl)")
    ap.add_argument("--timeline", action="store_true", help="per-stream busy time and compute-stream gaps")
    ap.add_argument("--trace-out", default=None, help="also keep the chrome trace (rank 0) at this path")
    args = ap.parse_args(argv)
    import torch
    import torch.distributed as dist
    from torch.profiler import ProfilerActivity, profile

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench
    from ..models import build_model
    from ..optim import AdamW, AdamWConfig, FlatParams
    from ..trainer import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    cfg = bench.bench_config(args.model)
    m, t = cfg.model, cfg.trainer
    ep = world if (world > 1 and m.num_experts) else 1
    model = build_model(m, device=dev, seed=0, ep_group=dist.group.WORLD if ep > 1 else None)
    ocfg = AdamWConfig(lr=t.learning_rate)
    if world > 1:
        from ..parallel.ddp import make_ddp_optimizer
        opt = make_ddp_optimizer(model.named_parameters(), ocfg, dev, args.backend or "fused", model=model)
    else:
        opt = AdamW(FlatParams(list(model.named_parameters()), dev), ocfg)
    B, S, V = t.batch_size, m.max_seq_len, m.vocab_size
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    blk = torch.randint(0, V, (B, S + 1), device=dev, generator=g)

    class Batches:
        batch_size, seq_len = B, S

        def dataset_size(self):
            return 10 ** 12

        def next_batch(self):
            return blk[:, :-1], blk[:, 1:]

    tr = Trainer(cfg, model, opt, Batches(), device=dev, headless=True, out=lambda s: None,
                 cuda_graph=args.cuda_graph, rank=rank, world_size=world)
    for _ in range(3):
        tr.training_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            tr.training_step()
        torch.cuda.synchronize()
    if rank == 0:
        rows = [e for e in prof.key_averages() if e.device_type.name == "CUDA"]
        total = sum(e.device_time_total for e in rows) or 1.0
        rows.sort(key=lambda e: -e.device_time_total)
        print(f"model {args.model} on {world} GPU(s) ({args.backend or 'single'}): "
              f"{total / args.steps / 1000:.2f} ms device time per step "
              f"({'CUDA graph' if tr.cuda_graph else 'eager'})")
        for e in rows[:args.rows]:
            print(f"{e.device_time_total / args.steps / 1000:9.3f} ms {100 * e.device_time_total / total:5.1f}% "
                  f"n={e.count // args.steps:5d}  {e.key[:120]}")
        if args.timeline or args.trace_out:
            path = args.trace_out or os.path.join(tempfile.mkdtemp(prefix="oxi_prof_"), "trace.json")
            prof.export_chrome_trace(path)
            if args.timeline:
                _timeline(path, args.steps, args.rows)
    if hasattr(opt, "close"):
        opt.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
