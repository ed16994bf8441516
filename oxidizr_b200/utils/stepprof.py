"""Per-kernel device time of one training step of a ``bench.py`` model (torch.profiler,
CUDA activity only), for finding where a step's time goes.

    python -m oxidizr_b200.utils.stepprof --model mamba3 [--steps 2] [--rows 40] [--cuda-graph]

Prints the total device time per step and the top kernels with their share and launch
count per step.  Runs three untimed warm-up steps first.  One GPU.
"""
from __future__ import annotations

import argparse
import os
import sys


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--rows", type=int, default=40)
    ap.add_argument("--cuda-graph", action="store_true")
    args = ap.parse_args(argv)
    import torch
    from torch.profiler import ProfilerActivity, profile

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench
    from ..models import build_model
    from ..optim import AdamW, AdamWConfig, FlatParams
    from ..trainer import Trainer

    cfg = bench.bench_config(args.model)
    m, t = cfg.model, cfg.trainer
    dev = torch.device("cuda", 0)
    model = build_model(m, device=dev, seed=0)
    opt = AdamW(FlatParams(list(model.named_parameters()), dev), AdamWConfig(lr=t.learning_rate))
    B, S, V = t.batch_size, m.max_seq_len, m.vocab_size
    blk = torch.randint(0, V, (B, S + 1), device=dev)

    class Batches:
        batch_size, seq_len = B, S

        def dataset_size(self):
            return 10 ** 12

        def next_batch(self):
            return blk[:, :-1], blk[:, 1:]

    tr = Trainer(cfg, model, opt, Batches(), device=dev, headless=True, out=lambda s: None,
                 cuda_graph=args.cuda_graph)
    for _ in range(3):
        tr.training_step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            tr.training_step()
        torch.cuda.synchronize()
    rows = [e for e in prof.key_averages() if e.device_type.name == "CUDA"]
    total = sum(e.device_time_total for e in rows) or 1.0
    rows.sort(key=lambda e: -e.device_time_total)
    print(f"model {args.model}: {total / args.steps / 1000:.2f} ms device time per step "
          f"({'CUDA graph' if tr.cuda_graph else 'eager'})")
    for e in rows[:args.rows]:
        print(f"{e.device_time_total / args.steps / 1000:9.3f} ms {100 * e.device_time_total / total:5.1f}% "
              f"n={e.count // args.steps:5d}  {e.key[:120]}")


if __name__ == "__main__":
    main()
