"""Multi-process data-parallel self-test, run as one process per rank.

    python -m oxidizr_b200.parallel.selftest --backend {cpustaging,nccl,fused} --steps 3 --out result.json
    (under torch.distributed.run, or with RANK/WORLD_SIZE/MASTER_* set)

Trains a small GQA model for a few steps on rank-specific data and writes the
per-step losses/grad norms and a parameter checksum of rank 0 to ``--out``.
Every rank checks that its replica equals rank 0's after each step.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def small_config(device_type: str):
    from ..config import LitConfig
    dtype = "bf16" if device_type == "cuda" else "f32"
    return LitConfig.from_dict({
        "model": {"name": "ddp_selftest", "hidden_size": 256, "num_layers": 2, "num_heads": 2, "kv_heads": 1,
                  "intermediate_size": 256, "vocab_size": 1000, "max_seq_len": 128, "rope_theta": 10000.0,
                  "dtype": dtype},
        "trainer": {"learning_rate": 1e-3, "batch_size": 2, "max_steps": 3, "num_epochs": 1,
                    "gradient_accumulation": 1, "checkpoint_dir": "/tmp/oxi_ddp_selftest", "log_interval": 1,
                    "save_interval": 100, "load_balance_alpha": 0.0, "group_size": 4, "beta_kl": 0.04},
    })


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--backend", default="nccl")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--out", default=None)
    ap.add_argument("--timeout", type=int, default=120)
    args = ap.parse_args(argv)
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    use_cuda = args.backend in ("nccl", "nccl_sharded", "fused")
    if use_cuda:
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=args.timeout))
    else:
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=args.timeout))
    from ..models import build_model
    from ..optim import AdamWConfig, FlatParams
    cfg = small_config(dev.type)
    model = build_model(cfg.model, device=dev, seed=0)
    ocfg = AdamWConfig(lr=1e-3)
    from .ddp import make_ddp_optimizer
    kw = {"model": model} if args.backend in ("fused", "nccl_sharded") else {}
    opt = make_ddp_optimizer(model.named_parameters(), ocfg, dev, args.backend, bucket_bytes=1 << 18, **kw)
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    losses, norms = [], []
    for step in range(args.steps):
        ids = torch.randint(0, 1000, (2, 129), generator=g).to(dev)
        loss, _ = model(ids[:, :-1], ids[:, 1:])
        loss.backward()
        gn = opt.step()
        lt = loss.detach().float().reshape(1).clone()
        dist.all_reduce(lt)
        losses.append(float(lt) / world)
        norms.append(float(gn))
        # replicas must stay identical (a sharded optimizer's all-gather lands first)
        if hasattr(opt, "sync_params"):
            opt.sync_params()
        flat = torch.cat([p.detach().float().reshape(-1) for p in model.parameters()])
        ck = torch.stack([flat.sum(), flat.abs().sum()]).to(dev)
        allck = [torch.zeros_like(ck) for _ in range(world)]
        dist.all_gather(allck, ck)
        for c in allck:
            assert torch.allclose(c, allck[0]), f"replica mismatch at step {step}: {allck}"
    if use_cuda:
        from ..ops._C import check_status
        torch.cuda.synchronize()
        check_status(dev)
    if rank == 0 and args.out:
        with open(args.out, "w") as fh:
            json.dump({"backend": args.backend, "world": world, "losses": losses, "grad_norms": norms,
                       "checksum": [float(x) for x in allck[0]]}, fh)
    if hasattr(opt, "close"):
        opt.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
