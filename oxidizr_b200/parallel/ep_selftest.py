"""Expert-parallel MoE self-test, one process per rank.

    python -m torch.distributed.run --nproc-per-node W -m oxidizr_b200.parallel.ep_selftest \
        [--device cuda|cpu] [--backend nvlink|nccl] --out result.json

Every rank builds the same MoE layer twice from one seed: sharded over the
group (E/W experts each) and whole (all E experts).  With rank-specific
tokens it checks, for the sharded layer against the whole one:
* the output and the input gradient on every rank;
* the router gradient (a per-rank quantity before data-parallel averaging);
* the gradient of every local expert == the sum over ranks of the whole
  layer's gradient of that expert.
Rank 0 writes the relative errors to ``--out``.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def _rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--backend", default="nvlink", help="nvlink (sm_100a kernels) | nccl (all-to-all)")
    ap.add_argument("--tokens", type=int, default=300)
    ap.add_argument("--experts", type=int, default=8)
    ap.add_argument("--topk", type=int, default=2)
    ap.add_argument("--hidden", type=int, default=256)
    ap.add_argument("--inter", type=int, default=128)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--two-layers", action="store_true",
                    help="a second MoE layer on the same group with twice the tokens (grows shared buffers)")
    ap.add_argument("--initial-rows", type=int, default=0,
                    help="start the receive buffers this small (the first step runs over capacity, is flagged as "
                         "skipped, and the buffers regrow before the next step)")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    os.environ["OXI_EP_BACKEND"] = args.backend
    if args.initial_rows:
        os.environ["OXI_EP_INITIAL_ROWS"] = str(args.initial_rows)
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    if args.device == "cuda":
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        dtype = torch.bfloat16
    else:
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        dtype = torch.float32
    from ..config import ModelConfig, _build
    from ..models.moe import MoE
    cfg = _build(ModelConfig, {
        "name": "ep", "hidden_size": args.hidden, "num_layers": 1, "num_heads": 4, "kv_heads": 2,
        "num_experts": args.experts, "experts_per_tok": args.topk, "intermediate_size": args.inter,
        "vocab_size": 100, "max_seq_len": 64, "rope_theta": 10000.0, "num_shared_experts": 0,
    }, "model")
    res = {"world": world, "backend": args.backend, "device": args.device}
    errs = []
    sharded = MoE(cfg, dev, dtype, ep_group=dist.group.WORLD)
    whole = MoE(cfg, dev, dtype, ep_group=None)
    gen_dev = dev
    sharded.reset_parameters(0.05, torch.Generator(device=gen_dev).manual_seed(11))
    whole.reset_parameters(0.05, torch.Generator(device=gen_dev).manual_seed(11))
    pairs = [(sharded, whole, args.tokens)]
    if args.two_layers:
        sb = MoE(cfg, dev, dtype, ep_group=dist.group.WORLD)
        wb = MoE(cfg, dev, dtype, ep_group=None)
        sb.reset_parameters(0.05, torch.Generator(device=gen_dev).manual_seed(12))
        wb.reset_parameters(0.05, torch.Generator(device=gen_dev).manual_seed(12))
        pairs.append((sb, wb, 2 * args.tokens))
    El = args.experts // world
    lo = rank * El
    assert torch.equal(sharded.w_gu.detach(), whole.w_gu.detach()[lo:lo + El])
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    for step in range(args.steps):
        for sh, wh, _ in pairs:
            for m in (sh, wh):
                for p in m.parameters():
                    p.grad = None
        outs = []
        loss_s, loss_w = 0.0, 0.0
        # every layer's forward first, then one backward: the layers' exchanges
        # interleave the way they do in a model
        for sh, wh, ntok in pairs:
            x = (torch.randn(1, ntok, args.hidden, generator=g)).to(dev, dtype)
            resid = (torch.randn(1, ntok, args.hidden, generator=g)).to(dev, dtype)
            dy = (torch.randn(1, ntok, args.hidden, generator=g)).to(dev, dtype)
            xs = x.clone().requires_grad_()
            xw = x.clone().requires_grad_()
            ys, aux_s = sh(xs, resid)
            yw, aux_w = wh(xw, resid)
            loss_s = loss_s + (ys.float() * dy.float()).sum() + aux_s
            loss_w = loss_w + (yw.float() * dy.float()).sum() + aux_w
            outs.append((sh, wh, xs, xw, ys, yw))
        loss_s.backward()
        loss_w.backward()
        skipped = 0
        if args.device == "cuda" and args.backend == "nvlink":
            # what an optimizer does after its update: read the over-capacity word, then end the step
            from .ep import ep_skip_word, ep_step_end
            w = ep_skip_word(dev)
            skipped = int(w.item()) if w is not None else 0
            ep_step_end(dev)
        for sh, wh, xs, xw, ys, yw in outs:
            e = {"y": _rel(ys, yw), "dx": _rel(xs.grad, xw.grad), "router": _rel(sh.router.grad, wh.router.grad)}
            for name in ("w_gu", "w_down"):
                full = getattr(wh, name).grad.float().clone()
                dist.all_reduce(full)
                e[name] = _rel(getattr(sh, name).grad, full[lo:lo + El])
            t = torch.tensor([max(e.values())], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e["max_over_ranks"] = float(t)
            e["step"], e["skipped"] = step, skipped
            errs.append(e)
    if args.device == "cuda":
        from ..ops._C import check_status
        torch.cuda.synchronize()
        check_status(dev)
    res["errors"] = errs
    if args.device == "cuda" and args.backend == "nvlink":
        from .ep import EPGroup
        res["regrows"] = sum(g.regrows for g in EPGroup._groups.values())
    if rank == 0 and args.out:
        with open(args.out, "w") as fh:
            json.dump(res, fh)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
