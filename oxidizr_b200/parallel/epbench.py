"""Expert-parallel MoE layer microbenchmark (one process per GPU).

    python -m torch.distributed.run --nproc-per-node W --master-addr 127.0.0.1 \\
        -m oxidizr_b200.parallel.epbench [--tokens 16384] [--iters 5]

One MoE layer of BASELINE config 5 (hidden 2048, 64 experts, top 8, expert width
1024; E/W experts per rank), ``--tokens`` tokens per rank, forward + backward.
Times on the device with CUDA events (mean over ``--iters``, max over ranks):

* ``nvlink``: our path, with the phases of ``parallel/ep.py::EPExperts`` --
  dispatch (count exchange, token rows stored into the owners' receive buffers,
  wait for every peer), gate/up GEMM, down GEMM with the combine fused into its
  epilogue (rows stored straight into the sources' buffers) and the local top-k
  sum; backward: output-gradient push, expert weight gradients, input-gradient
  GEMM with the return scatter fused and the local sum;
* ``nccl``: the same layer with NCCL all-to-all dispatch / combine (the baseline).

Roofline per phase and GPU: the slower of its NVLink bytes at the measured 770
GB/s per direction (the larger of the rows this GPU sends and receives, H bf16
values each) and, for phases with a GEMM, its FLOPs at the measured sustained
bf16 peak.  Rows are counted from this run's routing.  Rank 0 prints one JSON
line.  Upstream layer: model.rs:541-593 (dense, one device).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU

# (phase, first event, last event, kind of work for the roofline)
PHASES = [
    ("dispatch", "fwd_start", "dispatched", "send_fwd"),
    ("gate_up_gemm", "dispatched", "gate_up", "gemm_gu"),
    ("down_gemm_combine", "gate_up", "combined", "gemm_down_ret"),
    ("dy_push", "bwd_start", "dy_pushed", "send_bwd"),
    ("expert_grads", "dy_pushed", "expert_grads", "gemm_wgrad"),
    ("dx_gemm_return", "expert_grads", "dx_combined", "gemm_dx_ret"),
]


def phase_rooflines(rows_out: int, rows_in: int, rows_local: int, H: int, I: int, peak_flops: float,
                    nvlink_gbs: float = NVLINK_GBS) -> dict:
    """Roofline (ms) of each phase kind for one rank: NVLink time of the larger of the rows
    it sends and receives (H bf16 values each); GEMM FLOPs of the rows its experts process
    at ``peak_flops``; the phases with a fused return scatter take the slower of the two."""
    t_link = max(rows_out, rows_in) * 2 * H / (nvlink_gbs * 1e9) * 1e3
    fl = {"gemm_gu": 2 * rows_local * H * 2 * I, "gemm_down_ret": 2 * rows_local * I * H,
          "gemm_wgrad": 2 * rows_local * H * 3 * I, "gemm_dx_ret": 2 * rows_local * 2 * I * H}
    roof = {"send_fwd": t_link, "send_bwd": t_link}
    for kind, f in fl.items():
        roof[kind] = max(f / peak_flops * 1e3, t_link if kind.endswith("_ret") else 0.0)
    return roof


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384, help="tokens per rank (config 5: 4 x 4096)")
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--inter", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--no-nccl", action="store_true")
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    W, rank = dist.get_world_size(), dist.get_rank()
    from ..config import ModelConfig, _build
    from ..models.moe import MoE
    from ..ops._C import check_status
    from ..utils.kbench import measured_peaks
    from .ep import ep_step_end
    peak = measured_peaks()["bf16_tflops_sustained"] * 1e12
    T, H, E, k, I = args.tokens, args.hidden, args.experts, args.topk, args.inter
    cfg = _build(ModelConfig, {
        "name": "epbench", "hidden_size": H, "num_layers": 1, "num_heads": 16, "kv_heads": 4,
        "num_experts": E, "experts_per_tok": k, "intermediate_size": I, "vocab_size": 100, "max_seq_len": 64,
        "rope_theta": 10000.0, "num_shared_experts": 0}, "model")
    moe = MoE(cfg, dev, torch.bfloat16, ep_group=dist.group.WORLD)
    moe.reset_parameters(0.02, torch.Generator(device=dev).manual_seed(0))
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(1, T, H, device=dev, generator=gen).bfloat16().requires_grad_()
    resid = torch.randn(1, T, H, device=dev, generator=gen).bfloat16()
    dy = torch.randn(1, T, H, device=dev, generator=gen).bfloat16()

    def step():
        for p in moe.parameters():
            p.grad = None
        x.grad = None
        y, aux = moe(x, resid)
        torch.autograd.backward([y, aux], [dy, torch.ones_like(aux)])

    # routing of this input: rows this rank sends to / receives from the others
    with torch.no_grad():
        from ..models.moe import route_with_aux
        from ..ops import api
        topi = route_with_aux(api.linear(x.view(T, H), moe.router), k, E, moe.aux_kind)[0]
    owner = topi.reshape(-1).long() // (E // W)
    sent = torch.bincount(owner, minlength=W).to(torch.int64)
    mat = torch.empty(W, W, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(mat, sent)
    rows_out = int(mat[rank].sum() - mat[rank, rank])
    rows_in = int(mat[:, rank].sum() - mat[rank, rank])
    rows_local = int(mat[:, rank].sum())  # rows this rank's experts process
    roof = phase_rooflines(rows_out, rows_in, rows_local, H, I, peak)
    res = {"world": W, "tokens_per_rank": T, "hidden": H, "experts": E, "topk": k, "inter": I,
           "rows_out": rows_out, "rows_in": rows_in, "rows_local": rows_local, "nvlink_gbs": NVLINK_GBS,
           "peak_tflops": peak / 1e12}

    def timed(backend):
        os.environ["OXI_EP_BACKEND"] = backend
        step()
        ep_step_end(dev)
        torch.cuda.synchronize(dev)
        dist.barrier()
        sums, tot = {}, 0.0
        for _ in range(args.iters):
            moe._ep_timer = []
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            torch.cuda.synchronize(dev)
            ep_step_end(dev)
            tot += e0.elapsed_time(e1)
            ev = dict(moe._ep_timer)
            for name, a, b, _ in PHASES:
                if a in ev and b in ev:
                    sums[name] = sums.get(name, 0.0) + ev[a].elapsed_time(ev[b])
            moe._ep_timer = None
        vals = [tot / args.iters] + [sums.get(n, 0.0) / args.iters for n, _, _, _ in PHASES]
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out = {"layer_fwd_bwd_ms": round(float(t[0]), 3)}
        if sums:
            for i, (name, _, _, kind) in enumerate(PHASES):
                ms = float(t[i + 1])
                out[name] = {"ms": round(ms, 3), "roofline_ms": round(roof[kind], 3),
                             "frac_of_roofline": round(roof[kind] / ms, 3) if ms > 0 else None}
        return out

    res["nvlink"] = timed("nvlink")
    check_status(dev)
    if not args.no_nccl:
        res["nccl"] = timed("nccl")
        res["speedup_vs_nccl"] = round(res["nccl"]["layer_fwd_bwd_ms"] / res["nvlink"]["layer_fwd_bwd_ms"], 3)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
