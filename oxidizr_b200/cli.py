"""``oxidizr`` command line: ``train``, ``pack``, ``push`` and the legacy
``oxidizr -f <config>`` form (main.rs:20-151, commands/train.rs:17-75,
commands/pack.rs:15-35, commands/push.rs:14-34).

Flags and defaults follow upstream, including its ``--dtype`` default of
``f32`` overriding the YAML ``dtype`` (commands/train.rs:71-74, 324-333).
``--sync-backend`` additionally accepts ``fused`` (the NVLink kernel path).
With more than one id in ``--gpus`` the command re-launches itself as one
process per GPU (torch.distributed over NCCL, rendezvous on 127.0.0.1); each
process trains a replica on its own shard of the token file.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import shutil
import socket
import subprocess
import sys
import time
from typing import List, Optional

from .config import ConfigError, LitConfig, parse_dtype, parse_sync_backend


# ====================================================================== args
def _add_train_args(p: argparse.ArgumentParser, legacy: bool = False):
    p.add_argument("-f", "--config", dest="config_file", default=None if legacy else "models/nano.yaml")
    p.add_argument("-d", "--data", dest="data_file", default=None)
    p.add_argument("--target-device", dest="target_device", default=None)
    p.add_argument("--seq-len", dest="seq_length", type=int, default=None)
    p.add_argument("--batch-size", dest="batch_size", type=int, default=None)
    p.add_argument("--grad-accum", dest="gradient_accumulation", type=int, default=None)
    p.add_argument("--headless", action="store_true")
    p.add_argument("--max-steps", dest="max_steps", type=int, default=None)
    p.add_argument("--resume", default=None)
    p.add_argument("--gpus", default=None)
    p.add_argument("--sync-backend", dest="sync_backend", default=None if legacy else "cpu")
    p.add_argument("--prefetch", type=int, default=None if legacy else 0)
    p.add_argument("--max-checkpoints", dest="max_checkpoints", type=int, default=None)
    p.add_argument("--dtype", default=None if legacy else "f32")
    p.add_argument("--seed", type=int, default=None, help="seed for init and synthetic tokens")
    p.add_argument("--cuda-graph", dest="cuda_graph", action="store_true",
                   help="capture the whole training step in a CUDA graph (one GPU; replayed each step)")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="oxidizr", description="LLM pre-training framework for NVIDIA B200")
    sub = ap.add_subparsers(dest="command")
    t = sub.add_parser("train", help="Train a model (default command)")
    _add_train_args(t)
    pk = sub.add_parser("pack", help="Package a trained model for distribution")
    pk.add_argument("--checkpoint-dir", default="./checkpoints")
    pk.add_argument("-c", "--checkpoint", default=None)
    pk.add_argument("-n", "--name", default=None)
    pk.add_argument("-o", "--output", default=None)
    pk.add_argument("-u", "--username", default=None)
    pu = sub.add_parser("push", help="Push a packaged model to the HuggingFace Hub")
    pu.add_argument("-m", "--model", default=None)
    pu.add_argument("--create-repo", default=True, type=lambda s: s.lower() != "false")
    pu.add_argument("--private", action="store_true")
    pu.add_argument("-t", "--token", default=None)
    pu.add_argument("-y", "--yes", action="store_true")
    return ap


def parse_gpu_ids(s: Optional[str]) -> List[int]:
    """``"0,1,2"`` -> [0, 1, 2]; unparsable entries are skipped; default [0]."""
    if s is None:
        return [0]
    out = []
    for tok in s.split(","):
        try:
            out.append(int(tok.strip()))
        except ValueError:
            pass
    return out


# ===================================================================== train
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch_workers(gpu_ids: List[int], argv: List[str], run_dir: str) -> int:
    """One process per GPU; returns the first non-zero exit code (or 0).

    Watchdog: once a worker has failed, the others get ``OXI_FAIL_GRACE``
    seconds (default 30) to notice it through the process group and exit;
    the ones still running after that are terminated (then killed)."""
    port = _free_port()
    procs = []
    for rank, gid in enumerate(gpu_ids):
        env = dict(os.environ)
        env.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(len(gpu_ids)),
                    "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "OXIDIZED_RUN_DIR": run_dir,
                    "OXI_GPU_ID": str(gid)})
        procs.append(subprocess.Popen([sys.executable, "-m", "oxidizr_b200"] + argv, env=env))
    grace = float(os.environ.get("OXI_FAIL_GRACE", "30"))
    rc, failed_at = 0, None
    while True:
        codes = [p.poll() for p in procs]
        for r, c in enumerate(codes):
            if c not in (None, 0) and failed_at is None:
                failed_at = time.time()
                rc = c
                print(f"Worker {r} exited with code {c}", file=sys.stderr)
        if all(c is not None for c in codes):
            break
        if failed_at is not None and time.time() - failed_at > grace:
            for p in procs:
                if p.poll() is None:
                    p.terminate()
            for p in procs:
                try:
                    p.wait(timeout=10)
                except subprocess.TimeoutExpired:
                    p.kill()
                    p.wait()
            break
        time.sleep(0.2)
    return rc or next((c for c in (p.returncode for p in procs) if c), 0)


def run_train(args, argv: List[str]) -> int:
    import torch

    headless = args.headless
    out = print
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    run_dir = os.environ.get("OXIDIZED_RUN_DIR")
    if run_dir is None:
        run_dir = os.path.join(".", "runs", datetime.datetime.now().strftime("%Y%m%d_%H%M%S"))
    os.makedirs(run_dir, exist_ok=True)
    say = (lambda s: out(s)) if (not headless and rank == 0) else (lambda s: None)
    say("=== Oxidizr Training Framework ===")
    say(f"Run directory: {run_dir}\n")
    say(f"Loading configuration from: {args.config_file}")
    cfg = LitConfig.from_yaml(args.config_file)
    m, t = cfg.model, cfg.trainer
    if args.seq_length is not None:
        say(f"CLI override: seq_length = {args.seq_length} (was {m.max_seq_len})")
        m.max_seq_len = args.seq_length
    if args.batch_size is not None:
        say(f"CLI override: batch_size = {args.batch_size} (was {t.batch_size})")
        t.batch_size = args.batch_size
    if args.gradient_accumulation is not None:
        say(f"CLI override: gradient_accumulation = {args.gradient_accumulation} (was {t.gradient_accumulation})")
        t.gradient_accumulation = args.gradient_accumulation
    if args.max_steps is not None:
        say(f"CLI override: max_steps = {args.max_steps} (was {t.max_steps})")
        t.max_steps = args.max_steps
    gpu_ids = parse_gpu_ids(args.gpus)
    backend = parse_sync_backend(args.sync_backend or "cpu")
    if len(gpu_ids) > 1:
        t.distributed.enabled = True
        t.distributed.gpu_ids = gpu_ids
        t.distributed.backend = backend
        say(f"CLI override: distributed training enabled with {len(gpu_ids)} GPUs: {gpu_ids}")
    elif args.gpus is not None:
        t.distributed.gpu_ids = gpu_ids
    if args.max_checkpoints is not None:
        say(f"CLI override: max_checkpoints = {args.max_checkpoints} (was {t.max_checkpoints})")
        t.max_checkpoints = args.max_checkpoints
    dt = parse_dtype(args.dtype or "f32")
    if dt is None:
        print(f"Warning: Unknown dtype '{args.dtype}', using config default ({m.dtype})", file=sys.stderr)
    elif dt != m.dtype:
        say(f"CLI override: dtype = {dt} (was {m.dtype})")
        m.dtype = dt
    if args.seed is not None:
        m.seed = args.seed
    use_cpu = (args.target_device or t.target_device).lower() == "cpu"

    # one process per GPU
    if t.distributed.enabled and "RANK" not in os.environ:
        return _launch_workers(gpu_ids, argv, run_dir)

    if use_cpu or not torch.cuda.is_available():
        device = torch.device("cpu")
    else:
        gid = int(os.environ.get("OXI_GPU_ID", gpu_ids[rank] if rank < len(gpu_ids) else 0))
        torch.cuda.set_device(gid)
        device = torch.device("cuda", gid)
    say(f"Using device: {device}")
    group = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl" if device.type == "cuda" else "gloo",
                                timeout=datetime.timedelta(seconds=int(os.environ.get("OXI_PG_TIMEOUT", "600"))))
        group = dist.group.WORLD

    from . import checkpoint as C
    from .data import TokenDataLoader, synthetic_tokens
    from .models import build_model
    from .optim import AdamW, AdamWConfig, FlatParams
    from .trainer import NonFiniteLoss, Trainer

    say(f"Initializing model with {m.estimate_params_banner()} parameters...")
    ep_group = group if (m.ep_size and m.ep_size > 1 and world > 1) else None
    model = build_model(m, device=device, ep_group=ep_group)
    ocfg = AdamWConfig(lr=t.learning_rate,
                       weight_decay=t.weight_decay if t.weight_decay is not None else 0.01,
                       max_grad_norm=t.max_grad_norm if t.max_grad_norm is not None else 1.0)
    if world > 1:
        from .parallel.ddp import make_ddp_optimizer
        be = backend if backend != "single" else "nccl"
        if be in ("fused", "nccl_sharded") and device.type != "cuda":
            be = "cpustaging"
        opt = make_ddp_optimizer(model.named_parameters(), ocfg, device, be, group=group, model=model)
        flat = getattr(opt, "flat", None) if be not in ("fused", "nccl_sharded") else None
    else:
        flat = FlatParams(list(model.named_parameters()), device)
        opt = AdamW(flat, ocfg)

    # ------------------------------------------------------------ resume
    start_step = 0
    resume_path = None
    if args.resume:
        if args.resume == "auto":
            say(f"Auto-resume: searching for latest checkpoint in {t.checkpoint_dir}")
            found = C.find_latest_checkpoint(t.checkpoint_dir)
            if found is None:
                say("No checkpoint found, starting fresh")
            else:
                ckpt, meta_path, step = found
                say(f"Found checkpoint: {ckpt} (step {step})")
                if args.data_file:
                    v = C.CheckpointMeta.load(meta_path).validate(m, args.data_file)
                    if not v["is_valid"]:
                        msg = ["Checkpoint mismatch detected!"]
                        if not v["model_matches"]:
                            msg.append(f"Model config mismatch: checkpoint {v['checkpoint_model_hash']} "
                                       f"current {v['current_model_hash']}")
                        if not v["data_matches"]:
                            msg.append(f"Data file mismatch: checkpoint {v['checkpoint_data_hash']} "
                                       f"current {v['current_data_hash']}")
                        if headless:
                            raise RuntimeError("Checkpoint validation failed in headless mode. "
                                               "Clear checkpoints manually or fix config mismatch. " +
                                               "; ".join(msg[1:]))
                        print("\n".join(msg))
                        ans = input("Do you want to clear old checkpoints and start fresh? [y/N]: ")
                        if ans.strip().lower() in ("y", "yes"):
                            n = C.clear_checkpoint_directory(t.checkpoint_dir)
                            print(f"Removed {n} checkpoint file(s)\nStarting fresh training from step 0\n")
                        else:
                            raise RuntimeError("Training aborted by user")
                    else:
                        if not v["dtype_matches"]:
                            say(f"dtype mismatch: checkpoint={v['checkpoint_dtype']}, current={v['current_dtype']}. "
                                "Weights will be converted.")
                        resume_path, start_step = ckpt, step
                else:
                    say("No data file specified, skipping validation")
                    resume_path, start_step = ckpt, step
        else:
            resume_path, start_step = args.resume, C.step_from_filename(args.resume)
    cursor = None
    if resume_path:
        say(f"Loading checkpoint from: {resume_path}")
        C.load_weights(model, resume_path)
        opt.sync_master_from_params()
        meta = C.load_optimizer_sidecar(opt, resume_path)
        if getattr(opt, "local", None) is not None:
            C.load_local_optimizer(opt.local, resume_path, rank)
        if meta and "data_cursor" in meta:
            cursor = int(meta["data_cursor"])
        if start_step:
            say(f"Resuming from step {start_step}")

    # ------------------------------------------------------------ data
    B, S = t.batch_size, m.max_seq_len
    if args.data_file:
        say(f"Loading training data from memory-mapped file: {args.data_file}")
        src = args.data_file
    else:
        say("Creating dummy training data...")
        src = synthetic_tokens(m.vocab_size, 1_000_000 * max(world, 1), seed=m.seed or 0)
    loader = TokenDataLoader(src, B, S, device=device, rank=rank, world_size=world, prefetch=args.prefetch or 0)
    if cursor is not None and world == 1:
        loader.set_cursor(cursor)
    say(f"Data loader ready with {loader.dataset_size()} tokens\n")

    trainer = Trainer(cfg, model, opt, loader, device=device, headless=headless,
                      steps_json_path=os.path.join(run_dir, "steps.json"), start_step=start_step,
                      data_file_path=args.data_file, rank=rank, world_size=world, out=out,
                      cuda_graph=bool(getattr(args, "cuda_graph", False)))
    if not headless and rank == 0:
        _banner(cfg, loader, trainer)
    status, err = "completed", None
    try:
        trainer.fit()
    except Exception as e:  # recorded in run.json like upstream
        status, err = "failed", repr(e)
        if "out of memory" in str(e).lower():
            err = "CUDA out of memory"
            if not headless:
                print("\nCUDA OUT OF MEMORY: reduce batch_size or seq_len, or use --dtype bf16")
    finally:
        loader.close()
    if rank == 0:
        run = {
            "run_dir": run_dir,
            "config": {
                "model": {"name": m.name, "hidden_size": m.hidden_size, "num_layers": m.num_layers,
                          "num_heads": m.num_heads, "num_experts": m.num_experts,
                          "experts_per_tok": m.experts_per_tok, "vocab_size": m.vocab_size,
                          "max_seq_len": m.max_seq_len, "dtype": m.dtype},
                "trainer": {"learning_rate": t.learning_rate, "batch_size": B, "seq_len": S,
                            "gradient_accumulation": t.gradient_accumulation, "max_steps": t.max_steps,
                            "num_epochs": t.num_epochs, "effective_batch_size": B * t.gradient_accumulation,
                            "total_steps": trainer.total_steps},
            },
            "dataset_size": loader.dataset_size(),
            "device": str(device),
            "status": status,
            "error": err,
        }
        with open(os.path.join(run_dir, "run.json"), "w") as fh:
            json.dump(run, fh, indent=2)
        if status == "completed":
            say(f"\nTraining complete! Checkpoints saved to: {t.checkpoint_dir}")
            say(f"Run metadata saved to: {run_dir}/run.json")
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if status != "completed":
        print(f"Error: {err}", file=sys.stderr)
        return 1
    return 0


def _banner(cfg, loader, trainer):
    m, t = cfg.model, cfg.trainer
    n_mamba = len(m.mamba_layers or [])
    kind = "Mamba2" if m.mamba2_num_heads is not None else "Mamba"
    print("\n" + "=" * 60 + "\nOXIDIZR TRAINING\n" + "=" * 60 + "\n")
    print("Configuration:")
    print(f"  Model: {m.estimate_params_banner()} parameters ({n_mamba} {kind} + {m.num_layers - n_mamba} "
          f"attention layers)")
    print(f"  Dataset: {loader.dataset_size()} tokens")
    print(f"  Checkpoint Dir: {t.checkpoint_dir}\n")
    print(f"  Max Seq Length: {m.max_seq_len}")
    if m.num_experts:
        print(f"  MoE: {m.num_experts} experts, Top-{m.experts_per_tok or 1} routing, "
              f"Load balance alpha={t.load_balance_alpha:.3f}")
    print(f"  Batch Size: {t.batch_size}, Gradient Accumulation: {t.gradient_accumulation}")
    print(f"  Learning Rate: {t.learning_rate:.6f}")
    print(f"  Epochs: {t.num_epochs}\n")
    print(f"Training Plan: {trainer.steps_per_epoch} steps/epoch | Total steps = {trainer.total_steps}")
    print("=" * 60 + "\nSTARTING TRAINING\n" + "=" * 60 + "\n")


# ================================================================= pack/push
def _dotenv():
    if os.path.exists(".env"):
        for line in open(".env"):
            line = line.strip()
            if line and not line.startswith("#") and "=" in line:
                k, v = line.split("=", 1)
                os.environ.setdefault(k.strip(), v.strip().strip('"').strip("'"))


def run_pack(args) -> int:
    from .pack import pack
    _dotenv()
    return pack(args.checkpoint_dir, args.checkpoint, args.name, args.output, args.username)


def run_push(args) -> int:
    from .pack import push
    _dotenv()
    return push(args.model, args.private, args.token, args.yes)


# ===================================================================== main
def main(argv: Optional[List[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] in ("train", "pack", "push", "-h", "--help"):
        args = build_parser().parse_args(argv)
        if args.command == "train":
            return run_train(args, argv)
        if args.command == "pack":
            return run_pack(args)
        if args.command == "push":
            return run_push(args)
        return 0
    # legacy form: oxidizr -f <config> [train flags]
    lp = argparse.ArgumentParser(prog="oxidizr")
    _add_train_args(lp, legacy=True)
    args = lp.parse_args(argv)
    if args.config_file is None:
        print("Oxidizr: LLM pre-training framework for NVIDIA B200\n")
        print("Usage:")
        print("  oxidizr train -f <config.yaml>     Train a model")
        print("  oxidizr pack                       Package a trained model")
        print("  oxidizr push                       Push model to HuggingFace")
        print("\nLegacy usage (backwards compatible):")
        print("  oxidizr -f <config.yaml>           Same as 'oxidizr train -f'")
        return 0
    args.sync_backend = args.sync_backend or "cpu"
    args.prefetch = args.prefetch or 0
    args.dtype = args.dtype or "f32"
    return run_train(args, ["train"] + argv)


if __name__ == "__main__":
    sys.exit(main())
