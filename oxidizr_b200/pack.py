"""``pack`` and ``push`` (commands/pack.rs, commands/push.rs).

pack: find ``*_final.safetensors`` under the checkpoint dir (recursively),
select one (``latest`` = highest step else first, ``final``, a step number,
or an interactive choice), and write ``hf/<user>/<model>/`` with
``model.safetensors`` (copy of the weights), ``config.json`` (copy of the
inference config next to the checkpoint), ``training_config.json`` (copy of the
newest ``runs/*/run.json``, when present) and a generated ``README.md`` model
card.

push: validate ``hf/<user>/<model>`` and run
``hf upload <user>/<model> <dir> --repo-type model [--token T] [--private]``.

Upstream lines: ``PackArgs`` commands/pack.rs:15-35, ``scan_checkpoints`` commands/pack.rs:58-77,
``select_checkpoint`` commands/pack.rs:124-167, ``generate_model_card`` commands/pack.rs:228-400,
``run_pack`` commands/pack.rs:525-638; ``PushArgs`` commands/push.rs:14-34, ``scan_packaged_models``
commands/push.rs:76-128, ``run_push`` commands/push.rs:172-277 (command at commands/push.rs:240-255).
"""
from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
from typing import List, Optional


class CkptInfo:
    def __init__(self, path: str):
        self.path = path
        self.name = os.path.splitext(os.path.basename(path))[0]
        self.parent_dir = os.path.basename(os.path.dirname(path)) or None
        self.is_final = self.name.endswith("_final")
        self.step = None
        if not self.is_final and "_step_" in self.name:
            try:
                self.step = int(self.name.split("_step_")[-1])
            except ValueError:
                self.step = None
        self.size_mb = os.path.getsize(path) / (1024 * 1024)

    def display_name(self) -> str:
        pre = f"{self.parent_dir}/" if self.parent_dir else ""
        return f"{pre}{self.name} - {self.size_mb:.1f} MB"


def scan_checkpoints(checkpoint_dir: str) -> List[CkptInfo]:
    if not os.path.isdir(checkpoint_dir):
        raise FileNotFoundError(f"Checkpoint directory does not exist: {checkpoint_dir}")
    found = []
    for root, _, files in os.walk(checkpoint_dir):
        for f in files:
            if f.endswith(".safetensors") and not f.endswith(".optim.safetensors"):
                found.append(CkptInfo(os.path.join(root, f)))
    found = [c for c in found if c.is_final]
    found.sort(key=lambda c: c.name)
    return found


def select_checkpoint(cks: List[CkptInfo], selection: Optional[str]) -> CkptInfo:
    if not cks:
        raise RuntimeError("No checkpoints found in directory")
    if selection == "latest":
        stepped = [c for c in cks if not c.is_final and c.step is not None]
        return max(stepped, key=lambda c: c.step) if stepped else cks[0]
    if selection == "final":
        for c in cks:
            if c.is_final:
                return c
        raise RuntimeError("No final checkpoint found")
    if selection is not None:
        try:
            step = int(selection)
        except ValueError:
            raise RuntimeError("Invalid checkpoint selector. Use 'latest', 'final', or a step number")
        for c in cks:
            if c.step == step:
                return c
        raise RuntimeError(f"Checkpoint for step {step} not found")
    for i, c in enumerate(cks):
        print(f"  [{i}] {c.display_name()}")
    ans = input("Select a checkpoint to pack [0]: ").strip() or "0"
    return cks[int(ans)]


def _latest_run_file(name: str) -> Optional[str]:
    runs = "./runs"
    if not os.path.isdir(runs):
        return None
    dirs = sorted(d for d in os.listdir(runs) if os.path.isdir(os.path.join(runs, d)))
    if not dirs:
        return None
    p = os.path.join(runs, dirs[-1], name)
    return p if os.path.exists(p) else None


def _training_stats(checkpoint_dir: str) -> Optional[dict]:
    for p in (_latest_run_file("steps.json"), os.path.join(checkpoint_dir, "steps.json")):
        if p and os.path.exists(p):
            lines = [l for l in open(p).read().splitlines() if l.strip()]
            if lines:
                try:
                    return json.loads(lines[-1])
                except json.JSONDecodeError:
                    pass
    return None


def describe_architecture(cfg: dict) -> str:
    parts = []
    n_m = len(cfg.get("mamba_layers", []))
    if n_m and cfg.get("mamba2_num_heads") is not None:
        parts.append(f"{n_m} {'Mamba3' if cfg.get('mamba3_enabled') else 'Mamba2'}")
    n_a = max(cfg["num_layers"] - n_m, 0)
    if n_a:
        parts.append(f"{n_a} {'MLA' if cfg.get('kv_latent_dim') is not None else 'Attention'}")
    if cfg.get("num_experts") is not None:
        parts.append(f"MoE ({cfg['num_experts']} experts, top-{cfg.get('experts_per_tok') or 2})")
    return " + ".join(parts) if parts else "Transformer"


def estimate_params(cfg: dict) -> str:
    H, V, L = cfg["hidden_size"], cfg["vocab_size"], cfg["num_layers"]
    I = cfg.get("intermediate_size") or 4 * H
    total = V * H + L * (4 * H * H + 3 * H * I) + H * V
    if total > 1_000_000_000:
        return f"{total / 1e9:.2f}B"
    if total > 1_000_000:
        return f"{total / 1e6:.2f}M"
    return f"{total // 1000}K"


def model_card(model_name: str, username: str, cfg: dict, stats: Optional[dict]) -> str:
    tags = ["oxidizr", "llm"] + (["mamba"] if cfg.get("mamba2_num_heads") is not None else []) + \
        (["mla"] if cfg.get("kv_latent_dim") is not None else []) + (["moe"] if cfg.get("num_experts") else [])
    arch = describe_architecture(cfg)
    params = estimate_params(cfg)
    lines = ["---", "license: apache-2.0", "library_name: oxidizr", "tags:"] + [f"- {t}" for t in tags] + [
        "pipeline_tag: text-generation", "---", "", f"# {model_name}", "",
        f"{arch} language model, about {params} parameters, pre-trained with oxidizr on NVIDIA B200.", "",
        "## Specifications", "", "| Property | Value |", "|---|---|",
        f"| Architecture | {arch} |", f"| Parameters | {params} |", f"| Hidden size | {cfg['hidden_size']} |",
        f"| Layers | {cfg['num_layers']} |", f"| Vocabulary | {cfg['vocab_size']} |",
        f"| Context length | {cfg['max_seq_len']} |", ""]
    if stats:
        lines += ["## Training", ""]
        if "loss" in stats:
            lines.append(f"- Final loss: {stats['loss']:.4f}")
        if "step" in stats:
            lines.append(f"- Training steps: {stats['step']}")
        if "learning_rate" in stats:
            lines.append(f"- Learning rate: {stats['learning_rate']:.2e}")
        lines.append("")
    lines += ["## Files", "", "- `model.safetensors`: weights (upstream oxidizr tensor names)",
              "- `config.json`: inference configuration", "",
              f"Repository id: `{username}/{model_name}`", ""]
    return "\n".join(lines)


def pack(checkpoint_dir: str, selection: Optional[str], name: Optional[str], output: Optional[str],
         username: Optional[str]) -> int:
    username = username or os.environ.get("HF_USERNAME")
    if not username:
        print("HuggingFace username not specified. Use --username or set HF_USERNAME in .env", file=sys.stderr)
        return 1
    print("Oxidizr Model Packer\n")
    print(f"Scanning checkpoints in: {checkpoint_dir}")
    cks = scan_checkpoints(checkpoint_dir)
    print(f"Found {len(cks)} checkpoint(s)\n")
    ck = select_checkpoint(cks, selection)
    print(f"Selected: {ck.display_name()}\n")
    cfg_path = os.path.join(os.path.dirname(ck.path), "config.json")
    if not os.path.exists(cfg_path):
        print(f"config.json not found in {os.path.dirname(ck.path)}. Was this model trained with oxidizr?",
              file=sys.stderr)
        return 1
    cfg = json.load(open(cfg_path))
    if name is None:
        fn = ck.name
        name = fn[:fn.index("_step_")] if "_step_" in fn else (fn[:-len("_final")] if fn.endswith("_final") else fn)
    out_dir = output or os.path.join("hf", username, name)
    os.makedirs(out_dir, exist_ok=True)
    print(f"Packing model: {name}\nOutput directory: {out_dir}\n")
    shutil.copyfile(ck.path, os.path.join(out_dir, "model.safetensors"))
    shutil.copyfile(cfg_path, os.path.join(out_dir, "config.json"))
    rj = _latest_run_file("run.json")
    if rj:
        shutil.copyfile(rj, os.path.join(out_dir, "training_config.json"))
    with open(os.path.join(out_dir, "README.md"), "w") as fh:
        fh.write(model_card(name, username, cfg, _training_stats(checkpoint_dir)))
    print("Model packed successfully!")
    print(f"Next: oxidizr push --model {out_dir}")
    return 0


def scan_packaged() -> List[dict]:
    out = []
    if not os.path.isdir("hf"):
        return out
    for user in sorted(os.listdir("hf")):
        up = os.path.join("hf", user)
        if not os.path.isdir(up):
            continue
        for model in sorted(os.listdir(up)):
            mp = os.path.join(up, model)
            if os.path.isdir(mp):
                out.append({"path": mp, "user": user, "model": model,
                            "has_model": os.path.exists(os.path.join(mp, "model.safetensors")),
                            "has_config": os.path.exists(os.path.join(mp, "config.json"))})
    return out


def push_command(repo_id: str, path: str, token: Optional[str], private: bool) -> List[str]:
    cmd = ["hf", "upload", repo_id, path, "--repo-type", "model"]
    if token:
        cmd += ["--token", token]
    if private:
        cmd.append("--private")
    return cmd


def push(model: Optional[str], private: bool, token: Optional[str], yes: bool) -> int:
    if shutil.which("hf") is None:
        print("hf CLI not found. Install it with: pip install huggingface_hub; then run: hf login",
              file=sys.stderr)
        return 1
    token = token or os.environ.get("HF_TOKEN")
    models = scan_packaged()
    print(f"Found {len(models)} packaged model(s)\n")
    if model is None:
        if not models:
            print("No packaged models found in hf/ directory. Run 'oxidizr pack' first.", file=sys.stderr)
            return 1
        for i, m in enumerate(models):
            ok = "ok" if m["has_model"] and m["has_config"] else "incomplete"
            print(f"  [{i}] {m['user']}/{m['model']} ({ok})")
        sel = models[int(input("Select a model to push [0]: ").strip() or "0")]
    else:
        cand = [m for m in models if os.path.normpath(m["path"]) == os.path.normpath(model)
                or f"{m['user']}/{m['model']}" == model]
        if not cand:
            print(f"Model not found: {model}", file=sys.stderr)
            return 1
        sel = cand[0]
    if not (sel["has_model"] and sel["has_config"]):
        print(f"Model {sel['user']}/{sel['model']} is incomplete", file=sys.stderr)
        return 1
    repo = f"{sel['user']}/{sel['model']}"
    if not yes and input(f"Push to https://huggingface.co/{repo}? [Y/n]: ").strip().lower() in ("n", "no"):
        print("Aborted.")
        return 0
    rc = subprocess.call(push_command(repo, sel["path"], token, private))
    if rc == 0:
        print(f"Upload complete: https://huggingface.co/{repo}")
        return 0
    print("Upload failed. Check your token and try again. If not logged in, run: hf login", file=sys.stderr)
    return 1
