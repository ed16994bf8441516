"""End-to-end ``oxidizr train`` runs on CPU (single process and gloo ranks),
checkpoint resume, expert-parallel checkpoints, and host-side failure
detection (a rank that raises, hangs or produces a NaN loss)."""
import glob
import json
import os
import subprocess
import sys
import time

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(tmp_path, moe=False, ep=None, steps=4, save_interval=2):
    model = {
        "name": "tiny", "hidden_size": 64, "num_layers": 2, "num_heads": 4, "kv_heads": 2,
        "intermediate_size": 128, "vocab_size": 512, "max_seq_len": 32, "rope_theta": 10000.0,
    }
    if moe:
        model.update({"num_experts": 4, "experts_per_tok": 2, "num_shared_experts": 1})
    if ep:
        model["ep_size"] = ep
    import yaml
    cfg = {"model": model, "trainer": {
        "learning_rate": 1e-3, "batch_size": 2, "max_steps": steps, "num_epochs": 1, "gradient_accumulation": 1,
        "checkpoint_dir": str(tmp_path / "ckpt"), "log_interval": 1, "save_interval": save_interval,
        "load_balance_alpha": 0.01 if moe else 0.0, "group_size": 4, "beta_kl": 0.04}}
    p = tmp_path / "cfg.yaml"
    p.write_text(yaml.safe_dump(cfg))
    from oxidizr_b200 import data as D
    dp = tmp_path / "tokens.bin"
    D.write_tokens(str(dp), D.synthetic_tokens(512, 20000, seed=1))
    return str(p), str(dp)


def _train(tmp_path, cfg, data, *extra, env=None, timeout=240, headless=True):
    e = dict(os.environ, PYTHONPATH=REPO, OMP_NUM_THREADS="1", OXIDIZED_RUN_DIR=str(tmp_path / "run"))
    os.makedirs(e["OXIDIZED_RUN_DIR"], exist_ok=True)
    e.update(env or {})
    cmd = [sys.executable, "-m", "oxidizr_b200", "train", "-f", cfg, "-d", data, "--target-device", "cpu",
           *(["--headless"] if headless else []), *extra]
    t0 = time.time()
    r = subprocess.run(["timeout", "-k", "20", str(timeout)] + cmd, cwd=str(tmp_path), env=e, capture_output=True,
                       text=True)
    return r, time.time() - t0


def _steps(stdout):
    return [json.loads(l) for l in stdout.splitlines() if l.startswith('{"step"')]


def test_train_cpu_then_resume(tmp_path):
    # interactive mode saves step checkpoints (headless saves only the final one, like upstream)
    cfg, data = _cfg(tmp_path, steps=4)
    r, _ = _train(tmp_path, cfg, data, headless=False)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "Training complete" in r.stdout
    ck = tmp_path / "ckpt"
    assert glob.glob(str(ck / "*_final.safetensors"))
    assert glob.glob(str(ck / "*_step_2.safetensors")) and glob.glob(str(ck / "checkpoint_step_2.meta.json"))
    assert glob.glob(str(ck / "*_step_2.optim.safetensors"))
    run = json.load(open(tmp_path / "run" / "run.json"))
    assert run["status"] == "completed"
    # resume (headless): the newest step checkpoint is picked up and training continues to max_steps
    r2, _ = _train(tmp_path, cfg, data, "--max-steps", "6", "--resume", "auto")
    assert r2.returncode == 0, r2.stderr[-3000:]
    lines = _steps(r2.stdout)
    assert all(set(l) == {"step", "loss", "grad_norm", "learning_rate", "epoch", "it/s", "vram"} for l in lines)
    steps2 = [l["step"] for l in lines]
    assert steps2 and steps2[0] > 1 and steps2[-1] == 6, steps2


def test_ddp_gloo_expert_parallel_checkpoint(tmp_path):
    cfg, data = _cfg(tmp_path, moe=True, ep=2, steps=3, save_interval=2)
    r, _ = _train(tmp_path, cfg, data, "--gpus", "0,1", "--sync-backend", "cpu", headless=False)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    from safetensors.torch import load_file
    final = glob.glob(str(tmp_path / "ckpt" / "*_final.safetensors"))[0]
    sd = load_file(final)
    for i in range(2):
        for e in range(4):
            assert f"layers.{i}.mlp.experts.{e}.gate_proj.weight" in sd or \
                any(k.endswith(f".experts.{e}.gate_proj.weight") and k.startswith(f"layers.{i}.") for k in sd), (i, e)
    # every rank wrote the optimizer state of its own experts
    assert len(glob.glob(str(tmp_path / "ckpt" / "*_step_2.optim.local*.safetensors"))) == 2


@pytest.mark.parametrize("kind", ["raise", "hang", "nan"])
def test_failure_detection_gloo(tmp_path, kind):
    """A faulty rank ends the whole job quickly with an error status."""
    cfg, data = _cfg(tmp_path, steps=8, save_interval=100)
    env = {"OXI_FAULT": f"1:2:{kind}" if kind != "nan" else "0:2:nan", "OXI_PG_TIMEOUT": "15",
           "OXI_FAIL_GRACE": "5", "OXI_FAULT_HANG_S": "120"}
    r, dt = _train(tmp_path, cfg, data, "--gpus", "0,1", "--sync-backend", "cpu", env=env, timeout=150)
    assert r.returncode != 0, r.stdout[-2000:]
    assert dt < 100, dt
    run = json.load(open(tmp_path / "run" / "run.json"))
    assert run["status"] == "failed"
    if kind == "nan":
        assert "NaN" in run["error"]


def test_pack_then_push_with_a_fake_hf(tmp_path):
    """pack copies the final checkpoint and config into hf/<user>/<model>/ with a model card;
    push runs `hf upload <user>/<model> <dir> --repo-type model [--token] [--private]`
    (a fake `hf` on PATH records its arguments; nothing is uploaded)."""
    cfg, data = _cfg(tmp_path, steps=2, save_interval=1000)
    r, _ = _train(tmp_path, cfg, data)
    assert r.returncode == 0, r.stderr[-3000:]
    e = dict(os.environ, PYTHONPATH=REPO, OXIDIZED_RUN_DIR=str(tmp_path / "run"))
    rp = subprocess.run([sys.executable, "-m", "oxidizr_b200", "pack", "--checkpoint-dir", str(tmp_path / "ckpt"),
                         "-c", "final", "-u", "alice", "-n", "tiny-test"], cwd=str(tmp_path), env=e,
                        capture_output=True, text=True, timeout=120)
    assert rp.returncode == 0, rp.stderr[-2000:]
    out = tmp_path / "hf" / "alice" / "tiny-test"
    for f in ("model.safetensors", "config.json", "README.md"):
        assert (out / f).exists(), f
    bindir = tmp_path / "bin"
    bindir.mkdir()
    rec = tmp_path / "hf_args.txt"
    fake = bindir / "hf"
    fake.write_text(f'#!/bin/sh\nprintf "%s\\n" "$@" > "{rec}"\n')
    fake.chmod(0o755)
    e2 = dict(e, PATH=f"{bindir}{os.pathsep}{os.environ.get('PATH', '')}")
    e2.pop("HF_TOKEN", None)
    ru = subprocess.run([sys.executable, "-m", "oxidizr_b200", "push", "-m", "alice/tiny-test", "--private",
                         "-t", "tok123", "-y"], cwd=str(tmp_path), env=e2, capture_output=True, text=True, timeout=120)
    assert ru.returncode == 0, ru.stderr[-2000:]
    assert rec.read_text().split("\n")[:-1] == ["upload", "alice/tiny-test", os.path.join("hf", "alice", "tiny-test"),
                                                 "--repo-type", "model", "--token", "tok123", "--private"]
    assert "Upload complete: https://huggingface.co/alice/tiny-test" in ru.stdout


def test_throughput_sweep_on_cpu(tmp_path):
    """The (seq, batch, accumulation) sweep writes upstream's logs.txt / results.csv layout with
    the numbers read from the trainer's JSON lines."""
    from oxidizr_b200.utils import sweep
    cfg, data = _cfg(tmp_path, steps=4)
    res = sweep.run([(16, 1, 1), (16, 2, 2)], cfg, 1, ["-d", data, "--target-device", "cpu"],
                    str(tmp_path / "benchmark"), timeout=240)
    lines = open(res).read().splitlines()
    assert lines[0] == sweep.HEADER and len(lines) == 3
    rows = [ln.split(",") for ln in lines[1:]]
    assert [r[:4] for r in rows] == [["16", "1", "1", "1"], ["16", "2", "2", "4"]]
    assert all(r[6] == "" and float(r[5]) > 0 for r in rows), rows
    assert os.path.exists(os.path.join(os.path.dirname(res), "logs.txt"))
    assert len(sweep.DEFAULT_GRID) == 50


def test_sweep_classifies_failures():
    from oxidizr_b200.utils.sweep import classify
    assert classify(1, "RuntimeError: CUDA out of memory. Tried to allocate")[0] == "OOM"
    assert classify(1, "Traceback (most recent call last):\nValueError: bad")[0] == "ERROR"
    assert classify(3, "")[0] == "UNKNOWN_ERROR"
    assert classify(None, "")[0] == "TIMEOUT"
    assert classify(0, "no json here")[0] == "NO_OUTPUT"
    notes, rec = classify(0, '{"step": 1, "loss": 6.1, "it/s": 3.25, "vram": "0"}\nSaving final checkpoint')
    assert notes == "" and rec["it/s"] == 3.25
