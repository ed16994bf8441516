"""bench.py's contract with its caller, on the CPU: the reference arm's one-line JSON, the
clock sampler's parsing of nvidia-smi lines, and the model configs against the BASELINE.json
configs they claim to be."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def test_reference_arm_prints_one_unavailable_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--gpus", "1",
                        "--steps", "3", "--warmup", "3"], capture_output=True, text=True, timeout=120, cwd=REPO)
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"]


def test_clock_sampler_parses_clocks_and_reasons():
    import bench

    class Proc:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            return 0

        def kill(self):
            pass

    class Thread:
        def join(self, timeout=None):
            pass

    cs = bench.ClockSampler(0)
    cs.proc, cs.t = Proc(), Thread()
    cs.lines = [
        "0, 1965, 1965, 480.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1500, 1965, 990.5, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1600, 1965, 985.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "not a sample",
    ]
    r = cs.stop()
    assert r["samples"] == 3 and r["sm_mhz"] == 1600.0 and r["sm_max_mhz"] == 1965.0
    assert r["power_w_max"] == 990.5 and r["reasons"] == ["sw_power_cap"]


def test_clock_sampler_without_nvidia_smi():
    import bench
    r = bench.ClockSampler(0).stop()
    assert r["sm_mhz"] is None and r["reasons"] == ["nvidia-smi unavailable"]


@pytest.mark.parametrize("name,expect", [
    ("llama", dict(hidden_size=2048, num_layers=16, num_heads=16, kv_heads=8, intermediate_size=5632,
                   vocab_size=128354, max_seq_len=2048, rope_theta=1e4, batch=8)),
    ("hybrid", dict(hidden_size=768, num_layers=8, mamba2_state_size=128, mamba2_head_dim=64, mamba2_expand=2,
                    mamba2_conv_kernel=4, mamba2_chunk_size=256, num_heads=12, q_latent_dim=512, kv_latent_dim=256,
                    d_rope=32, num_experts=32, experts_per_tok=4, num_shared_experts=1, intermediate_size=512,
                    vocab_size=100277, max_seq_len=1024, batch=16, load_balance_alpha=0.01)),
    ("mamba3", dict(hidden_size=1024, num_layers=24, mamba2_state_size=128, mamba2_head_dim=64, mamba2_expand=2,
                    mamba3_enabled=True, mamba3_complex_rope=True, mamba3_mimo_rank=4, mamba2_chunk_size=256,
                    vocab_size=100277, max_seq_len=4096, batch=4)),
    ("moe", dict(hidden_size=2048, num_layers=16, num_heads=16, kv_heads=4, rope_theta=5e5, num_experts=64,
                 experts_per_tok=8, num_shared_experts=2, intermediate_size=1024, vocab_size=128354,
                 max_seq_len=4096, batch=4)),
])
def test_bench_models_are_the_baseline_configs(name, expect):
    import bench
    cfg = bench.bench_config(name)
    m, t = cfg.model, cfg.trainer
    for k, v in expect.items():
        if k == "batch":
            assert t.batch_size == v
        elif k == "load_balance_alpha":
            assert t.load_balance_alpha == v
        else:
            assert getattr(m, k) == v, (k, getattr(m, k), v)
    assert m.dtype == "bf16"
    if name == "hybrid":  # 6 Mamba2 layers and 2 MLA + MoE layers
        assert len(m.mamba_layers) == 6 and not m.mamba3_enabled
    if name == "mamba3":
        assert list(m.mamba_layers) == list(range(24))
