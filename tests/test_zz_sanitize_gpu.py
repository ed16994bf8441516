"""Sanitizer stand-ins on the GPU: the tcgen05 GEMM writes nothing outside its output (canary
guards on every layout, bf16 and f32 += outputs, ragged sizes), and a small bf16 model's
training steps rerun to within the run-to-run spread of f32 atomics."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_gemm_outputs_keep_their_guards():
    from oxidizr_b200.utils import sanitize as S
    rep = S.canary_gemm_sweep(torch.device("cuda", 0))
    assert len(rep) == 24
    bad = {k: (r.head_overwritten, r.tail_overwritten) for k, r in rep.items() if not r.ok}
    assert not bad, bad


def test_training_steps_rerun_on_gpu(tmp_path):
    from oxidizr_b200.config import LitConfig
    from oxidizr_b200.utils import sanitize as S
    cfg = LitConfig.from_dict({"model": {
        "name": "rerun", "hidden_size": 256, "num_layers": 2, "num_heads": 2, "kv_heads": 1,
        "intermediate_size": 256, "vocab_size": 1000, "max_seq_len": 128, "rope_theta": 10000.0, "dtype": "bf16"},
        "trainer": {"learning_rate": 1e-3, "batch_size": 2, "max_steps": 0, "num_epochs": 1,
                    "gradient_accumulation": 1, "checkpoint_dir": str(tmp_path), "log_interval": 1,
                    "save_interval": 1000, "load_balance_alpha": 0.0, "group_size": 4, "beta_kl": 0.0}})
    runs = [S.train_run(cfg, 3, torch.device("cuda", 0)) for _ in range(2)]
    losses = [l for l, _ in runs[0]["losses"]]
    assert all(l == l and l > 0 for l in losses)
    # split-K and the norm / bias reductions add f32 partials in a run-dependent order
    assert S.max_abs_diff(runs[0]["losses"], runs[1]["losses"]) < 1e-2
    assert S.max_abs_diff(runs[0]["params"], runs[1]["params"]) < 1e-2
