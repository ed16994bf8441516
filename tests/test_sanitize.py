"""Host-side sanitizer stand-ins (oxidizr_b200/utils/sanitize.py): canary guards catch
out-of-bounds writes, the rerun comparison separates deterministic from racy work, and a
tiny model's training steps rerun bit-identically on the CPU."""
import pytest
import torch

from oxidizr_b200.utils import sanitize as S


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float64, torch.int32, torch.uint8])
def test_guards_catch_writes_past_either_end(dtype):
    g = S.Guarded((3, 5), dtype, "cpu", guard=16)
    g.tensor.fill_(1)  # writes inside the tensor only
    assert g.check().ok
    g.buf[g.guard - 1] = 0          # one element before the start
    g.buf[g.guard + g.n + 3] = 2    # and two past the end
    g.buf[g.guard + g.n + 4] = 2
    r = g.check()
    assert (r.head_overwritten, r.tail_overwritten) == (1, 2) and not r.ok


def test_guarded_view_is_the_requested_tensor():
    g = S.Guarded((4, 8), torch.float32, "cpu", guard=32, fill=0.5)
    assert g.tensor.shape == (4, 8) and g.tensor.is_contiguous()
    assert bool((g.tensor == 0.5).all())
    assert g.tensor.data_ptr() == g.buf.data_ptr() + 32 * 4


def test_max_abs_diff_nested_and_nan():
    a = {"x": torch.tensor([1.0, 2.0]), "y": [torch.tensor([3.0]), 4.0]}
    b = {"x": torch.tensor([1.0, 2.5]), "y": [torch.tensor([3.0]), 4.25]}
    assert S.max_abs_diff(a, b) == 0.5
    nan = float("nan")
    assert S.max_abs_diff(torch.tensor([nan, 1.0]), torch.tensor([nan, 1.0])) == 0.0
    d = S.max_abs_diff(torch.tensor([nan]), torch.tensor([0.0]))
    assert d != d


def test_rerun_check_separates_deterministic_from_racy_work():
    def det():
        g = torch.Generator().manual_seed(0)
        x = torch.randn(64, 64, generator=g)
        return x @ x.t()

    calls = {"n": 0}

    def racy():  # a result that depends on the run, as a race would make it
        calls["n"] += 1
        return torch.full((4,), float(calls["n"]))

    assert S.rerun_check(det, runs=3) == 0.0
    assert S.rerun_check(racy, runs=2) == 1.0


def test_training_steps_rerun_bit_identically_on_cpu(tmp_path):
    from oxidizr_b200.config import LitConfig
    cfg = LitConfig.from_dict({"model": {
        "name": "rerun", "hidden_size": 64, "num_layers": 2, "num_heads": 2, "kv_heads": 1,
        "intermediate_size": 128, "vocab_size": 97, "max_seq_len": 16, "rope_theta": 10000.0, "dtype": "f32"},
        "trainer": {"learning_rate": 1e-3, "batch_size": 2, "max_steps": 0, "num_epochs": 1,
                    "gradient_accumulation": 1, "checkpoint_dir": str(tmp_path), "log_interval": 1,
                    "save_interval": 1000, "load_balance_alpha": 0.0, "group_size": 4, "beta_kl": 0.0}})
    runs = [S.train_run(cfg, 2, torch.device("cpu")) for _ in range(2)]
    assert len(runs[0]["losses"]) == 2
    assert S.max_abs_diff(runs[0]["losses"], runs[1]["losses"]) == 0.0
    assert S.max_abs_diff(runs[0]["params"], runs[1]["params"]) == 0.0
    # and the steps did change the parameters
    from oxidizr_b200.models import build_model
    init = {n: p.detach().clone() for n, p in build_model(cfg.model, device=torch.device("cpu"), seed=0)
            .named_parameters()}
    assert S.max_abs_diff(init, runs[0]["params"]) > 0.0
