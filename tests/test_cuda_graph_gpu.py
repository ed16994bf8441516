"""Whole-step CUDA graph (Trainer(cuda_graph=True)) against eager steps."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(model_extra=None):
    from oxidizr_b200.config import LitConfig
    from oxidizr_b200.models import build_model
    from oxidizr_b200.optim import AdamW, AdamWConfig, FlatParams
    m = {"name": "graph", "hidden_size": 256, "num_layers": 2, "num_heads": 2, "kv_heads": 1,
         "intermediate_size": 256, "vocab_size": 1000, "max_seq_len": 128, "rope_theta": 10000.0, "dtype": "bf16"}
    m.update(model_extra or {})
    cfg = LitConfig.from_dict({"model": m, "trainer": {
        "learning_rate": 1e-3, "batch_size": 2, "max_steps": 0, "num_epochs": 1, "gradient_accumulation": 2,
        "checkpoint_dir": "/tmp/oxi_graph", "log_interval": 1, "save_interval": 1000, "load_balance_alpha": 0.01,
        "group_size": 4, "beta_kl": 0.04}})
    dev = torch.device("cuda", 0)
    model = build_model(cfg.model, device=dev, seed=0)
    opt = AdamW(FlatParams(list(model.named_parameters()), dev), AdamWConfig(lr=1e-3))
    return cfg, model, opt, dev


class _Batches:
    batch_size, seq_len = 2, 128

    def __init__(self, dev):
        g = torch.Generator(device=dev).manual_seed(7)
        self.pool = [torch.randint(0, 1000, (2, 129), generator=g, device=dev) for _ in range(24)]
        self.i = 0

    def dataset_size(self):
        return 10 ** 9

    def next_batch(self):
        b = self.pool[self.i % len(self.pool)]
        self.i += 1
        return b[:, :-1], b[:, 1:]


@pytest.mark.parametrize("extra", [None, {"num_experts": 4, "experts_per_tok": 2, "shared_expert_enabled": True,
                                          "num_shared_experts": 1}])
def test_graphed_steps_match_eager(extra):
    from oxidizr_b200.trainer import Trainer
    from oxidizr_b200.ops._C import check_status
    losses = {}
    params = {}
    for graph in (False, True):
        cfg, model, opt, dev = _setup(extra)
        tr = Trainer(cfg, model, opt, _Batches(dev), device=dev, out=lambda s: None, cuda_graph=graph)
        assert tr.cuda_graph == graph
        seq = []
        for _ in range(8):
            loss, gn = tr.training_step()
            seq.append((float(loss), float(gn)))
        torch.cuda.synchronize()
        check_status(dev)
        losses[graph] = seq
        params[graph] = torch.cat([p.detach().float().flatten() for p in model.parameters()])
        if graph:
            assert tr._graph is not None and tr._graph_launches > 0
    for (le, ge), (lg, gg) in zip(losses[False], losses[True]):
        assert abs(le - lg) <= 2e-3 * abs(le) and abs(ge - gg) <= 2e-2 * abs(ge) + 1e-4, (losses[False], losses[True])
    d = (params[False] - params[True]).norm() / params[False].norm()
    assert d < 1e-2, d
