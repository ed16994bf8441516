"""Token loader semantics, checkpoint files and resume (CPU)."""
import json
import os

import numpy as np
import pytest
import torch

from oxidizr_b200 import checkpoint as C
from oxidizr_b200 import data as D
from oxidizr_b200.config import LitConfig

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_loader_batches_overlap_and_wrap(tmp_path):
    toks = np.arange(100, dtype=np.uint32)
    p = str(tmp_path / "t.bin")
    D.write_tokens(p, toks)
    assert os.path.getsize(p) == 400
    ld = D.TokenDataLoader(p, batch_size=2, seq_len=8)
    x, y = ld.next_batch()
    assert x.tolist() == [list(range(0, 8)), list(range(9, 17))]
    assert y.tolist() == [list(range(1, 9)), list(range(10, 18))]
    x2, _ = ld.next_batch()  # cursor advanced by B*S = 16 (overlap of B tokens)
    assert x2[0, 0].item() == 16
    for _ in range(10):
        xx, _ = ld.next_batch()
    assert ld.cursor <= 100
    assert ld.dataset_size() == 100


def test_loader_sharding_and_prefetch(tmp_path):
    toks = np.arange(1000, dtype=np.uint32)
    p = str(tmp_path / "t.bin")
    D.write_tokens(p, toks)
    a = D.TokenDataLoader(p, 2, 8, rank=0, world_size=3)
    b = D.TokenDataLoader(p, 2, 8, rank=2, world_size=3, prefetch=3)
    assert a.shard_size() == 333 and b.shard_size() == 334
    xa, _ = a.next_batch()
    xb, _ = b.next_batch()
    assert xa[0, 0].item() == 0 and xb[0, 0].item() == 666
    seq = [b.next_batch()[0][0, 0].item() for _ in range(5)]
    assert seq == [666 + 16 * (i + 1) for i in range(5)]
    b.close()


def test_loader_rejects_bad_file(tmp_path):
    p = tmp_path / "bad.bin"
    p.write_bytes(b"\x00" * 7)
    with pytest.raises(RuntimeError, match="multiple of u32"):
        D.TokenDataLoader(str(p), 1, 1)


def test_synthetic_tokens_seeded():
    a = D.synthetic_tokens(1000, 50, seed=5)
    b = D.synthetic_tokens(1000, 50, seed=5)
    assert (a == b).all() and a.max() < 1000 and a.dtype == np.uint32


def _cfg(tmp_path):
    c = LitConfig.from_yaml(os.path.join(REPO, "models", "nano-start.yaml"))
    c.model.max_seq_len = 16
    c.trainer.checkpoint_dir = str(tmp_path / "ck")
    return c


def test_checkpoint_roundtrip_and_rotation(tmp_path):
    from oxidizr_b200.models import build_model
    from oxidizr_b200.optim import AdamW, AdamWConfig, FlatParams
    c = _cfg(tmp_path)
    m = build_model(c.model, "cpu", seed=1)
    opt = AdamW(FlatParams(list(m.named_parameters()), "cpu"), AdamWConfig(lr=1e-3))
    ids = torch.randint(0, c.model.vocab_size, (2, 17))
    loss, aux = m(ids[:, :-1], ids[:, 1:])
    loss.backward()
    opt.step()
    dpath = str(tmp_path / "d.bin")
    D.write_tokens(dpath, D.synthetic_tokens(c.model.vocab_size, 1000))
    for step in (10, 20, 30):
        C.save_checkpoint(m, opt, step, c.model, c.trainer.checkpoint_dir, dpath, max_checkpoints=2)
    files = sorted(os.listdir(c.trainer.checkpoint_dir))
    assert "checkpoint_step_10.meta.json" not in files and "checkpoint_step_30.meta.json" in files
    pre = c.model.checkpoint_prefix()
    assert f"{pre}_step_30.safetensors" in files and f"{pre}_step_30.optim.safetensors" in files
    assert f"{pre}_step_10.safetensors" not in files
    latest = C.find_latest_checkpoint(c.trainer.checkpoint_dir)
    assert latest[2] == 30
    meta = json.load(open(latest[1]))
    assert list(meta) == list(C.CheckpointMeta.FIELDS) and meta["step"] == 30 and meta["dtype"] == "f32"
    v = C.CheckpointMeta.load(latest[1]).validate(c.model, dpath)
    assert v["is_valid"]
    # upstream tensor names
    from safetensors.torch import load_file
    sd = load_file(latest[0])
    assert "layers.0.mamba2.mixer.A_log" in sd and "layers.3.self_attn.w_dkv.weight" in sd
    assert "layers.3.moe.experts.1.gate_proj.weight" in sd and "layers.3.moe.router.gate.weight" in sd
    # reload into a fresh model: identical next-step loss
    m2 = build_model(c.model, "cpu", seed=99)
    opt2 = AdamW(FlatParams(list(m2.named_parameters()), "cpu"), AdamWConfig(lr=1e-3))
    C.load_weights(m2, latest[0])
    C.load_optimizer_sidecar(opt2, latest[0])
    assert opt2.step_count == opt.step_count
    for (n1, p1), (n2, p2) in zip(m.named_parameters(), m2.named_parameters()):
        assert torch.equal(p1, p2), n1
    ids2 = torch.randint(0, c.model.vocab_size, (2, 17))
    l1, _ = m(ids2[:, :-1], ids2[:, 1:])
    l2, _ = m2(ids2[:, :-1], ids2[:, 1:])
    assert l1.item() == l2.item()
    # mismatched data -> invalid
    D.write_tokens(dpath, D.synthetic_tokens(c.model.vocab_size, 1000, seed=3))
    assert not C.CheckpointMeta.load(latest[1]).validate(c.model, dpath)["is_valid"]


def test_step_from_filename():
    assert C.step_from_filename("/a/nano_512_117m_bf16_step_100.safetensors") == 100
    assert C.step_from_filename("x_final.safetensors") == 0


def test_async_checkpoint_writes_the_state_of_the_save_call(tmp_path, monkeypatch):
    """A periodic checkpoint is written on a background thread from host copies taken when
    ``save`` is called: a training step that runs while the write is pending changes nothing
    in the files."""
    import threading
    from safetensors.torch import load_file
    from oxidizr_b200 import trainer as T
    from oxidizr_b200.config import LitConfig
    from oxidizr_b200.models import build_model
    from oxidizr_b200.optim import AdamW, AdamWConfig, FlatParams

    monkeypatch.delenv("OXI_SYNC_CHECKPOINT", raising=False)
    cfg = LitConfig.from_dict({"model": {
        "name": "asyncck", "hidden_size": 64, "num_layers": 1, "num_heads": 2, "kv_heads": 1,
        "intermediate_size": 128, "vocab_size": 97, "max_seq_len": 16, "rope_theta": 10000.0, "dtype": "f32"},
        "trainer": {"learning_rate": 1e-2, "batch_size": 2, "max_steps": 0, "num_epochs": 1,
                    "gradient_accumulation": 1, "checkpoint_dir": str(tmp_path / "ck"), "log_interval": 1,
                    "save_interval": 1000, "max_checkpoints": 2, "load_balance_alpha": 0.0, "group_size": 4,
                    "beta_kl": 0.0}})
    dev = torch.device("cpu")
    model = build_model(cfg.model, device=dev, seed=0)
    opt = AdamW(FlatParams(list(model.named_parameters()), dev), AdamWConfig(lr=1e-2))
    blk = torch.randint(0, 97, (2, 17), generator=torch.Generator().manual_seed(0))

    class Batches:
        batch_size, seq_len = 2, 16

        def dataset_size(self):
            return 10 ** 6

        def next_batch(self):
            return blk[:, :-1], blk[:, 1:]

    gate = threading.Event()
    real = T.save_checkpoint

    def slow_save(*a, **k):
        assert gate.wait(30)
        return real(*a, **k)

    monkeypatch.setattr(T, "save_checkpoint", slow_save)
    tr = T.Trainer(cfg, model, opt, Batches(), device=dev, out=lambda s: None)
    tr.training_step()
    at_save = {k: v.clone() for k, v in model.export_ref().items()}
    step_at_save = opt.step_count
    tr.save(1)
    assert tr._writer.busy
    tr.training_step()  # changes the parameters while the write waits
    assert any(not torch.equal(at_save[k], v) for k, v in model.export_ref().items())
    gate.set()
    tr.flush_checkpoints()
    path = os.path.join(cfg.trainer.checkpoint_dir, f"{cfg.model.checkpoint_prefix()}_step_1.safetensors")
    saved = load_file(path)
    assert set(saved) == set(at_save)
    assert all(torch.equal(saved[k], at_save[k]) for k in at_save)
    from safetensors import safe_open
    with safe_open(C.optim_sidecar_path(path), "pt") as fh:
        assert fh.metadata()["step"] == str(step_at_save)


def test_async_checkpoint_writer_reports_a_failed_write():
    w = C.AsyncCheckpointWriter()

    def boom():
        raise OSError("disk full")

    w.submit(boom)
    with pytest.raises(OSError, match="disk full"):
        w.wait()
    w.wait()  # reported once


def test_baseline_config1_cpu_checkpoint_roundtrip(tmp_path):
    """BASELINE.json config 1 (Llama decoder, CPU fp32: hidden 512, 8 layers, 8 / 4 heads of 64,
    SwiGLU 2048, vocab 128354, seq 512, batch 2, AdamW lr 3e-4, seeded uniform u32 tokens):
    train, save, load into a differently initialised model and optimizer, and check bitwise-equal
    parameters and the identical next-step loss."""
    from oxidizr_b200.models import build_model
    from oxidizr_b200.optim import AdamW, AdamWConfig, FlatParams
    from oxidizr_b200.trainer import Trainer

    cfg = LitConfig.from_dict({"model": {
        "name": "config1", "hidden_size": 512, "num_layers": 8, "num_heads": 8, "kv_heads": 4,
        "intermediate_size": 2048, "vocab_size": 128354, "max_seq_len": 512, "rope_theta": 10000.0, "dtype": "f32"},
        "trainer": {"learning_rate": 3e-4, "batch_size": 2, "max_steps": 20, "num_epochs": 1,
                    "gradient_accumulation": 1, "checkpoint_dir": str(tmp_path / "ck"), "log_interval": 1,
                    "save_interval": 1000, "load_balance_alpha": 0.0, "group_size": 4, "beta_kl": 0.0}})
    assert cfg.model.hidden_size // cfg.model.num_heads == 64
    dev = torch.device("cpu")
    toks = torch.from_numpy(D.synthetic_tokens(128354, 2 * 513 * 4, seed=11).astype(np.int64)).view(4, 2, 513)

    class Batches:
        batch_size, seq_len = 2, 512

        def __init__(self):
            self.i = 0

        def dataset_size(self):
            return 10 ** 9

        def next_batch(self):
            b = toks[self.i % 4]
            self.i += 1
            return b[:, :-1], b[:, 1:]

    def make(seed):
        model = build_model(cfg.model, device=dev, seed=seed)
        opt = AdamW(FlatParams(list(model.named_parameters()), dev), AdamWConfig(lr=3e-4))
        batches = Batches()
        return model, opt, batches, Trainer(cfg, model, opt, batches, device=dev, out=lambda s: None)

    model_a, opt_a, bat_a, tr_a = make(0)
    losses = [float(tr_a.training_step()[0]) for _ in range(3)]
    assert all(np.isfinite(losses)) and abs(losses[0] - np.log(128354)) < 1.0
    path = C.save_checkpoint(model_a, opt_a, 3, cfg.model, cfg.trainer.checkpoint_dir, None, 2)

    model_b, opt_b, bat_b, tr_b = make(123)
    C.load_weights(model_b, path)
    meta = C.load_optimizer_sidecar(opt_b, path)
    assert meta is not None and opt_b.step_count == 3
    for (n, pa), (_, pb) in zip(model_a.named_parameters(), model_b.named_parameters()):
        assert torch.equal(pa, pb), n
    bat_b.i = bat_a.i
    la, lb = float(tr_a.training_step()[0]), float(tr_b.training_step()[0])
    assert la == lb


def test_checkpoint_files_are_written_whole(tmp_path, monkeypatch):
    """A write that fails part way leaves no file under the real name (and no temporary file)."""
    import safetensors.torch as st
    path = str(tmp_path / "w.safetensors")
    real = st.save_file

    def failing(tensors, filename, metadata=None):
        with open(filename, "wb") as fh:
            fh.write(b"partial")
        raise OSError("disk full")

    monkeypatch.setattr(C, "save_file", failing)
    with pytest.raises(OSError):
        C._save_atomic({"a": torch.ones(3)}, path)
    assert os.listdir(tmp_path) == []
    monkeypatch.setattr(C, "save_file", real)
    C._save_atomic({"a": torch.ones(3)}, path)
    assert os.listdir(tmp_path) == ["w.safetensors"]


def test_host_copies_for_safetensors(tmp_path):
    """Views of one flat buffer are copied out, a tensor that owns its storage passes through once,
    a second name for it gets a copy, and the snapshot never aliases live tensors."""
    from safetensors.torch import load_file
    flat = torch.arange(12, dtype=torch.float32)
    own = torch.ones(3)
    sd = {"a": flat[:6].view(2, 3), "b": flat[6:], "own": own, "own_again": own}
    out = C._cpu_contig(sd)
    assert out["own"] is not None and out["own"].data_ptr() == own.data_ptr()
    assert out["own_again"].data_ptr() != own.data_ptr()
    assert out["a"].data_ptr() != flat.data_ptr() and out["b"].untyped_storage().nbytes() == 6 * 4
    path = str(tmp_path / "x.safetensors")
    C._save_atomic(out, path)
    back = load_file(path)
    assert all(torch.equal(back[k], sd[k]) for k in sd)
    snap = C.host_snapshot(sd)
    flat.add_(100.0)
    own.add_(1.0)
    assert torch.equal(snap["a"], torch.arange(6, dtype=torch.float32).view(2, 3))
    assert torch.equal(snap["own"], torch.ones(3))
