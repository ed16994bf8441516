"""Config schema (serde semantics), hashing, naming and serialisation formats."""
import json
import os

import pytest

from oxidizr_b200.config import (ConfigError, LitConfig, blazr_config, blazr_config_json, model_config_json,
                                 parse_dtype, parse_sync_backend, serde_json_dumps)
from oxidizr_b200.utils.hashing import compute_file_hash, rust_default_hash_str, siphash

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

MIN = """
model:
  hidden_size: 64
  num_layers: 2
  num_heads: 4
  vocab_size: 100
  max_seq_len: 32
  rope_theta: 10000.0
trainer:
  learning_rate: 0.001
  batch_size: 2
  max_steps: 5
  num_epochs: 1
  gradient_accumulation: 1
  checkpoint_dir: /tmp/x
  log_interval: 1
  save_interval: 10
  load_balance_alpha: 0.0
  group_size: 4
  beta_kl: 0.04
"""


def test_defaults_and_unknown_keys():
    c = LitConfig.from_yaml_str(MIN + "  unknown_key: 5\n")
    assert c.model.name == "model" and c.model.dtype == "f32"
    assert c.trainer.max_checkpoints == 10 and c.trainer.target_device == "gpu"
    assert c.trainer.distributed.enabled is False and c.trainer.distributed.backend == "single"
    assert c.model.kv_heads is None


@pytest.mark.parametrize("field", ["hidden_size", "vocab_size", "rope_theta"])
def test_required_model_fields(field):
    text = "\n".join(l for l in MIN.splitlines() if not l.strip().startswith(field + ":"))
    with pytest.raises(ConfigError, match=field):
        LitConfig.from_yaml_str(text)


@pytest.mark.parametrize("field", ["load_balance_alpha", "group_size", "beta_kl"])
def test_required_trainer_fields(field):
    # upstream README examples omit these and fail to parse (no serde default)
    text = "\n".join(l for l in MIN.splitlines() if not l.strip().startswith(field + ":"))
    with pytest.raises(ConfigError, match=field):
        LitConfig.from_yaml_str(text)


def test_type_and_variant_errors():
    with pytest.raises(ConfigError):
        LitConfig.from_yaml_str(MIN.replace("hidden_size: 64", "hidden_size: 64.5"))
    with pytest.raises(ConfigError):
        LitConfig.from_yaml_str(MIN.replace("  rope_theta: 10000.0", "  rope_theta: 10000.0\n  dtype: fp8"))
    c = LitConfig.from_yaml_str(MIN.replace("  rope_theta: 10000.0", "  rope_theta: 10000.0\n  dtype: bf16"))
    assert c.model.dtype == "bf16"


def test_mamba2_constraint():
    bad = MIN.replace("  max_seq_len: 32", "  max_seq_len: 32\n  mamba2_num_heads: 3\n  mamba2_head_dim: 16\n"
                                          "  mamba2_expand: 2")
    with pytest.raises(ConfigError, match="Mamba2 config invalid"):
        LitConfig.from_yaml_str(bad)


def test_distributed_backend_alias():
    c = LitConfig.from_yaml_str(MIN + "  distributed:\n    enabled: true\n    backend: cpu\n    gpu_ids: [0, 1]\n")
    assert c.trainer.distributed.backend == "cpustaging" and c.trainer.distributed.world_size() == 2
    assert parse_sync_backend("CPU_STAGING") == "cpustaging"
    assert parse_sync_backend("none") == "single"
    with pytest.raises(ConfigError):
        parse_sync_backend("mpi")
    assert parse_dtype("BFloat16") == "bf16" and parse_dtype("x") is None


def test_all_example_configs_parse():
    import glob
    files = sorted(glob.glob(os.path.join(REPO, "models", "*.yaml")))
    assert len(files) >= 6
    kinds = set()
    for f in files:
        c = LitConfig.from_yaml(f)
        kinds |= {c.model.layer_kind(i) for i in range(c.model.num_layers)}
    assert {"mamba2", "mamba3", "mla_moe"} <= kinds


def test_checkpoint_prefix_and_estimate():
    c = LitConfig.from_yaml(os.path.join(REPO, "models", "nano.yaml"))
    assert c.model.checkpoint_prefix() == "nano_512_117m_f32"
    c.model.hidden_size, c.model.num_layers, c.model.intermediate_size = 2048, 16, 5632
    c.model.num_heads, c.model.kv_heads = 16, 8
    assert c.model.estimate_params_short() == "1.3b"


def test_siphash_paper_vectors():
    k0 = int.from_bytes(bytes(range(8)), "little")
    k1 = int.from_bytes(bytes(range(8, 16)), "little")
    assert siphash(b"", k0, k1, 2, 4) == 0x726FDB47DD0E0E31
    assert siphash(bytes(range(15)), k0, k1, 2, 4) == 0xA129CA6149BE45E5
    # streaming equivalence across the 8-byte block boundary
    assert siphash(b"a" * 16) != siphash(b"a" * 17)


def test_model_config_json_and_hash_stable():
    c = LitConfig.from_yaml(os.path.join(REPO, "models", "nano.yaml"))
    js = model_config_json(c.model)
    assert js.startswith('{"name":"nano","hidden_size":384,')
    assert '"rope_theta":10000.0,"dtype":"f32"}' in js
    assert '"kv_heads":null' in js and '"mamba_layers":[0,1,2,4,5,6]' in js
    # extension fields do not change the hash
    from oxidizr_b200.utils.hashing import compute_model_config_hash
    h1 = compute_model_config_hash(c.model)
    c.model.num_shared_experts = 2
    assert compute_model_config_hash(c.model) == h1
    assert len(h1) == 16 and int(h1, 16) == rust_default_hash_str(js)


def test_file_hash(tmp_path):
    p = tmp_path / "t.bin"
    p.write_bytes(b"\x01\x02\x03\x04" * 10)
    h = compute_file_hash(str(p))
    import struct
    data = struct.pack("<Q", 40) + p.read_bytes() + struct.pack("<Q", 40)
    assert h == f"{siphash(data):016x}"


def test_blazr_config_skips_none():
    c = LitConfig.from_yaml(os.path.join(REPO, "models", "nano.yaml"))
    d = blazr_config(c.model)
    assert "mamba3_enabled" not in d and d["num_attention_heads"] == 6 and d["rms_norm_eps"] == 1e-5
    js = blazr_config_json(c.model)
    assert json.loads(js) == d
    assert '  "rms_norm_eps": 0.00001,' in js


def test_serde_json_float_formatting():
    assert serde_json_dumps({"a": 1e-5}) == '{"a":0.00001}'
    assert serde_json_dumps({"a": 3e-4, "b": 1.0, "c": 1e21}) == '{"a":0.0003,"b":1.0,"c":1e21}'


def test_rust_exp_format():
    from oxidizr_b200.trainer import format_duration, rust_exp
    assert rust_exp(3e-4) == "3.000000e-4"
    assert rust_exp(0.002) == "2.000000e-3"
    assert rust_exp(12.5) == "1.250000e1"
    assert format_duration(59) == "59s" and format_duration(61) == "1m01s" and format_duration(3700) == "1h01m"
