"""YAML model/trainer schema with the same required/optional/default rules as the
upstream serde structs.

Upstream: ``src/config.rs:16-72`` (ModelConfig), ``src/config.rs:172-198``
(TrainerConfig), ``src/distributed/sync.rs:13-86`` (DistributedConfig/SyncBackend),
``src/config.rs:525-636`` (BlazrConfig ``config.json``).

Rules reproduced here:

* a field without a default is required; a missing one raises ``ConfigError``;
* ``Option`` fields default to ``None`` and accept ``null``;
* keys that the schema does not know are ignored (serde's default);
* ``dtype`` accepts ``f32|f16|bf16`` (lowercase); ``target_device`` ``gpu|cpu``;
* ``validate`` enforces ``hidden_size * mamba2_expand == mamba2_num_heads * mamba2_head_dim``.

Extensions (all optional, ignored by the upstream parser because serde skips
unknown keys): ``num_shared_experts``, ``init_std``, ``seed``, ``compat``,
``ep_size``, ``moe_aux_loss``.  They are NOT part of the model-config hash, so a
config without them hashes exactly like upstream.
"""
from __future__ import annotations

import dataclasses
import json
import math
import sys
from dataclasses import dataclass, field
from typing import Any, List, Optional

import yaml


class ConfigError(ValueError):
    pass


DTYPES = ("f32", "f16", "bf16")
_DTYPE_ALIASES = {
    "f32": "f32", "fp32": "f32", "float32": "f32",
    "f16": "f16", "fp16": "f16", "float16": "f16",
    "bf16": "bf16", "bfloat16": "bf16",
}


def parse_dtype(s: str) -> Optional[str]:
    """CLI dtype parser (``DTypePrecision::from_str``, config.rs:104-111)."""
    return _DTYPE_ALIASES.get(str(s).lower())


def torch_dtype(s: str):
    import torch
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[s]


SYNC_BACKENDS = ("single", "cpustaging", "nccl", "nccl_sharded", "fused")


def parse_sync_backend(s: str) -> str:
    """``SyncBackend::from_str`` (sync.rs:25-35) plus the ``fused`` NVLink backend."""
    v = str(s).lower()
    if v in ("single", "none"):
        return "single"
    if v in ("cpu", "cpu_staging", "cpustaging"):
        return "cpustaging"
    if v == "nccl":
        return "nccl"
    if v in ("nccl_sharded", "nccl-sharded"):
        return "nccl_sharded"
    if v == "fused":
        return "fused"
    raise ConfigError(f"Unknown sync backend: {s}. Valid options: single, cpu, nccl, nccl_sharded, fused")


_REQUIRED = object()


def _f(default=_REQUIRED, *, kind=None):
    md = {"kind": kind}
    if default is _REQUIRED:
        return field(default=None, metadata={**md, "required": True})
    return field(default=default, metadata={**md, "required": False})


@dataclass
class ModelConfig:
    # Order of fields == upstream struct order (it determines the hash JSON).
    name: str = _f("model", kind=str)
    hidden_size: int = _f(kind=int)
    num_layers: int = _f(kind=int)
    num_heads: int = _f(kind=int)
    kv_heads: Optional[int] = _f(None, kind=int)
    kv_latent_dim: Optional[int] = _f(None, kind=int)
    q_latent_dim: Optional[int] = _f(None, kind=int)
    d_rope: Optional[int] = _f(None, kind=int)
    num_experts: Optional[int] = _f(None, kind=int)
    experts_per_tok: Optional[int] = _f(None, kind=int)
    shared_expert_enabled: Optional[bool] = _f(None, kind=bool)
    intermediate_size: Optional[int] = _f(None, kind=int)
    mamba_layers: Optional[List[int]] = _f(None, kind=list)
    mamba2_num_heads: Optional[int] = _f(None, kind=int)
    mamba2_head_dim: Optional[int] = _f(None, kind=int)
    mamba2_state_size: Optional[int] = _f(None, kind=int)
    mamba2_chunk_size: Optional[int] = _f(None, kind=int)
    mamba2_n_groups: Optional[int] = _f(None, kind=int)
    mamba2_conv_kernel: Optional[int] = _f(None, kind=int)
    mamba2_expand: Optional[int] = _f(None, kind=int)
    mamba3_enabled: Optional[bool] = _f(None, kind=bool)
    mamba3_complex_rope: Optional[bool] = _f(None, kind=bool)
    mamba3_mimo_rank: Optional[int] = _f(None, kind=int)
    mamba3_use_conv: Optional[bool] = _f(None, kind=bool)
    vocab_size: int = _f(kind=int)
    max_seq_len: int = _f(kind=int)
    rope_theta: float = _f(kind=float)
    dtype: str = _f("f32", kind="dtype")
    # ---- extensions (not hashed) ----
    num_shared_experts: Optional[int] = _f(None, kind=int)
    init_std: Optional[float] = _f(None, kind=float)
    seed: Optional[int] = _f(None, kind=int)
    compat: Optional[str] = _f(None, kind=str)
    ep_size: Optional[int] = _f(None, kind=int)
    moe_aux_loss: Optional[str] = _f(None, kind=str)

    UPSTREAM_FIELDS = (
        "name", "hidden_size", "num_layers", "num_heads", "kv_heads", "kv_latent_dim",
        "q_latent_dim", "d_rope", "num_experts", "experts_per_tok", "shared_expert_enabled",
        "intermediate_size", "mamba_layers", "mamba2_num_heads", "mamba2_head_dim",
        "mamba2_state_size", "mamba2_chunk_size", "mamba2_n_groups", "mamba2_conv_kernel",
        "mamba2_expand", "mamba3_enabled", "mamba3_complex_rope", "mamba3_mimo_rank",
        "mamba3_use_conv", "vocab_size", "max_seq_len", "rope_theta", "dtype",
    )

    # -------- derived helpers --------
    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def n_shared_experts(self) -> int:
        return 1 if self.num_shared_experts is None else int(self.num_shared_experts)

    @property
    def std(self) -> float:
        return 0.02 if self.init_std is None else float(self.init_std)

    @property
    def reference_compat(self) -> bool:
        return (self.compat or "").lower() == "reference"

    def layer_kind(self, i: int) -> str:
        """Per-layer block type (model.rs:795-870), plus the GQA+MoE extension.

        Returns one of ``mamba3``, ``mamba2``, ``mamba1``, ``mla_moe``, ``gqa_moe``, ``gqa_mlp``.
        """
        is_mamba = bool(self.mamba_layers) and i in self.mamba_layers
        use_m3 = bool(self.mamba3_enabled)
        use_m2 = self.mamba2_num_heads is not None
        if is_mamba and use_m3 and use_m2:
            return "mamba3"
        if is_mamba and use_m2:
            return "mamba2"
        if is_mamba:
            return "mamba1"
        if self.kv_latent_dim is not None:
            return "mla_moe"
        if self.num_experts is not None and self.experts_per_tok is not None and self.kv_heads is not None:
            return "gqa_moe"
        return "gqa_mlp"

    def checkpoint_prefix(self) -> str:
        """``{name}_{seq}_{params}_{dtype}`` (config.rs:126-134)."""
        return f"{self.name.lower()}_{self.max_seq_len}_{self.estimate_params_short()}_{self.dtype.lower()}"

    def _dense_param_estimate(self) -> int:
        hd = self.hidden_size // self.num_heads
        kvh = self.kv_heads if self.kv_heads is not None else self.num_heads
        kv = kvh * hd
        inter = self.intermediate_size if self.intermediate_size is not None else self.hidden_size * 4
        h = self.hidden_size
        embed = self.vocab_size * h
        attn = h * h + h * kv + h * kv + h * h
        mlp = h * inter * 3
        layer = attn + mlp + 2 * h
        head = h * self.vocab_size + h
        return embed + self.num_layers * layer + head

    def estimate_params_short(self) -> str:
        """Dense-GQA estimate used only in names (config.rs:137-168)."""
        total = self._dense_param_estimate()
        if total >= 1_000_000_000:
            return f"{total / 1e9:.1f}b"
        return f"{total // 1_000_000}m"

    def estimate_params_banner(self) -> str:
        """Banner format (commands/train.rs:172-220)."""
        total = self._dense_param_estimate()
        if total > 1_000_000_000:
            return f"{total / 1e9:.2f}B"
        if total > 1_000_000:
            return f"{total / 1e6:.2f}M"
        return f"{total // 1000}K"

    def upstream_dict(self) -> dict:
        return {k: getattr(self, k) for k in self.UPSTREAM_FIELDS}


@dataclass
class DistributedConfig:
    enabled: bool = _f(False, kind=bool)
    backend: str = _f("single", kind="backend")
    gpu_ids: List[int] = _f(None, kind=list)

    def __post_init__(self):
        if self.gpu_ids is None:
            self.gpu_ids = []

    def world_size(self) -> int:
        return max(len(self.gpu_ids), 1)


@dataclass
class TrainerConfig:
    learning_rate: float = _f(kind=float)
    batch_size: int = _f(kind=int)
    max_steps: int = _f(kind=int)
    num_epochs: int = _f(kind=int)
    gradient_accumulation: int = _f(kind=int)
    checkpoint_dir: str = _f(kind=str)
    log_interval: int = _f(kind=int)
    save_interval: int = _f(kind=int)
    max_checkpoints: int = _f(10, kind=int)
    load_balance_alpha: float = _f(kind=float)
    target_device: str = _f("gpu", kind="device")
    distributed: DistributedConfig = _f(None, kind=DistributedConfig)
    group_size: int = _f(kind=int)
    beta_kl: float = _f(kind=float)
    # ---- extensions ----
    weight_decay: Optional[float] = _f(None, kind=float)
    max_grad_norm: Optional[float] = _f(None, kind=float)

    def __post_init__(self):
        if self.distributed is None:
            self.distributed = DistributedConfig()


def _coerce(name: str, kind, v: Any, where: str):
    if v is None:
        return None
    if kind is int:
        if isinstance(v, bool) or not isinstance(v, int):
            raise ConfigError(f"{where}.{name}: invalid type: expected an integer, got {v!r}")
        if v < 0:
            raise ConfigError(f"{where}.{name}: invalid value: {v}, expected usize")
        return v
    if kind is float:
        if isinstance(v, bool) or not isinstance(v, (int, float)):
            raise ConfigError(f"{where}.{name}: invalid type: expected a number, got {v!r}")
        return float(v)
    if kind is bool:
        if not isinstance(v, bool):
            raise ConfigError(f"{where}.{name}: invalid type: expected a boolean, got {v!r}")
        return v
    if kind is str:
        if not isinstance(v, str):
            raise ConfigError(f"{where}.{name}: invalid type: expected a string, got {v!r}")
        return v
    if kind is list:
        if not isinstance(v, list) or not all(isinstance(x, int) and not isinstance(x, bool) for x in v):
            raise ConfigError(f"{where}.{name}: invalid type: expected a sequence of integers")
        return list(v)
    if kind == "dtype":
        if v not in DTYPES:
            raise ConfigError(f"{where}.{name}: unknown variant `{v}`, expected one of `f32`, `f16`, `bf16`")
        return v
    if kind == "device":
        if v not in ("gpu", "cpu"):
            raise ConfigError(f"{where}.{name}: unknown variant `{v}`, expected `gpu` or `cpu`")
        return v
    if kind == "backend":
        # serde: rename_all lowercase + alias "cpu"
        if v == "cpu":
            return "cpustaging"
        if v not in ("single", "cpustaging", "nccl", "fused"):
            raise ConfigError(f"{where}.{name}: unknown variant `{v}`")
        return v
    if kind is DistributedConfig:
        if not isinstance(v, dict):
            raise ConfigError(f"{where}.{name}: expected a mapping")
        return _build(DistributedConfig, v, f"{where}.{name}")
    raise AssertionError(kind)


def _build(cls, d: dict, where: str):
    if not isinstance(d, dict):
        raise ConfigError(f"{where}: expected a mapping")
    kwargs = {}
    for f_ in dataclasses.fields(cls):
        md = f_.metadata
        if f_.name in d:
            val = d[f_.name]
            if val is None and md.get("required"):
                raise ConfigError(f"{where}.{f_.name}: invalid type: null")
            kwargs[f_.name] = _coerce(f_.name, md.get("kind"), val, where)
            if kwargs[f_.name] is None and not md.get("required") and f_.default is not None:
                # serde(default) fields do not accept null either
                raise ConfigError(f"{where}.{f_.name}: invalid type: null")
        elif md.get("required"):
            raise ConfigError(f"{where}: missing field `{f_.name}`")
    return cls(**kwargs)


@dataclass
class LitConfig:
    model: ModelConfig
    trainer: TrainerConfig

    @staticmethod
    def from_dict(d: dict) -> "LitConfig":
        if not isinstance(d, dict):
            raise ConfigError("config: expected a mapping")
        if "model" not in d:
            raise ConfigError("missing field `model`")
        if "trainer" not in d:
            raise ConfigError("missing field `trainer`")
        cfg = LitConfig(_build(ModelConfig, d["model"], "model"),
                        _build(TrainerConfig, d["trainer"], "trainer"))
        cfg.validate()
        return cfg

    @staticmethod
    def from_yaml_str(text: str) -> "LitConfig":
        return LitConfig.from_dict(yaml.safe_load(text))

    @staticmethod
    def from_yaml(path: str) -> "LitConfig":
        with open(path, "r") as fh:
            return LitConfig.from_yaml_str(fh.read())

    def validate(self) -> None:
        """config.rs:229-266."""
        m = self.model
        if m.mamba2_num_heads is not None and m.mamba2_head_dim is not None and m.mamba2_expand is not None:
            expected = m.mamba2_num_heads * m.mamba2_head_dim
            actual = m.hidden_size * m.mamba2_expand
            if actual != expected:
                raise ConfigError(
                    f"Mamba2 config invalid: hidden_size * expand ({actual}) != num_heads * head_dim ({expected})")
        if m.mamba_layers and m.mamba2_num_heads is None:
            print("WARNING: Using Mamba-1 (sequential SSM) layers; Mamba-2 (SSD) needs mamba2_* fields.",
                  file=sys.stderr)
        if m.hidden_size % m.num_heads != 0:
            raise ConfigError("hidden_size must be divisible by num_heads")


# ---------------------------------------------------------------------------
# serde_json compatible serialisation (used by the config hash and config.json)
# ---------------------------------------------------------------------------

def _ryu_like_f32(x: float) -> str:
    """Format an f32 the way serde_json (ryu) does: shortest round-trip digits,
    plain notation for decimal exponents in (-6, 21], scientific otherwise."""
    import numpy as np
    if math.isnan(x) or math.isinf(x):
        return "null"
    v = np.float32(x)
    if v == 0:
        return "-0.0" if math.copysign(1.0, float(v)) < 0 else "0.0"
    s = np.format_float_scientific(v, unique=True, trim="-")  # e.g. '1.e+04' / '1.5e-07'
    mant, exp = s.split("e")
    neg = mant.startswith("-")
    mant = mant.lstrip("-")
    digits = mant.replace(".", "").rstrip("0") or "0"
    e = int(exp)
    return ("-" if neg else "") + _ryu_layout(digits, e)


def _ryu_layout(digits: str, e: int, max_int_digits: int = 16) -> str:
    # digits d1d2...dn with value d1.d2..dn * 10^e; kk = position of the decimal point.
    # ryu's "pretty" layout uses 16 as the plain-notation limit for f64 and 13 for f32.
    n = len(digits)
    kk = e + 1
    k = kk - n
    if 0 <= k and kk <= max_int_digits:
        return digits + "0" * k + ".0"
    if 0 < kk <= max_int_digits:
        return digits[:kk] + "." + digits[kk:]
    if -5 < kk <= 0:
        return "0." + "0" * (-kk) + digits
    if n == 1:
        return f"{digits}e{kk - 1}"
    return f"{digits[0]}.{digits[1:]}e{kk - 1}"


def _ryu_like_f64(x: float) -> str:
    if math.isnan(x) or math.isinf(x):
        return "null"
    if x == 0:
        return "-0.0" if math.copysign(1.0, x) < 0 else "0.0"
    r = repr(float(x))
    neg = r.startswith("-")
    r = r.lstrip("-")
    if "e" in r:
        mant, exp = r.split("e")
        e = int(exp)
    else:
        mant, e = r, 0
    if "." in mant:
        ip, fp = mant.split(".")
    else:
        ip, fp = mant, ""
    digits = (ip + fp).lstrip("0")
    # exponent of the first significant digit
    if ip.strip("0"):
        e1 = len(ip.lstrip("0")) - 1 + e
    else:
        lead = len(fp) - len(fp.lstrip("0"))
        e1 = -lead - 1 + e
    digits = digits.rstrip("0") or "0"
    return ("-" if neg else "") + _ryu_layout(digits, e1)


def serde_json_dumps(obj, *, f32_keys=(), pretty=False, _indent=0) -> str:
    """Minimal serde_json serializer: compact (``to_string``) or pretty
    (``to_string_pretty``: two-space indent, ``": "`` separators)."""
    def enc(o, key=None, ind=0):
        if o is None:
            return "null"
        if o is True:
            return "true"
        if o is False:
            return "false"
        if isinstance(o, int):
            return str(o)
        if isinstance(o, float):
            return _ryu_like_f32(o) if key in f32_keys else _ryu_like_f64(o)
        if isinstance(o, str):
            return json.dumps(o, ensure_ascii=False)
        if isinstance(o, (list, tuple)):
            if not o:
                return "[]"
            if pretty:
                pad = "  " * (ind + 1)
                return "[\n" + ",\n".join(pad + enc(x, None, ind + 1) for x in o) + "\n" + "  " * ind + "]"
            return "[" + ",".join(enc(x, None, ind) for x in o) + "]"
        if isinstance(o, dict):
            if not o:
                return "{}"
            if pretty:
                pad = "  " * (ind + 1)
                return "{\n" + ",\n".join(
                    pad + json.dumps(k) + ": " + enc(v, k, ind + 1) for k, v in o.items()) + "\n" + "  " * ind + "}"
            return "{" + ",".join(json.dumps(k) + ":" + enc(v, k, ind) for k, v in o.items()) + "}"
        raise TypeError(type(o))
    return enc(obj, None, _indent)


def model_config_json(m: ModelConfig) -> str:
    """``serde_json::to_string(&ModelConfig)`` over the upstream fields."""
    return serde_json_dumps(m.upstream_dict(), f32_keys=("rope_theta",))


# ---------------------------------------------------------------------------
# BlazrConfig (config.json for the inference server)
# ---------------------------------------------------------------------------

def blazr_config(m: ModelConfig) -> dict:
    """``BlazrConfig::from_model_config`` (config.rs:587-628) with
    ``skip_serializing_if`` applied (None / empty vec omitted)."""
    d = {
        "hidden_size": m.hidden_size,
        "num_layers": m.num_layers,
        "vocab_size": m.vocab_size,
        "mamba2_num_heads": m.mamba2_num_heads,
        "mamba2_head_dim": m.mamba2_head_dim,
        "mamba2_state_size": m.mamba2_state_size,
        "mamba2_chunk_size": m.mamba2_chunk_size,
        "mamba2_expand": m.mamba2_expand,
        "mamba2_conv_kernel": m.mamba2_conv_kernel,
        "mamba3_enabled": m.mamba3_enabled,
        "mamba3_complex_rope": m.mamba3_complex_rope,
        "mamba3_mimo_rank": m.mamba3_mimo_rank,
        "mamba3_use_conv": m.mamba3_use_conv,
        "num_attention_heads": m.num_heads,
        "kv_latent_dim": m.kv_latent_dim,
        "q_latent_dim": m.q_latent_dim,
        "d_rope": m.d_rope,
        "num_experts": m.num_experts,
        "experts_per_tok": m.experts_per_tok,
        "shared_expert_enabled": m.shared_expert_enabled,
        "intermediate_size": m.intermediate_size,
        "mamba_layers": list(m.mamba_layers or []),
        "rms_norm_eps": 1e-5,
        "max_seq_len": m.max_seq_len,
    }
    out = {}
    for k, v in d.items():
        if v is None:
            continue
        if k == "mamba_layers" and not v:
            continue
        out[k] = v
    return out


def blazr_config_json(m: ModelConfig) -> str:
    return serde_json_dumps(blazr_config(m), pretty=True)
