"""Checkpoint tensor names and shapes per block type, as the upstream VarBuilder prefixes make
them (model.rs:320-323,442-444,517-530,856-866,964-972; mamba.rs:71-97; mamba2.rs:263-300,768;
mamba3.rs:303-378,959), and a bitwise export -> import round trip into a differently seeded model."""
import pytest
import torch

from oxidizr_b200.config import LitConfig
from oxidizr_b200.models import build_model

BASE = {"name": "names", "hidden_size": 64, "num_layers": 2, "num_heads": 4, "kv_heads": 2, "intermediate_size": 128,
        "vocab_size": 97, "max_seq_len": 16, "rope_theta": 1e4, "dtype": "f32"}
TRAINER = {"learning_rate": 1e-3, "batch_size": 1, "max_steps": 0, "num_epochs": 1, "gradient_accumulation": 1,
           "checkpoint_dir": "unused", "log_interval": 1, "save_interval": 10, "load_balance_alpha": 0.0,
           "group_size": 4, "beta_kl": 0.0}
M2 = {"mamba2_num_heads": 4, "mamba2_head_dim": 32, "mamba2_state_size": 16, "mamba2_chunk_size": 8,
      "mamba2_expand": 2, "mamba2_conv_kernel": 4, "mamba2_n_groups": 1}

GQA = {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
       "input_layernorm.weight", "post_attention_layernorm.weight"}
MLP = {"mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"}
MLA = {f"self_attn.{n}.weight" for n in ("w_dkv", "w_dq", "w_uq", "w_uk", "w_uv", "w_qr", "w_kr", "o_proj")} | {
    "input_layernorm.weight", "post_attention_layernorm.weight"}


def moe(E):
    s = {"moe.router.gate.weight"} | {f"moe.shared_expert.{p}.weight" for p in ("gate_proj", "up_proj", "down_proj")}
    return s | {f"moe.experts.{e}.{p}.weight" for e in range(E) for p in ("gate_proj", "up_proj", "down_proj")}


MAMBA1 = {f"mamba.{n}" for n in ("in_proj.weight", "conv1d.weight", "conv1d.bias", "x_proj.weight", "dt_proj.weight",
                                 "dt_proj.bias", "a_log", "d", "out_proj.weight")} | {"norm.weight"}
MAMBA2 = {"mamba2.norm.weight", "mamba2.norm.bias"} | {f"mamba2.mixer.{n}" for n in (
    "in_proj.weight", "in_proj.bias", "conv1d.weight", "conv1d.bias", "dt_bias", "A_log", "D", "norm.weight",
    "out_proj.weight", "out_proj.bias")}


def mamba3(rope, conv, mimo):
    n = {"in_proj.weight", "in_proj.bias", "out_proj.weight", "out_proj.bias", "lambda_proj.weight",
         "lambda_proj.bias", "b_bias", "c_bias", "dt_bias", "A_log", "D", "bc_norm.weight", "norm.weight"}
    if rope:
        n |= {"theta_proj.weight", "theta_proj.bias"}
    if conv:
        n |= {"conv1d.weight", "conv1d.bias"}
    if mimo:
        n |= {"mimo_x_up.weight", "mimo_x_up.bias", "mimo_x_down.weight", "mimo_x_down.bias"}
    return {"mamba3.norm.weight", "mamba3.norm.bias"} | {f"mamba3.mixer.{k}" for k in n}


CASES = {
    "gqa_mlp": ({}, [GQA | MLP, GQA | MLP]),
    "mla_moe_and_mamba2": (dict(M2, mamba_layers=[1], kv_latent_dim=32, q_latent_dim=48, d_rope=8, num_experts=3,
                                experts_per_tok=2), [MLA | moe(3), MAMBA2]),
    "gqa_moe_two_shared": ({"num_experts": 5, "experts_per_tok": 2, "num_shared_experts": 2}, [GQA | moe(5)] * 2),
    "mamba1": ({"mamba_layers": [0]}, [MAMBA1, GQA | MLP]),
    "mamba3_rope_conv_mimo": (dict(M2, mamba_layers=[0, 1], mamba3_enabled=True, mamba3_complex_rope=True,
                                   mamba3_use_conv=True, mamba3_mimo_rank=2), [mamba3(True, True, True)] * 2),
    "mamba3_plain": (dict(M2, mamba_layers=[0], mamba3_enabled=True, mamba3_complex_rope=False,
                          mamba3_use_conv=False), [mamba3(False, False, False), GQA | MLP]),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_names_shapes_and_roundtrip(case):
    extra, layers = CASES[case]
    cfg = LitConfig.from_dict({"model": dict(BASE, **extra), "trainer": TRAINER}).model
    a = build_model(cfg, device=torch.device("cpu"), seed=0)
    sd = a.export_ref()
    want = {"embed_tokens.weight", "norm.weight", "lm_head.weight"}
    for i, names in enumerate(layers):
        want |= {f"layers.{i}.{n}" for n in names}
    assert set(sd) == want, (sorted(set(sd) - want), sorted(want - set(sd)))
    H, V = BASE["hidden_size"], BASE["vocab_size"]
    assert sd["embed_tokens.weight"].shape == (V, H) and sd["lm_head.weight"].shape == (V, H)
    assert sd["norm.weight"].shape == (H,)
    if case == "mamba1":
        assert sd["layers.0.mamba.conv1d.weight"].shape == (2 * H, 1, 4)
        assert sd["layers.0.mamba.a_log"].shape == (2 * H, 16) and sd["layers.0.mamba.d"].shape == (2 * H,)
    if case.startswith("mamba3"):
        assert sd["layers.0.mamba3.mixer.b_bias"].shape == (4, 16)
        assert sd["layers.0.mamba3.mixer.bc_norm.weight"].shape == (16,)
    if case == "mla_moe_and_mamba2":
        assert sd["layers.0.moe.router.gate.weight"].shape == (3, H)
        assert sd["layers.1.mamba2.mixer.A_log"].shape == (4,)
    b = build_model(cfg, device=torch.device("cpu"), seed=1)
    assert any(not torch.equal(sd[k], v) for k, v in b.export_ref().items())
    b.import_ref({k: v.clone() for k, v in sd.items()})
    sb = b.export_ref()
    assert all(torch.equal(sd[k], sb[k]) for k in sd)
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.equal(pa, pb), n
