"""Architecture descriptors and composed-checkpoint validation (CPU)."""
import pytest
import torch

from granite_switch_b200.checkpoint import save_state_dict
from granite_switch_b200.composer.arch import resolve_arch
from granite_switch_b200.composer.compose import compose_checkpoint
from granite_switch_b200.composer.synthetic import base_config, compose_synthetic, random_base_state, synthetic_adapters
from granite_switch_b200.composer.validators import (
    audit_saved_checkpoint,
    validate_cross_stream_population,
    validate_parameters,
)


def test_resolve_arch_families():
    dense = resolve_arch({"model_type": "granite"})
    assert dense.group_names == ["qkv_proj", "o_proj", "shared_input_linear", "shared_output_linear"]
    assert dense.group_of("up_proj")[0].name == "shared_input_linear" and dense.group_of("up_proj")[1] == 1
    hybrid = resolve_arch({"model_type": "granitemoehybrid", "num_local_experts": 8, "shared_intermediate_size": 64})
    assert hybrid.experts and hybrid.shared_mlp and hybrid.group_of("input_linear")[1] == -1
    moe = resolve_arch({"model_type": "granitemoe", "num_local_experts": 8})
    assert moe.group_names == ["qkv_proj", "o_proj"] and not moe.shared_mlp
    with pytest.raises(ValueError):
        moe.check_adapter_modules("x", {"q_proj", "gate_proj"})
    sr = resolve_arch({"model_type": "granite_switch"}, dual_stream=True)
    assert sr.group_names[-1] == "cross_stream" and sr.shadow_residual
    with pytest.raises(ValueError):
        resolve_arch({"model_type": "llama"})


def _compose(tmp_path, **kw):
    out = str(tmp_path / "ckpt")
    config = compose_synthetic(out, "tiny", num_adapters=2, rank=8, targets=("q", "k", "v", "o"), **kw)
    from granite_switch_b200.checkpoint import load_state_dict

    return out, config, load_state_dict(out)


def test_compose_records_validation(tmp_path):
    _, config, sd = _compose(tmp_path)
    v = config.compose_validation
    assert v["arch"] == "granite" and v["saved_tensors"] == len(sd)
    assert v["layers_populated"]["adapter_0"]["qkv_proj"] == config.num_decoder_layers


def test_validation_catches_broken_tensors(tmp_path):
    cfg = base_config("tiny")
    base = random_base_state(cfg, seed=0)
    ads = synthetic_adapters(cfg, 2, 8, ("q", "v"), seed=1)
    out = str(tmp_path / "ok")
    config = compose_checkpoint(cfg, base, ads, out, dtype=torch.float32)
    from granite_switch_b200.checkpoint import load_state_dict

    sd = load_state_dict(out)
    arch = resolve_arch(cfg)
    validate_parameters(sd, config, arch, ads, cfg)
    bad = dict(sd)
    bad["model.norm.weight"] = torch.full_like(sd["model.norm.weight"], float("nan"))
    with pytest.raises(ValueError, match="non-finite"):
        validate_parameters(bad, config, arch, ads, cfg)
    bad = dict(sd)
    del bad["model.layers.0.input_layernorm.weight"]
    with pytest.raises(ValueError, match="missing"):
        validate_parameters(bad, config, arch, ads, cfg)
    # the adapters train q and v: a populated k slice is a transfer bug ...
    bad = dict(sd)
    for n in ("lora_A_slices.1", "lora_B_slices.1"):
        key = f"model.layers.0.self_attn.qkv_proj.{n}"
        bad[key] = sd[key].clone()
        bad[key][1] = 1.0
    with pytest.raises(ValueError, match=r"qkv_proj\[1\] populated in layers \[0\]"):
        validate_parameters(bad, config, arch, ads, cfg)
    # ... and so is an all-zero slice of a trained module
    bad = dict(sd)
    key = "model.layers.1.self_attn.qkv_proj.lora_B_slices.2"
    bad[key] = torch.zeros_like(sd[key])
    with pytest.raises(ValueError, match=r"qkv_proj\[2\] is trained but all zero in layers \[1\]"):
        validate_parameters(bad, config, arch, ads, cfg)
    # on-disk audit
    assert audit_saved_checkpoint(out, sd) == len(sd)
    save_state_dict({k: v for k, v in sd.items() if k != "model.norm.weight"}, out)
    with pytest.raises(ValueError, match="missing"):
        audit_saved_checkpoint(out, sd)


def test_shadow_residual_checks(tmp_path):
    out, config, sd = _compose(tmp_path, cross_rank=4)
    assert config.dual_stream
    ads = [type("A", (), {"kind": "lora", "name": f"adapter_{i}"})() for i in range(2)]
    assert set(validate_cross_stream_population(sd, config, ads).values()) == {config.num_decoder_layers}
    bad = dict(sd)
    for i in range(config.num_decoder_layers):
        k = f"model.layers.{i}.cross_stream.lora_B"
        bad[k] = sd[k].clone()
        bad[k][1] = 0
    with pytest.raises(ValueError, match="adapter_1"):
        validate_cross_stream_population(bad, config, ads)
    # k/v LoRA on a Shadow-Residual adapter is rejected at compose time
    cfg = base_config("tiny")
    from granite_switch_b200.composer.synthetic import random_peft_adapter
    from granite_switch_b200.composer.compose import AdapterSpec

    t = random_peft_adapter(cfg, 8, ("q",), seed=3, cross_rank=4)
    t.update({k.replace("q_proj", "k_proj"): v for k, v in t.items() if "q_proj" in k})
    with pytest.raises(ValueError, match="k/v"):
        compose_checkpoint(cfg, random_base_state(cfg), [AdapterSpec("s", t, 8, 16.0)], str(tmp_path / "kv"))


def test_moe_base_rejects_mlp_adapters(tmp_path):
    cfg = base_config("tiny", num_local_experts=4, num_experts_per_tok=2, shared_intermediate_size=0,
                      model_type="granitemoe")
    from granite_switch_b200.composer.synthetic import random_peft_adapter
    from granite_switch_b200.composer.compose import AdapterSpec

    t = random_peft_adapter(dict(cfg, shared_intermediate_size=64, model_type="granite"), 8, ("q", "gate"), seed=2)
    with pytest.raises(ValueError, match="gate_proj"):
        compose_checkpoint(cfg, random_base_state(cfg), [AdapterSpec("m", t, 8, 16.0)], str(tmp_path / "m"))


@pytest.mark.parametrize("shared", [0, 64])
def test_compose_moe_bases(tmp_path, shared):
    extra = dict(shared_intermediate_size=shared) if shared else {}
    config = compose_synthetic(str(tmp_path / f"moe{shared}"), "tiny", num_adapters=2, rank=8,
                               targets=("q", "v", "gate", "up", "down"), num_local_experts=4,
                               num_experts_per_tok=2, **extra)
    v = config.compose_validation
    assert v["arch"] == "granitemoehybrid"
    assert ("shared_input_linear" in config.lora_target_modules) == bool(shared)
