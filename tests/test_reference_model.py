"""Composer + checkpoint + HF-style model on CPU (benchmark config 1 and friends)."""
import json
import os

import pytest
import torch

from granite_switch_b200.checkpoint import load_state_dict, tensor_names
from granite_switch_b200.composer.synthetic import compose_synthetic
from granite_switch_b200.config import GraniteSwitchConfig
from granite_switch_b200.models import GraniteSwitchForCausalLM


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tiny"))
    # config 1: 3 aLoRA adapters, rank 8 on q/k/v, A~N(0,.02), B~N(0,.01), scaling 2
    compose_synthetic(d, "tiny", num_adapters=3, rank=8, targets=("q", "k", "v"), seed=0,
                      dtype=torch.float32, invocation_len=4, alpha=16.0)
    return d


def test_layout_and_config(tiny_dir):
    cfg = GraniteSwitchConfig.from_pretrained(tiny_dir)
    assert cfg.num_adapters == 3 and cfg.num_hidden_layers == 4 + 2 and cfg.num_decoder_layers == 4
    assert cfg.vocab_size == 1024 + 3 and cfg.adapter_token_ids == [1024, 1025, 1026]
    assert cfg.lora_target_modules == ["qkv_proj"]
    names = set(tensor_names(tiny_dir))
    assert "model.layers.0.self_attn.qkv_proj.base_layer.weight" in names
    assert "model.layers.0.self_attn.qkv_proj.lora_A_slices.2" in names
    assert "model.layers.3.self_attn.o_proj.weight" in names  # not a LoRA target
    assert "model.switch.codebook" in names and "model.switch.control_to_substitute_lut" in names
    sd = load_state_dict(tiny_dir)
    assert sd["model.switch.codebook"].dtype == torch.float32
    assert sd["model.layers.0.self_attn.qkv_proj.lora_B_slices.0"].shape == (3, 1, 256, 8)
    idx = json.load(open(os.path.join(tiny_dir, "adapter_index.json")))
    assert [a["adapter_index"] for a in idx["adapters"]] == [1, 2, 3]


def test_save_load_roundtrip(tiny_dir, tmp_path):
    m = GraniteSwitchForCausalLM.from_pretrained(tiny_dir)
    m.save_pretrained(str(tmp_path))
    m2 = GraniteSwitchForCausalLM.from_pretrained(str(tmp_path))
    a, b = m.state_dict(), m2.state_dict()
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k], b[k]), k
    # double serialization keeps byte size
    m2.save_pretrained(str(tmp_path / "again"))
    s1 = sum(os.path.getsize(os.path.join(tmp_path, f)) for f in os.listdir(tmp_path) if f.endswith(".safetensors"))
    s2 = sum(os.path.getsize(os.path.join(tmp_path / "again", f)) for f in os.listdir(tmp_path / "again") if f.endswith(".safetensors"))
    assert s1 == s2


def _alora_batch(cfg, idx_json, seed=0, batch=4, seq=128):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 1024, (batch, seq), generator=g)
    base_ids = ids.clone()
    inserts, adapters = [], []
    for b in range(batch):
        a = int(torch.randint(0, cfg.num_adapters, (1,), generator=g))
        pos = int(torch.randint(32, 97, (1,), generator=g))
        inv = idx_json["adapters"][a]["invocation_token_ids"]
        ctrl = cfg.adapter_token_ids[a]
        ids[b, pos:pos + len(inv)] = torch.tensor([ctrl] + inv[1:])
        base_ids[b, pos:pos + len(inv)] = torch.tensor(inv)
        inserts.append(pos)
        adapters.append(a + 1)
    return ids, base_ids, inserts, adapters


def test_config1_pre_invocation_equals_base(tiny_dir):
    """Benchmark config 1: logits and KV before the invocation equal the base model's."""
    cfg = GraniteSwitchConfig.from_pretrained(tiny_dir)
    idx = json.load(open(os.path.join(tiny_dir, "adapter_index.json")))
    m = GraniteSwitchForCausalLM.from_pretrained(tiny_dir).eval()
    ids, base_ids, inserts, adapters = _alora_batch(cfg, idx)
    with torch.no_grad():
        out = m(ids, use_cache=True)
        ref = m(base_ids, use_cache=True)  # no control token: every position runs base weights
    routed = out.adapter_indices
    for b, (pos, a) in enumerate(zip(inserts, adapters)):
        assert routed[b, :pos].eq(0).all() and routed[b, pos:].eq(a).all()
        torch.testing.assert_close(out.logits[b, :pos], ref.logits[b, :pos], rtol=0, atol=0)
        for layer in range(cfg.num_decoder_layers):
            torch.testing.assert_close(out.past_key_values.keys[layer][b, :pos], ref.past_key_values.keys[layer][b, :pos], rtol=0, atol=0)
            torch.testing.assert_close(out.past_key_values.values[layer][b, :pos], ref.past_key_values.values[layer][b, :pos], rtol=0, atol=0)
        # from the invocation on, the adapter changes the computation
        assert (out.logits[b, pos + 1:] - ref.logits[b, pos + 1:]).abs().max() > 1e-4


def test_incremental_decode_matches_full_forward(tiny_dir):
    cfg = GraniteSwitchConfig.from_pretrained(tiny_dir)
    idx = json.load(open(os.path.join(tiny_dir, "adapter_index.json")))
    m = GraniteSwitchForCausalLM.from_pretrained(tiny_dir).eval()
    ids, _, _, _ = _alora_batch(cfg, idx, seed=3, batch=2, seq=64)
    with torch.no_grad():
        full = m(ids).logits
        out = m(ids[:, :40], use_cache=True)
        cache = out.past_key_values
        steps = [out.logits]
        for t in range(40, 64, 8):
            o = m(ids[:, t:t + 8], past_key_values=cache, use_cache=True)
            cache = o.past_key_values
            steps.append(o.logits)
    torch.testing.assert_close(torch.cat(steps, 1), full, rtol=1e-4, atol=1e-4)


def test_generate_greedy_runs(tiny_dir):
    m = GraniteSwitchForCausalLM.from_pretrained(tiny_dir).eval()
    ids = torch.randint(0, 1024, (2, 10))
    out = m.generate(ids, max_new_tokens=5)
    assert out.shape == (2, 15)


def test_single_switch_checkpoint_rejected():
    with pytest.raises(ValueError, match="SingleSwitch"):
        GraniteSwitchConfig.from_dict({"num_adapters": 2, "adapter_token_ids": [5, 6],
                                       "adapter_substitute_token_ids": [1, 2], "adapter_ranks": [8, 8]})
    with pytest.raises(ValueError, match="SingleSwitch"):
        GraniteSwitchConfig.from_dict({"num_adapters": 1, "switch_type": "single", "ms_code_m": 6})


def test_config_validation_errors():
    with pytest.raises(ValueError):
        GraniteSwitchConfig(num_adapters=2, adapter_token_ids=[1, 1], adapter_substitute_token_ids=[0, 0],
                            adapter_ranks=[8, 8])
    with pytest.raises(ValueError):
        GraniteSwitchConfig(num_adapters=1, adapter_token_ids=[1], adapter_ranks=[8])
    with pytest.raises(ValueError):
        GraniteSwitchConfig(num_adapters=1, adapter_token_ids=[1], adapter_substitute_token_ids=[0],
                            adapter_ranks=[4], max_lora_rank=8)
    with pytest.raises(ValueError):
        GraniteSwitchConfig(dual_stream=True)
    c = GraniteSwitchConfig(num_adapters=2, adapter_token_ids=[9, 10, 11], adapter_substitute_token_ids=[1, 2, 3],
                            adapter_ranks=[8, 4])
    assert c.has_base_reset and c.lora_target_modules[:2] == ["qkv_proj", "o_proj"]
    d = GraniteSwitchConfig.from_dict(c.to_dict())
    assert d == c


def test_transformers_auto_classes(tiny_dir):
    """Importing granite_switch_b200.hf registers model_type granite_switch with transformers' Auto classes."""
    import granite_switch_b200.hf  # noqa: F401
    from transformers import AutoConfig, AutoModelForCausalLM

    cfg = AutoConfig.from_pretrained(tiny_dir)
    assert cfg.model_type == "granite_switch"
    assert cfg.to_native().adapter_token_ids == GraniteSwitchConfig.from_pretrained(tiny_dir).adapter_token_ids
    m = AutoModelForCausalLM.from_pretrained(tiny_dir)
    assert isinstance(m, GraniteSwitchForCausalLM)
    ids = torch.randint(1, 900, (1, 12))
    with torch.no_grad():
        torch.testing.assert_close(m(ids).logits, GraniteSwitchForCausalLM.from_pretrained(tiny_dir)(ids).logits)
