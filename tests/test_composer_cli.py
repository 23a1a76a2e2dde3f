"""Composer CLI over on-disk PEFT adapter libraries, YAML manifests and built-in slots."""
import json
import os

import pytest
import torch
import yaml
from safetensors.torch import save_file

from granite_switch_b200.composer.adapter_discovery import discover_library, filter_adapters
from granite_switch_b200.composer.cli import compose_main
from granite_switch_b200.composer.synthetic import base_config, random_base_state, random_peft_adapter
from granite_switch_b200.config import GraniteSwitchConfig
from granite_switch_b200.models import GraniteSwitchForCausalLM


def _write_base(d):
    cfg = base_config("tiny", num_hidden_layers=2)
    os.makedirs(d, exist_ok=True)
    json.dump({**cfg, "model_type": "granite", "hidden_act": "silu"}, open(os.path.join(d, "config.json"), "w"))
    save_file(random_base_state(cfg, seed=0), os.path.join(d, "model.safetensors"))
    return cfg


def _write_adapter(d, cfg, seed, targets, tech="alora", r=8, alpha=16, io=True):
    os.makedirs(d, exist_ok=True)
    conf = {"r": r, "lora_alpha": alpha, "target_modules": [f"{t}_proj" for t in targets], "peft_type": "LORA"}
    if tech == "alora":
        conf["alora_invocation_tokens"] = [5 + seed, 6, 7]
    json.dump(conf, open(os.path.join(d, "adapter_config.json"), "w"))
    save_file(random_peft_adapter(cfg, r, targets, seed=seed), os.path.join(d, "adapter_model.safetensors"))
    if io:
        yaml.safe_dump({"name": os.path.basename(os.path.dirname(os.path.dirname(d))), "model": None},
                       open(os.path.join(d, "io.yaml"), "w"))


@pytest.fixture
def lib(tmp_path):
    base = str(tmp_path / "base")
    cfg = _write_base(base)
    root = tmp_path / "lib"
    _write_adapter(str(root / "answerability" / "base" / "alora"), cfg, 1, ("q", "k", "v"))
    _write_adapter(str(root / "answerability" / "base" / "lora"), cfg, 2, ("q", "k", "v"), tech="lora")
    _write_adapter(str(root / "citations" / "base" / "alora"), cfg, 3, ("q", "k", "v", "o"))
    _write_adapter(str(root / "query_rewrite" / "base" / "lora"), cfg, 4, ("q", "v", "gate", "up", "down"),
                   tech="lora")
    return base, str(root), cfg


def test_discovery_prefers_alora_and_filters(lib):
    _, root, _ = lib
    found = discover_library(root, "base")
    assert [(f.name, f.technology) for f in found] == [("answerability", "alora"), ("citations", "alora"),
                                                       ("query_rewrite", "lora")]
    assert [f.name for f in filter_adapters(found, include=["*ans*", "query_*"], exclude=["query_*"])] == \
        ["answerability"]
    assert [f.name for f in filter_adapters(found, technology="lora")] == ["query_rewrite"]


def test_compose_cli_end_to_end(lib, tmp_path):
    base, root, cfg = lib
    out = str(tmp_path / "out")
    rc = compose_main(["--adapters", root, "--base-model", base, "--target-model", "base", "--output", out,
                       "--dtype", "float32", "--built-in-adapters", "scratch", "--base-reset-token"])
    assert rc == 0
    c = GraniteSwitchConfig.from_pretrained(out)
    assert c.adapter_names == ["answerability", "citations", "query_rewrite", "scratch"]
    assert len(c.adapter_token_ids) == c.num_adapters + 1  # leading base-reset token
    assert set(c.lora_target_modules) == {"qkv_proj", "o_proj", "shared_input_linear", "shared_output_linear"}
    for f in ("adapter_index.json", "compose_report.json", "BUILD.md", "io_configs/answerability.yaml"):
        assert os.path.exists(os.path.join(out, f)), f
    m = GraniteSwitchForCausalLM.from_pretrained(out).eval()
    # aLoRA: everything before the control token equals the base model (no control token)
    idx = json.load(open(os.path.join(out, "adapter_index.json")))
    ctrl = idx["adapters"][0]["control_token"]["id"]
    ids = torch.randint(8, 1000, (1, 40))
    with torch.no_grad():
        plain = m(ids).logits
        switched = m(torch.cat([ids, torch.tensor([[ctrl, 6, 7]])], 1)).logits
    torch.testing.assert_close(switched[:, :40], plain, rtol=0, atol=0)
    # built-in slot has no weights: routing to it equals base
    ctrl_b = idx["adapters"][3]["control_token"]["id"]
    with torch.no_grad():
        b1 = m(torch.cat([ids, torch.tensor([[ctrl_b, 9]])], 1)).logits[:, -1]
        b0 = m(torch.cat([ids, torch.tensor([[c.adapter_substitute_token_ids[4], 9]])], 1)).logits[:, -1]
    torch.testing.assert_close(b1, b0, rtol=1e-5, atol=1e-5)


def test_yaml_manifest_and_missing_ioyaml(lib, tmp_path):
    base, root, cfg = lib
    bare = str(tmp_path / "bare" / "x" / "base" / "alora")
    _write_adapter(bare, cfg, 9, ("q",), io=False)
    man = tmp_path / "m.yaml"
    yaml.safe_dump({"adapters": [{"path": bare, "name": "bare_one", "type": "alora"}]}, open(man, "w"))
    out = str(tmp_path / "o2")
    with pytest.raises(FileNotFoundError):
        compose_main(["--adapters", str(man), "--base-model", base, "--output", out, "--dtype", "float32"])
    assert compose_main(["--adapters", str(man), "--base-model", base, "--output", out, "--dtype", "float32",
                         "--create-ioyaml"]) == 0
    assert GraniteSwitchConfig.from_pretrained(out).adapter_names == ["bare_one"]


def test_list_adapters(lib, capsys):
    _, root, _ = lib
    assert compose_main(["--adapters", root, "--target-model", "base", "--list-adapters"]) == 0
    assert "citations" in capsys.readouterr().out


def test_compose_cli_with_tokenizer_and_audio(lib, tmp_path):
    """Base directory with a tokenizer: control tokens, substitutes and the
    adapter-aware chat template are written with the checkpoint."""
    from transformers import AutoTokenizer

    from tests.tokenizer_stub import granite_template, make_tokenizer

    base, root, cfg = lib
    make_tokenizer(granite_template("4.1")).save_pretrained(base)
    out = str(tmp_path / "out_tok")
    rc = compose_main(["--adapters", root, "--base-model", base, "--target-model", "base", "--output", out,
                       "--dtype", "float32", "--enable-audio"])
    assert rc == 0
    c = GraniteSwitchConfig.from_pretrained(out)
    tok = AutoTokenizer.from_pretrained(out)
    ctrl = dict(zip(c.adapter_names, c.adapter_token_ids))
    sub = dict(zip(c.adapter_token_ids, c.adapter_substitute_token_ids))
    assert [tok.convert_ids_to_tokens(ctrl[n]) for n in c.adapter_names] == [f"<|{n}|>" for n in c.adapter_names]
    marker = tok.convert_tokens_to_ids("<|start_of_role|>")
    assert sub[ctrl["query_rewrite"]] == marker                       # LoRA: position-0 token
    inv = json.load(open(os.path.join(root, "answerability", "base", "alora", "adapter_config.json")))
    assert sub[ctrl["answerability"]] == inv["alora_invocation_tokens"][0]
    audio = tok.convert_tokens_to_ids("<|audio|>")
    assert audio < c.vocab_size
    msgs = [{"role": "user", "content": [{"type": "text", "text": "hi"}, {"type": "audio", "audio": None}]}]
    plain = tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True)
    assert "hi<|audio|>" in plain
    lora = tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True, adapter_name="query_rewrite")
    ids = tok.encode(lora, add_special_tokens=False)
    assert ids[0] == ctrl["query_rewrite"]
    assert [sub.get(i, i) for i in ids] == tok.encode(plain, add_special_tokens=False)
    # control and audio rows: never-emitted output rows copied from the reserved token
    from safetensors.torch import load_file

    sd = {}
    for f in os.listdir(out):
        if f.endswith(".safetensors"):
            sd.update(load_file(os.path.join(out, f)))
    emb = sd["model.embed_tokens.weight"]
    reserved = tok.convert_tokens_to_ids("<|unused_1|>")
    for t in list(ctrl.values()) + [audio]:
        torch.testing.assert_close(emb[t], emb[reserved])


def test_hf_repo_selective_download(lib, monkeypatch, tmp_path):
    """A repo id resolves through huggingface_hub with patterns limited to the target model,
    the included adapters and the technology (no network here: the download is faked)."""
    import huggingface_hub

    from granite_switch_b200.composer.adapter_discovery import hf_patterns, resolve

    _, root, _ = lib
    calls = []

    def fake(repo, allow_patterns=None, ignore_patterns=None, local_files_only=False):
        calls.append((repo, allow_patterns, ignore_patterns, local_files_only))
        return root

    monkeypatch.setattr(huggingface_hub, "snapshot_download", fake)
    monkeypatch.delenv("HF_HUB_OFFLINE", raising=False)
    found = resolve(["org/granitelib"], "base", "alora", include=["ans*", "cit*"], exclude=["cit*"])
    assert calls[0][0] == "org/granitelib" and calls[0][3] is False
    assert calls[0][1][:2] == ["ans*/base/alora/*", "cit*/base/alora/*"] and calls[0][2] == ["cit*/*"]
    assert {f.name for f in found} == {"answerability", "citations"}
    assert hf_patterns(None) == (None, None)
    assert hf_patterns("ibm-granite/granite-4.1-3b", technology="lora")[0][0] == "*/granite-4.1-3b/lora/*"
