"""Differential tests against the reference's own code (CPU).

The reference package (granite-switch, installed under ``baseline/_ref`` with
``pip install --target``) runs in child processes, so its transformers
registrations and module names never meet this package's:

* a checkpoint composed here loads in the reference's HF class, and its logits
  equal this build's fp32 model (reference: src/granite_switch/hf/modeling_granite_switch.py:784-931);
* the reference's composer and this one, given the same base model and PEFT
  adapter library, write the same config fields and the same tensors (the
  Kerdock codebook excepted: any unit-norm low-coherence code serves the
  switch, and this build orders its codewords its own way), and chat templates
  whose renders are identical for every ``adapter_name`` (reference:
  src/granite_switch/composer/compose_granite_switch.py:1075-1626,
  src/granite_switch/composer/tokenizer_setup.py:1360);
* a checkpoint written by the reference's composer serves here: the CPU engine
  generates what this build's HF-style model generates, and this model's logits
  equal the reference's HF class on that checkpoint.

Skipped when the reference is not installed.
"""
import json
import os
import subprocess
import sys

import pytest
import torch
import yaml
from safetensors.torch import load_file, save_file

from granite_switch_b200.composer.synthetic import base_config, random_base_state, random_peft_adapter
from tests.tokenizer_stub import granite_template, make_tokenizer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_path():
    ref = os.path.join(ROOT, "baseline", "_ref")
    for root in (ref, os.path.join(ref, "src")):
        if os.path.isfile(os.path.join(root, "granite_switch", "__init__.py")):
            return root
    return None


REF = _reference_path()
pytestmark = pytest.mark.skipif(REF is None, reason="the reference is not installed under baseline/_ref")

_REF_LOGITS = """
import sys, json, torch
from granite_switch.hf import load_model
m = load_model(sys.argv[1]).eval()
ids = torch.tensor(json.loads(sys.argv[2]))
with torch.no_grad():
    out = m(input_ids=ids)
torch.save(out.logits.float(), sys.argv[3])
"""


def _run_reference(args, cwd):
    env = dict(os.environ, PYTHONPATH=REF, HF_HUB_OFFLINE="1", TRANSFORMERS_OFFLINE="1")
    r = subprocess.run([sys.executable] + args, cwd=cwd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return r


def _reference_logits(model_dir, ids, tmp):
    script = os.path.join(tmp, "ref_logits.py")
    with open(script, "w") as f:
        f.write(_REF_LOGITS)
    out = os.path.join(tmp, "ref_logits.pt")
    _run_reference([script, model_dir, json.dumps(ids), out], tmp)
    return torch.load(out)


def _write_inputs(root, version):
    """A tiny Granite base (with a character-level tokenizer carrying the Granite chat
    template) and a library of one aLoRA and one LoRA PEFT adapter."""
    base = os.path.join(root, "base")
    cfg = base_config("tiny", num_hidden_layers=2)
    os.makedirs(base, exist_ok=True)
    tok = make_tokenizer(granite_template(version))
    json.dump({**cfg, "model_type": "granite", "hidden_act": "silu", "architectures": ["GraniteForCausalLM"]},
              open(os.path.join(base, "config.json"), "w"))
    save_file(random_base_state(cfg, seed=0), os.path.join(base, "model.safetensors"))
    tok.save_pretrained(base)
    lib = os.path.join(root, "lib")
    req = tok.encode("<requirements>", add_special_tokens=False)

    def adapter(name, tech, targets, seed):
        d = os.path.join(lib, name, "base", tech)
        os.makedirs(d, exist_ok=True)
        conf = {"r": 8, "lora_alpha": 16, "target_modules": [f"{t}_proj" for t in targets], "peft_type": "LORA"}
        if tech == "alora":
            conf["alora_invocation_tokens"] = req
        json.dump(conf, open(os.path.join(d, "adapter_config.json"), "w"))
        save_file(random_peft_adapter(cfg, 8, targets, seed=seed), os.path.join(d, "adapter_model.safetensors"))
        yaml.safe_dump({"name": name, "model": None}, open(os.path.join(d, "io.yaml"), "w"))

    adapter("answerability", "alora", ("q", "k", "v"), 1)
    adapter("citations", "lora", ("q", "k", "v", "o"), 3)
    return base, lib


def _state(d):
    sd = {}
    for f in sorted(os.listdir(d)):
        if f.endswith(".safetensors"):
            sd.update(load_file(os.path.join(d, f)))
    return sd


@pytest.fixture(scope="module", params=["4.1", "4.2"])
def composed(request, tmp_path_factory):
    """The same inputs composed by the reference's composer and by this one."""
    root = str(tmp_path_factory.mktemp(f"diff{request.param}"))
    base, lib = _write_inputs(root, request.param)
    ref_out, my_out = os.path.join(root, "ref_out"), os.path.join(root, "my_out")
    _run_reference(["-m", "granite_switch.composer.compose_granite_switch", "--adapters", lib, "--base-model", base,
                    "--target-model", "base", "--output", ref_out], root)
    from granite_switch_b200.composer.cli import compose_main

    assert compose_main(["--adapters", lib, "--base-model", base, "--target-model", "base", "--output", my_out]) == 0
    return request.param, root, ref_out, my_out


def test_composers_write_the_same_checkpoint(composed):
    _, _, ref_out, my_out = composed
    from granite_switch_b200.config import GraniteSwitchConfig

    a, b = GraniteSwitchConfig.from_pretrained(ref_out), GraniteSwitchConfig.from_pretrained(my_out)
    for field in ("num_adapters", "adapter_token_ids", "adapter_substitute_token_ids", "adapter_names",
                  "adapter_ranks", "max_lora_rank", "num_hidden_layers", "vocab_size", "hidden_size",
                  "num_attention_heads", "num_key_value_heads", "rope_theta", "tie_word_embeddings",
                  "ms_code_m", "ms_memory_gain", "torch_dtype"):
        assert getattr(a, field) == getattr(b, field), field
    assert sorted(a.lora_target_modules) == sorted(b.lora_target_modules)
    ra, rb = _state(ref_out), _state(my_out)
    assert set(ra) == set(rb)
    for k in ra:
        if k == "model.switch.codebook":  # same shape and unit rows; the codeword order is this build's own
            assert ra[k].shape == rb[k].shape
            torch.testing.assert_close(rb[k].norm(dim=1), torch.ones(rb[k].shape[0]))
            continue
        assert ra[k].dtype == rb[k].dtype and ra[k].shape == rb[k].shape, k
        assert torch.equal(ra[k], rb[k]), k


def test_chat_templates_render_the_same(composed):
    """Both composed tokenizers render every conversation id-for-id alike, with and without
    each adapter (aLoRA: control token before the invocation text, or before the generation
    prompt when the last user turn lacks it; LoRA: at the start)."""
    from transformers import AutoTokenizer

    _, _, ref_out, my_out = composed
    ta, tb = AutoTokenizer.from_pretrained(ref_out), AutoTokenizer.from_pretrained(my_out)
    convs = [
        [{"role": "user", "content": "Is this answerable? <requirements> short"}],
        [{"role": "system", "content": "You are a careful assistant."},
         {"role": "user", "content": "first question"},
         {"role": "assistant", "content": "first answer"},
         {"role": "user", "content": "second question with <requirements> inside"}],
        [{"role": "user", "content": "no invocation text here"}],
    ]
    for msgs in convs:
        for name in (None, "answerability", "citations"):
            kw = {} if name is None else {"adapter_name": name}
            a = ta.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False, **kw)
            b = tb.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False, **kw)
            assert a == b, (name, msgs)
            assert ta.encode(a, add_special_tokens=False) == tb.encode(b, add_special_tokens=False)


def test_reference_hf_class_loads_our_checkpoint(composed, tmp_path):
    _, _, _, my_out = composed
    from granite_switch_b200.models import GraniteSwitchForCausalLM

    idx = json.load(open(os.path.join(my_out, "adapter_index.json")))
    ctrl = [a["control_token"]["id"] for a in idx["adapters"]]
    ids = [[5, 6, 7, 8, 9, ctrl[0], 11, 12, 13, 14, ctrl[1], 15, 16],
           [21, 22, ctrl[1], 23, 24, 25, 26, 27, 28, 29, 30, 31, 32]]
    ref = _reference_logits(my_out, ids, str(tmp_path))
    m = GraniteSwitchForCausalLM.from_pretrained(my_out).eval()
    with torch.no_grad():
        mine = m(torch.tensor(ids)).logits.float()
    torch.testing.assert_close(mine, ref, rtol=1e-5, atol=1e-5)


def test_reference_composed_checkpoint_serves_here(composed, tmp_path):
    _, _, ref_out, _ = composed
    from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams
    from granite_switch_b200.models import GraniteSwitchForCausalLM

    idx = json.load(open(os.path.join(ref_out, "adapter_index.json")))
    ctrl = [a["control_token"]["id"] for a in idx["adapters"]]
    prompts = [[5, 6, 7, 8, ctrl[0], 107, 31], [40, 41, 42, 43, 44, ctrl[1], 45, 46, 47]]
    ref = _reference_logits(ref_out, [prompts[0]], str(tmp_path))
    m = GraniteSwitchForCausalLM.from_pretrained(ref_out).eval()
    with torch.no_grad():
        torch.testing.assert_close(m(torch.tensor([prompts[0]])).logits.float(), ref, rtol=1e-5, atol=1e-5)
    llm = LLM(ref_out, device="cpu", engine_config=EngineConfig(max_num_seqs=2, num_kv_blocks=32,
                                                                max_model_len=128))
    outs = llm.generate(prompts, SamplingParams(max_tokens=5))
    for p, o in zip(prompts, outs):
        g = m.generate(torch.tensor([p]), max_new_tokens=5)[0, len(p):].tolist()
        assert o.output_ids == g
