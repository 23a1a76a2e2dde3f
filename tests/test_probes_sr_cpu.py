"""Probe heads and Shadow-Residual (dual-stream) semantics of the HF-style model (CPU, fp32)."""
import json
import os

import pytest
import torch


@pytest.fixture(scope="module")
def probe_dir(tmp_path_factory):
    from granite_switch_b200.composer.synthetic import compose_synthetic

    d = str(tmp_path_factory.mktemp("probe"))
    compose_synthetic(d, "tiny", num_adapters=2, rank=8, num_probes=2, probe_read_layers=[1, None],
                      num_hidden_layers=2, seed=3)
    return d


@pytest.fixture(scope="module")
def sr_dir(tmp_path_factory):
    from granite_switch_b200.composer.synthetic import compose_synthetic

    d = str(tmp_path_factory.mktemp("sr"))
    compose_synthetic(d, "tiny", num_adapters=2, rank=8, cross_rank=16, num_hidden_layers=2, seed=4,
                      targets=("q", "k", "v", "o", "gate", "up", "down"), std_b=0.05)
    return d


def _capture(module):
    store = {}

    def hook(_m, _inp, out):
        store["out"] = out[0] if isinstance(out, tuple) else out

    return store, module.register_forward_hook(hook)


@pytest.mark.parametrize("slot", [0, 1])
def test_probe_verdict_replaces_marker_logits(probe_dir, slot):
    from granite_switch_b200.models.reference import GraniteSwitchForCausalLM

    m = GraniteSwitchForCausalLM.from_pretrained(probe_dir).eval()
    cfg = m.config
    g = torch.Generator().manual_seed(slot)
    ids = torch.randint(1, 1000, (1, 24), generator=g)
    marker = cfg.probe_control_token_ids[slot]
    ids[0, -1] = marker
    layer = cfg.probe_read_layers[2 + slot]
    target = m.model.layers[layer] if layer is not None else m.model.norm
    store, hnd = _capture(target)
    with torch.no_grad():
        out = m(ids)
    hnd.remove()
    hidden = store["out"][0, -1]
    w = m.model.probe_head.weight[2 + slot]
    b = m.model.probe_head.bias[2 + slot]
    labels = cfg.probe_label_token_ids[2 + slot]
    want = (w.float() @ hidden.float() + b.float())[: len(labels)]
    row = out.logits[0, -1]
    assert torch.isinf(row).sum().item() == row.numel() - len(labels)
    torch.testing.assert_close(row[torch.tensor(labels)], want, rtol=1e-4, atol=1e-4)
    # the marker position runs no LoRA delta: probe slots are not LoRA adapters
    last = m.model._last
    assert int(last["lora_indices"][0, -1]) == 0 and int(last["probe_indices"][0, -1]) == 3 + slot
    # earlier positions are untouched by the verdict
    assert not torch.isinf(out.logits[0, :-1]).any()


def test_probe_marker_must_be_last(probe_dir):
    from granite_switch_b200.models.reference import GraniteSwitchForCausalLM

    m = GraniteSwitchForCausalLM.from_pretrained(probe_dir).eval()
    ids = torch.randint(1, 1000, (1, 10))
    ids[0, 4] = m.config.probe_control_token_ids[0]
    with pytest.raises(RuntimeError, match="last token"):
        m(ids)


def test_sr_kv_is_base_only(sr_dir):
    """Shadow Residual: every position's K/V comes from the base stream, so the cache after an
    adapter's control token equals the cache of the same prompt with no adapter active."""
    from granite_switch_b200.models.reference import GraniteSwitchForCausalLM

    m = GraniteSwitchForCausalLM.from_pretrained(sr_dir).eval()
    cfg = m.config
    assert cfg.dual_stream and cfg.cross_stream_rank == 16
    idx = json.load(open(os.path.join(sr_dir, "adapter_index.json")))
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(1, 1000, (1, 30), generator=g)
    ctrl = idx["adapters"][1]["control_token"]["id"]
    ids[0, 12] = ctrl
    sub = cfg.adapter_substitute_token_ids[1]
    plain = ids.clone()
    plain[0, 12] = sub  # same embeddings, routing stays on the base model
    with torch.no_grad():
        a = m(ids, use_cache=True)
        b = m(plain, use_cache=True)
    ca, cb = a.past_key_values, b.past_key_values
    for ka, va, kb, vb in zip(ca.keys, ca.values, cb.keys, cb.values):
        torch.testing.assert_close(ka, kb, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(va, vb, rtol=1e-5, atol=1e-5)
    # before the control token the outputs agree; from it on the adapter stream differs
    torch.testing.assert_close(a.logits[0, :12], b.logits[0, :12], rtol=1e-5, atol=1e-5)
    assert (a.logits[0, 12:] - b.logits[0, 12:]).abs().max() > 1e-3


def _sr_prompts(d, n, seed=0):
    idx = json.load(open(os.path.join(d, "adapter_index.json")))
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        ids = torch.randint(1, 1000, (int(torch.randint(20, 50, (1,), generator=g)),), generator=g).tolist()
        a = i % 2
        ids += [idx["adapters"][a]["control_token"]["id"]] + idx["adapters"][a]["invocation_token_ids"][1:]
        out.append(ids)
    return out


@pytest.mark.parametrize("budget", [16, 512])
def test_engine_sr_matches_generate(sr_dir, budget):
    """The paged engine runs the dual stream like the HF-style model (chunked prefill included)."""
    from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams
    from granite_switch_b200.models.reference import GraniteSwitchForCausalLM

    prompts = _sr_prompts(sr_dir, 4)
    llm = LLM(sr_dir, device="cpu", engine_config=EngineConfig(max_num_seqs=3, max_num_batched_tokens=budget,
                                                               num_kv_blocks=64, max_model_len=256))
    outs = llm.generate(prompts, SamplingParams(max_tokens=5))
    m = GraniteSwitchForCausalLM.from_pretrained(sr_dir).eval()
    for o, p in zip(outs, prompts):
        ref = m.generate(torch.tensor([p]), max_new_tokens=5)[0, len(p):].tolist()
        assert o.output_ids == ref


def test_engine_probe_verdict(probe_dir):
    """A request ending in a probe's control token samples from the verdict (one of its labels),
    exactly as the HF-style model's rewritten logits."""
    from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams
    from granite_switch_b200.models.reference import GraniteSwitchForCausalLM

    m = GraniteSwitchForCausalLM.from_pretrained(probe_dir).eval()
    cfg = m.config
    g = torch.Generator().manual_seed(11)
    prompts = []
    for slot in (0, 1, 0):
        ids = torch.randint(1, 1000, (int(torch.randint(10, 40, (1,), generator=g)),), generator=g).tolist()
        prompts.append(ids + [cfg.probe_control_token_ids[slot]])
    llm = LLM(probe_dir, device="cpu", engine_config=EngineConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                                  num_kv_blocks=64, max_model_len=256))
    outs = llm.generate(prompts, SamplingParams(max_tokens=1))
    for o, p, slot in zip(outs, prompts, (0, 1, 0)):
        logits = m(torch.tensor([p])).logits[0, -1]
        assert o.output_ids == [int(logits.argmax())]
        assert o.output_ids[0] in cfg.probe_label_token_ids[2 + slot]
