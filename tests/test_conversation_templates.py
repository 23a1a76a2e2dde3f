"""Conversation over the composed chat templates of the Granite 4.1 (role markers) and 4.2
(ChatML) families (reference: tests/unit/test_conversation_policy.py, test_conversation_chatml.py)."""
import pytest

from granite_switch_b200.composer.compose import AdapterSpec
from granite_switch_b200.composer.tokenizer_setup import configure_tokenizer, encode
from granite_switch_b200.conversation import Conversation, KVHistoryPolicy
from tests.tokenizer_stub import granite_template, make_tokenizer

HEADER = {"4.1": "<|start_of_role|>assistant<|end_of_role|>", "4.2": "<|im_start|>assistant\n"}


class _Cfg:
    def __init__(self, ids):
        self.adapter_token_ids = ids


def _setup(version):
    tok = make_tokenizer(granite_template(version))
    ads = [AdapterSpec("ans", {}, 8, 8.0, technology="alora", invocation_tokens=encode(tok, HEADER[version])),
           AdapterSpec("rw", {}, 8, 8.0, technology="lora")]
    ids, _ = configure_tokenizer(tok, ads)
    return tok, _Cfg(ids), dict(zip(["ans", "rw"], ids))


@pytest.mark.parametrize("version", ["4.1", "4.2"])
def test_re_prefill_shares_the_base_history(version):
    tok, cfg, ctrl = _setup(version)
    kw = {"enable_thinking": False} if version == "4.2" else {}
    conv = Conversation(tok, KVHistoryPolicy.RE_PREFILL, cfg)
    conv.user("What is the fee for a permit?")
    p1 = list(conv.build_prompt("ans", **kw))
    assert p1.count(ctrl["ans"]) == 1
    conv.record_answer(encode(tok, "It is ten dollars."), adapter="ans")
    conv.user("And the deadline?")
    p2 = list(conv.build_prompt("ans", **kw))
    # history is sent in base form: only this turn's control token, and the ids equal a fresh encode
    assert p2.count(ctrl["ans"]) == 1
    full = tok.apply_chat_template(conv.messages, add_generation_prompt=True, tokenize=False, adapter_name="ans",
                                   **kw)
    assert p2 == encode(tok, full)
    # the first turn's prompt up to its control token is a prefix of the second prompt
    cut = p1.index(ctrl["ans"])
    assert p2[:cut] == p1[:cut]


def test_preserve_keeps_the_earlier_control_token():
    tok, cfg, ctrl = _setup("4.1")
    conv = Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY, cfg)
    conv.user("What is the fee for a permit?")
    p1 = list(conv.build_prompt("ans"))
    answer = encode(tok, "It is ten dollars.")
    conv.record_answer(answer, adapter="ans")
    sent = conv.sent_token_ids
    assert sent == p1 + answer + encode(tok, "<|end_of_text|>\n")
    conv.user("And the deadline?")
    p2 = list(conv.build_prompt("ans"))
    assert p2[:len(sent)] == sent and p2.count(ctrl["ans"]) == 2
    assert conv.reprefills == 0


def test_chatml_preserve_needs_thinking_off():
    tok, cfg, ctrl = _setup("4.2")
    conv = Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY, cfg)
    conv.user("What is the fee?")
    p1 = list(conv.build_prompt("ans", enable_thinking=False))
    conv.record_answer(encode(tok, "Ten dollars."), adapter="ans")
    assert conv.sent_token_ids == p1 + encode(tok, "Ten dollars.") + encode(tok, "<|im_end|>\n")
    conv.user("When?")
    p2 = list(conv.build_prompt("ans", enable_thinking=False))
    assert p2[:len(conv.sent_token_ids)] == conv.sent_token_ids and p2.count(ctrl["ans"]) == 2
    # with thinking on the generation prompt opens a think block that the history re-renders differently
    conv2 = Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY, cfg)
    conv2.user("What is the fee?")
    conv2.build_prompt("ans")
    with pytest.raises(RuntimeError):
        conv2.record_answer(encode(tok, "Ten dollars."), adapter="ans")


def _engine_with_template(tmp_path):
    import torch

    from granite_switch_b200.composer.compose import compose_checkpoint
    from granite_switch_b200.composer.synthetic import base_config, random_base_state, synthetic_adapters
    from granite_switch_b200.engine import LLM, EngineConfig

    tok = make_tokenizer(granite_template("4.1"))
    cfg = base_config("tiny", num_hidden_layers=2)
    ads = synthetic_adapters(cfg, 2, 8, ("q", "k", "v", "o"), seed=1)
    for a in ads:
        a.invocation_tokens = encode(tok, HEADER["4.1"])
    ids, setup = configure_tokenizer(tok, ads)
    d = str(tmp_path / "conv")
    config = compose_checkpoint(cfg, random_base_state(cfg), ads, d, dtype=torch.float32, control_token_ids=ids,
                                default_substitute=setup.lora_substitute)
    llm = LLM(d, device="cpu", engine_config=EngineConfig(max_num_seqs=2, max_num_batched_tokens=512,
                                                          num_kv_blocks=256, max_model_len=2048))
    return tok, config, llm


def test_turn_two_prefix_reuse_by_policy(tmp_path):
    """Turn 2 of an aLoRA conversation (reference: tests/integration/test_conversation_prefix_cache.py):
    PRESERVE sends the turn-1 ids verbatim, so all of them are cache hits; RE_PREFILL re-renders the
    history in base form and reuses the cache up to the turn-1 control token."""
    from granite_switch_b200.engine import SamplingParams

    tok, config, llm = _engine_with_template(tmp_path)
    cached = {}
    for policy in (KVHistoryPolicy.RE_PREFILL, KVHistoryPolicy.PRESERVE_MIXED_HISTORY):
        llm.engine.blocks.reset_prefix_cache()
        conv = Conversation(tok, policy, config)
        conv.system("Answer from the document. The permit fee is ten dollars and renewals take a week.")
        conv.user("What is the fee for a permit?")
        p1 = conv.build_prompt("adapter_0")
        out1 = llm.generate([list(p1)], SamplingParams(max_tokens=6))[0]
        conv.record_answer(out1.output_ids, adapter="adapter_0")
        conv.user("And how long does a renewal take?")
        p2 = conv.build_prompt("adapter_0")
        out2 = llm.generate([list(p2)], SamplingParams(max_tokens=2))[0]
        cached[policy] = (out2.num_cached_tokens, len(p1), p1.index(config.adapter_token_ids[0]))
    pre, pre_p1, _ = cached[KVHistoryPolicy.PRESERVE_MIXED_HISTORY]
    re, _, ctrl_pos = cached[KVHistoryPolicy.RE_PREFILL]
    assert pre >= 16 * (pre_p1 // 16)            # every full block of the sent turn-1 prompt
    assert 16 * (ctrl_pos // 16) <= re < pre     # base-form history: hits stop at the old control token
