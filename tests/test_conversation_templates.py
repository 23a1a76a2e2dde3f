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
