"""Conversation prompt building under both KV history policies (stub tokenizer)."""
import pytest

from granite_switch_b200.conversation import (
    MAX_RETAINED_CONTROL_TOKENS,
    Conversation,
    KVHistoryPolicy,
    PromptTokenIds,
)
from tests.conversation_stub import StubConfig, StubTokenizer


@pytest.fixture
def tok():
    return StubTokenizer({"uq": "alora", "ans": "alora", "rewrite": "lora"})


def _ans(tok, text):
    return tok(text)["input_ids"]


def test_preserve_keeps_earlier_control_tokens(tok):
    cfg = StubConfig(tok.control_token_ids())
    conv = Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY, cfg)
    conv.user("hello")
    ids1 = conv.build_prompt(adapter="uq")
    assert isinstance(ids1, PromptTokenIds) and ids1.requires_token_ids
    assert tok.special_ids["<|uq|>"] in ids1
    conv.record_answer(_ans(tok, "fine"), adapter="uq")
    conv.user("again")
    ids2 = conv.build_prompt(adapter="ans")
    # turn 2 extends exactly what was sent in turn 1 (prompt + answer + terminator)
    assert ids2[: len(ids1)] == list(ids1)
    assert tok.special_ids["<|uq|>"] in ids2 and tok.special_ids["<|ans|>"] in ids2
    assert conv.reprefills == 0
    assert conv.generated_control_tokens == [[]]


def test_preserve_lora_turn_reprefills(tok):
    conv = Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY, StubConfig(tok.control_token_ids()))
    conv.user("a")
    conv.build_prompt(adapter="uq")
    conv.record_answer(_ans(tok, "b"))
    conv.user("c")
    ids = conv.build_prompt(adapter="rewrite")  # LoRA token lands at position 0
    assert conv.reprefills == 1
    assert ids[0] == tok.special_ids["<|rewrite|>"]
    assert tok.special_ids["<|uq|>"] not in ids


def test_re_prefill_reuses_base_form_prefix(tok):
    conv = Conversation(tok, KVHistoryPolicy.RE_PREFILL)
    conv.user("q1")
    conv.build_prompt(adapter="uq")
    conv.record_answer("a1")
    conv.user("q2")
    ids2 = conv.build_prompt(adapter="ans")
    conv.record_answer("a2")
    conv.user("q3")
    ids3 = conv.build_prompt(adapter="uq")
    # earlier adapters are demoted to base: only this turn's control token is present
    assert tok.special_ids["<|ans|>"] not in ids3 and tok.special_ids["<|uq|>"] in ids3
    # history prefix sent at turn 2 (up to its control token) is reused verbatim at turn 3
    cut = ids2.index(tok.special_ids["<|ans|>"])
    assert ids3[:cut] == ids2[:cut]


def test_record_answer_requires_prompt(tok):
    conv = Conversation(tok)
    with pytest.raises(RuntimeError):
        conv.record_answer("x")


def test_preserve_requires_config(tok):
    with pytest.raises(ValueError):
        Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY)


def test_template_kwargs_drift_raises(tok):
    conv = Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY, StubConfig(tok.control_token_ids()))
    conv.user("a")
    conv.build_prompt(adapter="uq")
    conv.record_answer(_ans(tok, "b"))
    conv.user("c")
    with pytest.raises(RuntimeError, match="documents"):
        conv.build_prompt(adapter="ans", documents=["doc"])


def test_control_budget_reprefill(tok):
    conv = Conversation(tok, KVHistoryPolicy.PRESERVE_MIXED_HISTORY, StubConfig(tok.control_token_ids()))
    n = 0
    while conv.reprefills == 0 and n < 400:
        conv.user("q")
        conv.build_prompt(adapter="uq" if n % 2 else "ans")
        conv.record_answer(_ans(tok, "a"))
        n += 1
    assert conv.reprefills == 1
    assert n - 1 == MAX_RETAINED_CONTROL_TOKENS


def test_completion_payload(tok):
    conv = Conversation(tok)
    conv.user("x")
    body = conv.completion_payload(adapter="uq", max_tokens=5)
    assert body["max_tokens"] == 5 and isinstance(body["prompt"], list)
