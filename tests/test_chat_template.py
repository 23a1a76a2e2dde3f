"""Adapter-aware chat template on the Granite 4.1 (role markers) and 4.2 (ChatML) templates.

The central property (reference: tests/composer/test_chat_template.py and
test_chat_template_real_tokenizer.py): after token exchange (each control id
replaced by its substitute id) an adapter render is id-for-id the base
model's own render, so only the switch sees the control token.
"""
import jinja2
import pytest

from granite_switch_b200.composer.chat_template import (
    CHATML_FORMAT,
    GRANITE_FORMAT,
    detect_template_format,
    generation_prompt_variants,
    render,
    resolve_sr_site,
)
from granite_switch_b200.composer.compose import AdapterSpec
from granite_switch_b200.composer.tokenizer_setup import (
    configure_tokenizer,
    encode,
    find_reserved_never_emitted_token_id,
    lora_substitute_token_id,
    resolve_label_token_ids,
)
from tests.tokenizer_stub import granite_template, make_tokenizer

VERSIONS = ["4.1", "4.2"]
HEADER = {"4.1": "<|start_of_role|>assistant<|end_of_role|>", "4.2": "<|im_start|>assistant\n"}
SR_ANCHOR = {"4.1": "<|end_of_role|>", "4.2": "</think>"}


def _setup(version, audio=False):
    base = granite_template(version)
    tok = make_tokenizer(base)
    adapters = [
        AdapterSpec("rw", {}, 8, 8.0, technology="lora"),
        AdapterSpec("req", {}, 8, 8.0, technology="alora", invocation_tokens=encode(tok, "<requirements>")),
        AdapterSpec("ans", {}, 8, 8.0, technology="alora", invocation_tokens=encode(tok, HEADER[version])),
        AdapterSpec("srx", {}, 8, 8.0, technology="sr", last_context_token=SR_ANCHOR[version]),
        AdapterSpec("pb", {}, 1, 1.0, technology="lora", kind="probe"),
    ]
    ids, setup = configure_tokenizer(tok, adapters, base_reset=True, audio=audio)
    ctrl = {a.name: i for a, i in zip(adapters, ids[1:])}
    return base, tok, adapters, ctrl, setup


def _exchange(ids, ctrl, adapters):
    sub = {ctrl[a.name]: a.substitute_token_id for a in adapters}
    return [sub.get(i, i) for i in ids]


CHATS = [
    [{"role": "user", "content": "Is the sky blue? <requirements> be brief"}],
    [{"role": "system", "content": "You are terse."},
     {"role": "user", "content": "first <requirements> a"},
     {"role": "assistant", "content": "ok"},
     {"role": "user", "content": "second <requirements> b <requirements> c"}],
]


def test_format_detection():
    assert detect_template_format(granite_template("4.1")) is GRANITE_FORMAT
    assert detect_template_format(granite_template("4.2")) is CHATML_FORMAT
    assert detect_template_format("{{ messages }}") is None


@pytest.mark.parametrize("version", VERSIONS)
def test_no_adapter_is_the_base_render(version):
    base, tok, _, _, _ = _setup(version)
    for msgs in CHATS:
        for agp in (True, False):
            want = render(base, msgs, add_generation_prompt=agp)
            assert render(tok.chat_template, msgs, add_generation_prompt=agp) == want
            assert render(tok.chat_template, msgs, add_generation_prompt=agp, adapter_name="nope") == want


@pytest.mark.parametrize("version", VERSIONS)
@pytest.mark.parametrize("name", ["rw", "req", "ans", "srx"])
def test_token_exchange_restores_the_base_ids(version, name):
    base, tok, adapters, ctrl, _ = _setup(version)
    for msgs in CHATS:
        out = render(tok.chat_template, msgs, add_generation_prompt=True, adapter_name=name)
        ids = encode(tok, out)
        assert ids.count(ctrl[name]) == 1, out
        assert _exchange(ids, ctrl, adapters) == encode(tok, render(base, msgs, add_generation_prompt=True))


@pytest.mark.parametrize("version", VERSIONS)
def test_placement_sites(version):
    base, tok, _, _, setup = _setup(version)
    msgs = CHATS[1]
    r = lambda **kw: render(tok.chat_template, msgs, add_generation_prompt=True, **kw)  # noqa: E731
    assert r(adapter_name="rw").startswith("<|rw|>")
    # aLoRA: the last user message's last invocation, first token's chars dropped
    out = r(adapter_name="req")
    assert "b <|req|>> c" in out and out.count("<|req|>") == 1
    assert setup.placements["req"].drop_chars == len("<requirements")
    # assistant-boundary invocation: the control token takes the generation prompt's marker
    marker = setup.format.role_open_marker
    assert r(adapter_name="ans").endswith("<|ans|>" + HEADER[version][len(marker):] +
                                          ("<think>\n" if version == "4.2" else ""))
    # no user message carries the invocation -> generation-prompt fallback
    plain = [{"role": "user", "content": "hello"}]
    out = render(tok.chat_template, plain, add_generation_prompt=True, adapter_name="req")
    assert out.rsplit("<|req|>", 1)[1] == render(base, plain, add_generation_prompt=True).rsplit(marker, 1)[1]
    # probe: very last token, no generation prompt
    out = r(adapter_name="pb")
    assert out == render(base, msgs, add_generation_prompt=False) + "<|pb|>"


def test_sr_site_resolution():
    assert resolve_sr_site(["<|start_of_role|>assistant<|end_of_role|>"], "<|end_of_role|>",
                           lambda s: encode(make_tokenizer(), s)).site == "<|end_of_role|>"
    tok = make_tokenizer()
    variants = generation_prompt_variants(granite_template("4.2"))
    assert sorted(variants) == sorted(["<|im_start|>assistant\n<think>\n", "<|im_start|>assistant\n<think></think>"])
    s = resolve_sr_site(variants, "</think>", lambda t: encode(tok, t))
    assert s.site == "<think>" and s.head == "<|im_start|>assistant\n"
    assert s.tails == ("<think></think>", "<think>\n")
    with pytest.raises(ValueError):
        resolve_sr_site(["<|start_of_role|>assistant<|end_of_role|>"], "</think>", lambda t: encode(tok, t))


@pytest.mark.parametrize("version", VERSIONS)
def test_sr_all_generation_paths_and_history(version):
    base, tok, adapters, ctrl, setup = _setup(version)
    msgs = [{"role": "user", "content": "q1"}, {"role": "assistant", "content": "a1"},
            {"role": "user", "content": "q2"}, {"role": "assistant", "content": "a2"},
            {"role": "user", "content": "q3"}]
    flag_sets = [{}] + ([{"enable_thinking": False}] if version == "4.2" else [])
    for flags in flag_sets:
        want = encode(tok, render(base, msgs, add_generation_prompt=True, **flags))
        out = render(tok.chat_template, msgs, add_generation_prompt=True, adapter_name="srx", **flags)
        assert out.count("<|srx|>") == 1
        assert _exchange(encode(tok, out), ctrl, adapters) == want
        hist = render(tok.chat_template, msgs, add_generation_prompt=True, adapter_name="srx",
                      history_adapters=["srx", None], **flags)
        assert hist.count("<|srx|>") == 2
        first_turn = hist.split(setup.sr_site.head)[1]
        assert first_turn.startswith("<|srx|>")
        assert _exchange(encode(tok, hist), ctrl, adapters) == want
    # history entries must line up with the assistant turns and name SR adapters
    for bad in (["srx"], ["rw", None], "srx"):
        with pytest.raises(jinja2.exceptions.TemplateError):
            render(tok.chat_template, msgs, add_generation_prompt=True, adapter_name="srx", history_adapters=bad)


@pytest.mark.parametrize("version", VERSIONS)
def test_parts_lists_and_audio(version):
    base, tok, _, _, _ = _setup(version, audio=True)
    parts = [{"role": "user", "content": [{"type": "text", "text": "Listen:"}, {"type": "audio", "audio": None},
                                          {"type": "text", "text": "what <requirements> now?"}]}]
    out = render(tok.chat_template, parts, add_generation_prompt=True)
    assert "Listen:<|audio|>\nwhat <requirements> now?" in out
    out = render(tok.chat_template, parts, add_generation_prompt=True, adapter_name="req")
    assert "Listen:<|audio|>\nwhat <|req|>> now?" in out
    # text-only parts render like the same text as one string
    text = [{"role": "user", "content": [{"type": "text", "text": "a"}, {"type": "text", "text": "b"}]}]
    assert render(tok.chat_template, text, add_generation_prompt=True) == render(
        base, [{"role": "user", "content": "a\nb"}], add_generation_prompt=True)


def test_transformers_apply_chat_template_and_tokens():
    base, tok, adapters, ctrl, setup = _setup("4.1")
    msgs = CHATS[0]
    out = tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True, adapter_name="rw")
    assert out == render(tok.chat_template, msgs, add_generation_prompt=True, adapter_name="rw")
    assert lora_substitute_token_id(tok, base) == tok.convert_tokens_to_ids("<|start_of_role|>")
    subs = {a.name: a.substitute_token_id for a in adapters}
    assert subs["rw"] == subs["pb"] == tok.convert_tokens_to_ids("<|start_of_role|>")
    assert subs["srx"] == tok.convert_tokens_to_ids("<|end_of_role|>")
    assert subs["req"] == tok.convert_tokens_to_ids("<requirements")
    assert find_reserved_never_emitted_token_id(tok) == tok.convert_tokens_to_ids("<|unused_1|>")
    assert resolve_label_token_ids(tok, ["Y", "N"]) == encode(tok, "YN")
    with pytest.raises(ValueError):
        resolve_label_token_ids(tok, ["yes"])


def test_unknown_template_family_is_rejected():
    tok = make_tokenizer("{% for m in messages %}{{ m.content }}{% endfor %}")
    with pytest.raises(ValueError):
        configure_tokenizer(tok, [AdapterSpec("rw", {}, 8, 8.0, technology="lora")])
