"""Adapter-aware chat-template wrapping (rendered with jinja2's sandbox, as transformers does)."""
import jinja2
from jinja2.sandbox import ImmutableSandboxedEnvironment

from granite_switch_b200.composer.compose import AdapterSpec
from granite_switch_b200.composer.tokenizer_setup import wrap_chat_template

GRANITE_LIKE = (
    "{%- for m in messages -%}<|start_of_role|>{{ m['role'] }}<|end_of_role|>{{ m['content'] }}<|end_of_text|>\n"
    "{%- endfor -%}{%- if add_generation_prompt -%}<|start_of_role|>assistant<|end_of_role|>{%- endif -%}")
CHATML_LIKE = (
    "{%- for m in messages -%}<|im_start|>{{ m['role'] }}\n{{ m['content'] }}<|im_end|>\n{%- endfor -%}"
    "{%- if add_generation_prompt -%}<|im_start|>assistant\n{%- endif -%}")


def _render(tpl, msgs, **kw):
    env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True, undefined=jinja2.Undefined)
    return env.from_string(tpl).render(messages=msgs, add_generation_prompt=True, **kw)


def _adapters():
    return [AdapterSpec("ans", {}, 8, 8.0, technology="alora", invocation_tokens=[1, 2]),
            AdapterSpec("rw", {}, 8, 8.0, technology="lora")]


def test_alora_replaces_first_invocation_token_granite():
    tpl = wrap_chat_template(GRANITE_LIKE, _adapters(), {"ans": "<|start_of_role|>", "rw": None})
    msgs = [{"role": "user", "content": "hi"}]
    base = _render(tpl, msgs)
    assert base == _render(GRANITE_LIKE, msgs)
    out = _render(tpl, msgs, adapter_name="ans")
    assert out.endswith("<|ans|>assistant<|end_of_role|>")
    assert out.count("<|start_of_role|>") == base.count("<|start_of_role|>") - 1


def test_lora_goes_first_and_chatml_anchor():
    tpl = wrap_chat_template(CHATML_LIKE, _adapters(), {"ans": "<|im_start|>", "rw": None})
    msgs = [{"role": "user", "content": "hi"}]
    assert _render(tpl, msgs, adapter_name="rw").startswith("<|rw|><|im_start|>user")
    plain = _render(CHATML_LIKE, msgs)
    head, tail = plain.rsplit("<|im_start|>", 1)
    assert _render(tpl, msgs, adapter_name="ans") == head + "<|ans|>" + tail
    assert _render(tpl, msgs, adapter_name="unknown") == _render(CHATML_LIKE, msgs)
