"""Tokenizer side of composition: control tokens and the adapter-aware chat template.

* One special token ``<|name|>`` per adapter (a leading ``<|base_reset|>`` on
  request) is added to the base tokenizer; the token ids it assigns become
  ``adapter_token_ids``.
* The base chat template is wrapped, not rewritten: the original template
  renders the conversation into a captured string, and the wrapper places the
  control token of ``adapter_name`` (a template kwarg, as in the reference,
  src/granite_switch/composer/tokenizer_setup.py:1360-) in it:
    - LoRA: at position 0 of the rendering (the adapter applies to the whole prompt);
    - aLoRA and Shadow-Residual: in place of the first token of the adapter's
      invocation sequence, at its last occurrence (normally the generation
      prompt). The control token's substitute id is that first token, so after
      token exchange the decoder sees exactly the base model's input, and the
      adapter takes over from its invocation on. If the invocation's first
      token does not occur, the control token is appended at the end.
  Templates of both families (Granite role markers and ChatML) work unchanged,
  since the wrapper only searches for the invocation text.
"""
from __future__ import annotations

import json

from .compose import AdapterSpec

BASE_RESET = "<|base_reset|>"


def add_control_tokens(tokenizer, adapters: list[AdapterSpec], base_reset: bool = False) -> list[int]:
    """Add ``<|name|>`` special tokens; returns their ids in slot order (base-reset first)."""
    names = ([BASE_RESET] if base_reset else []) + [f"<|{a.name}|>" for a in adapters]
    existing = list(getattr(tokenizer, "additional_special_tokens", []) or [])
    tokenizer.add_special_tokens({"additional_special_tokens": existing + [n for n in names if n not in existing]})
    ids = [tokenizer.convert_tokens_to_ids(n) for n in names]
    if len(set(ids)) != len(ids):
        raise ValueError(f"control tokens did not get distinct ids: {ids}")
    return ids


def invocation_anchor(tokenizer, adapter: AdapterSpec) -> str | None:
    """Text of the first invocation token (what the control token replaces)."""
    if not adapter.invocation_tokens:
        return None
    return tokenizer.decode([adapter.invocation_tokens[0]], skip_special_tokens=False)


def wrap_chat_template(base_template: str, adapters: list[AdapterSpec], anchors: dict[str, str | None]) -> str:
    ctrl = {a.name: f"<|{a.name}|>" for a in adapters}
    kind = {a.name: ("lora" if a.technology == "lora" or not anchors.get(a.name) else "alora") for a in adapters}
    anchor = {a.name: anchors.get(a.name) or "" for a in adapters}
    return (
        "{%- set _gs_ctrl = " + json.dumps(ctrl) + " -%}\n"
        "{%- set _gs_kind = " + json.dumps(kind) + " -%}\n"
        "{%- set _gs_anchor = " + json.dumps(anchor) + " -%}\n"
        "{%- set _gs_render -%}" + base_template + "{%- endset -%}\n"
        "{%- if adapter_name is defined and adapter_name and adapter_name in _gs_ctrl -%}\n"
        "{%- if _gs_kind[adapter_name] == 'lora' -%}{{ _gs_ctrl[adapter_name] ~ _gs_render }}\n"
        "{%- else -%}{%- set _gs_parts = _gs_render.rsplit(_gs_anchor[adapter_name], 1) -%}\n"
        "{%- if _gs_parts | length == 2 -%}{{ _gs_parts[0] ~ _gs_ctrl[adapter_name] ~ _gs_parts[1] }}\n"
        "{%- else -%}{{ _gs_render ~ _gs_ctrl[adapter_name] }}{%- endif -%}\n"
        "{%- endif -%}\n"
        "{%- else -%}{{ _gs_render }}{%- endif -%}"
    )


def configure_tokenizer(tokenizer, adapters: list[AdapterSpec], base_reset: bool = False) -> list[int]:
    """Add control tokens and install the wrapped chat template; returns the control ids."""
    ids = add_control_tokens(tokenizer, adapters, base_reset)
    base = tokenizer.chat_template
    if isinstance(base, dict):
        base = base.get("default") or next(iter(base.values()))
    if base:
        anchors = {a.name: invocation_anchor(tokenizer, a) for a in adapters}
        tokenizer.chat_template = wrap_chat_template(base, adapters, anchors)
    return ids
