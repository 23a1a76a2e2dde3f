"""Tokenizer side of composition: control tokens, substitutes and the chat template.

* One special token ``<|name|>`` per adapter (a leading ``<|base_reset|>`` on
  request) is added to the base tokenizer; the ids it assigns become
  ``adapter_token_ids`` (reference: src/granite_switch/composer/tokenizer_setup.py:892-976).
* Each control token gets a substitute id: the token the control token stands
  in for in a rendered prompt, so after token exchange the decoder sees the
  base model's own input (reference: tokenizer_setup.py:1293-1333 and
  compose_granite_switch.py:151-213):
    - LoRA, built-in and base-reset: the token at position 0 of a no-adapter
      render (the role-open marker on Granite templates);
    - aLoRA: the first token of the adapter's ``alora_invocation_tokens``;
    - Shadow Residual: the generation-prompt token its control token replaces;
    - probe: the role-open marker.
* The base chat template is wrapped so ``adapter_name=...`` places the control
  token (see :mod:`.chat_template` for the four placement modes).
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field

from .chat_template import (
    Placement,
    SRSite,
    TemplateFormat,
    build_chat_template,
    detect_template_format,
    generation_prompt_variants,
    render,
    resolve_sr_site,
)
from .compose import AdapterSpec

BASE_RESET = "<|base_reset|>"
AUDIO_MARKER = "<|audio|>"
_UNUSED_RE = re.compile(r"^<\|unused_\d+\|>$")


def encode(tokenizer, text: str) -> list[int]:
    return list(tokenizer.encode(text, add_special_tokens=False))


def _special_tokens(tokenizer) -> list[str]:
    return list(getattr(tokenizer, "additional_special_tokens", None) or [])


def add_control_tokens(tokenizer, adapters: list[AdapterSpec], base_reset: bool = False) -> list[int]:
    """Add ``<|name|>`` special tokens; returns their ids in slot order (base-reset first)."""
    names = ([BASE_RESET] if base_reset else []) + [f"<|{a.name}|>" for a in adapters]
    if len(set(names)) != len(names):
        raise ValueError(f"duplicate adapter names: {names}")
    existing = _special_tokens(tokenizer)
    tokenizer.add_special_tokens({"additional_special_tokens": existing + [n for n in names if n not in existing]})
    ids = [tokenizer.convert_tokens_to_ids(n) for n in names]
    if len(set(ids)) != len(ids):
        raise ValueError(f"control tokens did not get distinct ids: {ids}")
    for n, i in zip(names, ids):
        if encode(tokenizer, n) != [i]:
            raise ValueError(f"control token {n} does not encode to its own id {i}")
    return ids


def add_audio_token(tokenizer, marker: str = AUDIO_MARKER) -> int:
    """Register the audio placeholder as one special token (existing specials kept); returns its id."""
    kept = [t for t in _special_tokens(tokenizer) if t != marker]
    tokenizer.add_special_tokens({"additional_special_tokens": kept + [marker]})
    return int(tokenizer.convert_tokens_to_ids(marker))


def find_reserved_never_emitted_token_id(tokenizer) -> int | None:
    """Highest id of a reserved ``<|unused_N|>`` token (a row the base never emits), or None."""
    ids = [i for t, i in tokenizer.get_vocab().items() if _UNUSED_RE.match(t)]
    return max(ids) if ids else None


def resolve_label_token_ids(tokenizer, labels: list[str]) -> list[int]:
    """Each probe label word must be exactly one token (the verdict writes one logit per label)."""
    out, bad = [], []
    for w in labels:
        ids = encode(tokenizer, w)
        if len(ids) != 1:
            bad.append(f"{w!r} -> {len(ids)} tokens")
        else:
            out.append(ids[0])
    if bad:
        raise ValueError("probe labels must be single tokens: " + ", ".join(bad))
    return out


def placement_mode(adapter: AdapterSpec) -> str:
    if adapter.kind == "probe":
        return "probe"
    if any(".cross_stream." in k for k in adapter.tensors) or adapter.technology == "sr":
        return "sr"
    if adapter.technology == "alora":
        return "alora"
    return "lora"


def activation_anchor(tokenizer, adapter: AdapterSpec) -> tuple[str, str]:
    """``(anchor_text, mode)`` from the adapter's config: ``alora_invocation_tokens``
    (decoded; mode alora) or ``last_context_token`` (one token, checked against
    ``last_context_token_id``; mode sr)."""
    if adapter.invocation_tokens:
        return tokenizer.decode(list(adapter.invocation_tokens), skip_special_tokens=False), "alora"
    if adapter.last_context_token:
        ids = encode(tokenizer, adapter.last_context_token)
        if len(ids) != 1:
            raise ValueError(f"{adapter.name}: last_context_token {adapter.last_context_token!r} encodes to "
                             f"{len(ids)} tokens; the control token replaces exactly one")
        if adapter.last_context_token_id is not None and adapter.last_context_token_id != ids[0]:
            raise ValueError(f"{adapter.name}: last_context_token {adapter.last_context_token!r} encodes to "
                             f"{ids[0]} but the adapter records {adapter.last_context_token_id}: it was "
                             f"trained with a different tokenizer")
        return adapter.last_context_token, "sr"
    raise ValueError(f"{adapter.name}: adapter_config.json carries neither alora_invocation_tokens nor "
                     f"last_context_token")


def base_template(tokenizer) -> str | None:
    t = tokenizer.chat_template
    if isinstance(t, dict):
        t = t.get("default") or next(iter(t.values()), None)
    return t or None


def lora_substitute_token_id(tokenizer, template: str | None = None) -> int:
    """The token at position 0 of a one-turn no-adapter render."""
    template = template or base_template(tokenizer)
    if template is None:
        raise ValueError("the tokenizer has no chat template to probe the LoRA substitute with")
    ids = encode(tokenizer, render(template, [{"role": "user", "content": "probe"}], add_generation_prompt=False))
    if not ids or ids[0] == tokenizer.unk_token_id:
        raise ValueError("the first token of a rendered chat is empty or unknown")
    return ids[0]


def role_marker_token_id(tokenizer, fmt: TemplateFormat) -> int:
    ids = encode(tokenizer, fmt.role_open_marker)
    if len(ids) != 1:
        raise ValueError(f"role-open marker {fmt.role_open_marker!r} is not one token")
    return ids[0]


@dataclass
class ChatTemplateSetup:
    format: TemplateFormat
    placements: dict[str, Placement]
    sr_site: SRSite | None
    substitutes: dict[str, int] = field(default_factory=dict)   # adapter name -> substitute id
    lora_substitute: int = 0


def configure_chat_template(tokenizer, adapters: list[AdapterSpec],
                            audio_marker: str | None = None) -> ChatTemplateSetup | None:
    """Install the adapter-aware chat template; None when the base has no template."""
    base = base_template(tokenizer)
    if base is None:
        return None
    fmt = detect_template_format(base)
    if fmt is None:
        raise ValueError("chat template uses neither <|im_start|> nor <|start_of_role|>: adapter control tokens "
                         "cannot be placed, so the composed checkpoint could never activate them")
    lora_sub = lora_substitute_token_id(tokenizer, base)
    placements: dict[str, Placement] = {}
    subs: dict[str, int] = {}
    sr_anchors: set[str] = set()
    for a in adapters:
        tok = f"<|{a.name}|>"
        mode = placement_mode(a)
        if mode == "probe":
            placements[a.name] = Placement(tok, "probe")
            subs[a.name] = role_marker_token_id(tokenizer, fmt)
        elif mode == "lora":
            placements[a.name] = Placement(tok, "lora")
            subs[a.name] = lora_sub
        else:
            text, found = activation_anchor(tokenizer, a)
            if mode == "sr" and found != "sr":
                raise ValueError(f"{a.name} is a Shadow Residual adapter (cross_stream weights) but its config "
                                 f"carries alora_invocation_tokens instead of last_context_token")
            if found == "sr":
                placements[a.name] = Placement(tok, "sr")
                sr_anchors.add(text)
            else:
                first = encode(tokenizer, text)[0]
                drop = len(tokenizer.decode([first], skip_special_tokens=False))
                placements[a.name] = Placement(tok, "alora", invocation_text=text, drop_chars=drop)
                subs[a.name] = int(a.invocation_tokens[0])
    site = None
    if sr_anchors:
        if len(sr_anchors) > 1:
            raise ValueError(f"Shadow Residual adapters of one checkpoint must share last_context_token, got "
                             f"{sorted(sr_anchors)}")
        site = resolve_sr_site(generation_prompt_variants(base), next(iter(sr_anchors)),
                               lambda s: encode(tokenizer, s))
        site_id = encode(tokenizer, site.site)[0]
        for n, p in placements.items():
            if p.mode == "sr":
                subs[n] = site_id
    tokenizer.chat_template = build_chat_template(base, fmt, placements, sr=site, audio_marker=audio_marker)
    return ChatTemplateSetup(fmt, placements, site, subs, lora_sub)


def configure_tokenizer(tokenizer, adapters: list[AdapterSpec], base_reset: bool = False,
                        audio: bool = False) -> tuple[list[int], ChatTemplateSetup | None]:
    """Add control (and audio) tokens, install the chat template and set each
    adapter's ``substitute_token_id``. Returns the control ids (slot order) and the setup."""
    ids = add_control_tokens(tokenizer, adapters, base_reset)
    marker = None
    if audio:
        add_audio_token(tokenizer)
        marker = AUDIO_MARKER
    setup = configure_chat_template(tokenizer, adapters, audio_marker=marker)
    if setup is not None:
        for a in adapters:
            if a.name in setup.substitutes:
                a.substitute_token_id = setup.substitutes[a.name]
    return ids, setup


__all__ = ["BASE_RESET", "AUDIO_MARKER", "add_control_tokens", "add_audio_token", "find_reserved_never_emitted_token_id",
           "resolve_label_token_ids", "placement_mode", "activation_anchor", "lora_substitute_token_id",
           "role_marker_token_id", "configure_chat_template", "configure_tokenizer", "ChatTemplateSetup",
           "base_template", "encode"]
