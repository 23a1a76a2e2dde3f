"""Adapter-aware chat template: where each adapter's control token goes.

A composed checkpoint ships one chat template that places the control token
of ``adapter_name`` (a template kwarg) in the rendered prompt, and restores
Shadow-Residual control tokens in history turns named by ``history_adapters``
(reference behaviour: src/granite_switch/composer/tokenizer_setup.py:1360-1963
and :672-889). Four placement modes:

* ``lora``  - the control token is the first token of the prompt and stands in
  for the role-open marker that would have been there (the marker is dropped,
  the control token's substitute id is that marker);
* ``alora`` - the control token goes right before the adapter's invocation
  text, at its last occurrence in the last user message containing it, and the
  first invocation token's characters are dropped after it (the control token's
  substitute is that first token). When no user message contains the text
  (the invocation is the assistant header), the control token takes the place of
  the generation prompt's role-open marker, or ends the prompt without one;
* ``sr``    - the control token replaces one token (the *site*) inside the
  generation prompt; the site is the adapter's ``last_context_token`` when every
  generation-prompt variant contains it, else the last single token of the
  variants' common prefix;
* ``probe`` - the control token is the very last token, after the last turn's
  close; the generation prompt is suppressed.

Design: instead of patching the base template's source at anchors that
differ between template families, the wrapper (1) rewrites the message list
(aLoRA insertion, content-part flattening for ChatML, audio parts to the audio
marker) and rebinds ``messages``, (2) renders the unmodified base template into
a string, and (3) places the control token in that string. Everything it needs
from the base template is found by rendering it (:func:`generation_prompt_variants`),
so the same code serves the Granite role-marker family and ChatML. The wrapper
is plain Jinja and renders in the immutable sandbox transformers and vLLM use.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

MODES = ("lora", "alora", "sr", "probe")

#: Characters a substitution site may not contain (they would straddle an
#: escape in the template source of the base model; the reference applies the
#: same rule, tokenizer_setup.py:419-422).
_SITE_FORBIDDEN = set("\\\n\r\t'\"")

#: Template kwargs whose value can change the generation prompt of a Granite
#: template (Granite 4.2: ``enable_thinking``).
GENERATION_FLAGS = ("enable_thinking", "thinking", "reasoning")


@dataclass(frozen=True)
class TemplateFormat:
    """A chat-template family: its role-open marker and whether message content
    must be flattened to a string before the base template sees it."""
    name: str
    role_open_marker: str
    flatten_content: bool


GRANITE_FORMAT = TemplateFormat("granite_format", "<|start_of_role|>", False)
CHATML_FORMAT = TemplateFormat("chatml", "<|im_start|>", True)


def detect_template_format(template: str | None) -> TemplateFormat | None:
    """``<|im_start|>`` -> ChatML (checked first), ``<|start_of_role|>`` -> Granite, else None."""
    if not template:
        return None
    if "<|im_start|>" in template:
        return CHATML_FORMAT
    if "<|start_of_role|>" in template:
        return GRANITE_FORMAT
    return None


@dataclass(frozen=True)
class Placement:
    """Where one adapter's control token goes."""
    token: str
    mode: str
    invocation_text: str = ""
    drop_chars: int = 0

    def __post_init__(self):
        if self.mode not in MODES:
            raise ValueError(f"unknown placement mode {self.mode!r}")
        if self.mode == "alora" and not self.invocation_text:
            raise ValueError(f"aLoRA placement of {self.token} needs its invocation text")


@dataclass(frozen=True)
class SRSite:
    """The generation-prompt token a Shadow-Residual control token replaces.

    ``head`` is the assistant header up to the site (history turns render it
    too) and ``tails`` the generation-prompt variants after ``head``, each
    starting with ``site``, longest first: a history turn is rewritten only
    when its text after ``head`` starts with one of them.
    """
    site: str
    head: str
    tails: tuple[str, ...]


# ---------------------------------------------------------------- rendering
def make_environment():
    """The Jinja environment chat templates are rendered with (transformers' settings)."""
    import jinja2
    from jinja2.ext import loopcontrols
    from jinja2.sandbox import ImmutableSandboxedEnvironment

    class _Generation(jinja2.ext.Extension):
        """Accept HF's ``{% generation %}`` block (renders its body)."""
        tags = {"generation"}

        def parse(self, parser):
            next(parser.stream)
            body = parser.parse_statements(("name:endgeneration",), drop_needle=True)
            return jinja2.nodes.Scope(body)

    env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True,
                                        extensions=[loopcontrols, _Generation])

    def raise_exception(message):
        raise jinja2.exceptions.TemplateError(message)

    env.globals["raise_exception"] = raise_exception
    env.filters.setdefault("tojson", lambda x, **kw: json.dumps(x, **kw))
    return env


def render(template: str, messages: list, **kwargs) -> str:
    kwargs.setdefault("add_generation_prompt", False)
    return make_environment().from_string(template).render(messages=messages, **kwargs)


def generation_prompt_variants(template: str) -> list[str]:
    """Every distinct generation prompt the template renders, found by rendering
    a one-turn chat with and without ``add_generation_prompt`` under each value
    of the generation flags the template reads."""
    msgs = [{"role": "user", "content": "hello"}]
    flag_sets = [{}]
    for f in GENERATION_FLAGS:
        if f in template:
            flag_sets += [{f: True}, {f: False}]
    out: list[str] = []
    for flags in flag_sets:
        without = render(template, msgs, add_generation_prompt=False, **flags)
        with_gp = render(template, msgs, add_generation_prompt=True, **flags)
        if not with_gp.startswith(without):
            raise ValueError("the generation prompt is not a suffix of the rendered chat "
                             f"(flags {flags}); cannot locate it")
        gp = with_gp[len(without):]
        if gp and gp not in out:
            out.append(gp)
    if not out:
        raise ValueError("the chat template renders no generation prompt")
    return out


def resolve_sr_site(variants: list[str], anchor: str, encode) -> SRSite:
    """Pick the token a Shadow-Residual control token replaces in every variant.

    ``encode(text) -> list[int]`` is the tokenizer without special tokens. The
    anchor is used when every variant contains it once; otherwise the site is
    the longest single-token suffix (starting on a token boundary) of the
    variants' common prefix: a control token carries one substitute embedding,
    so it must replace the same token on every render path.
    """
    if all(v.count(anchor) == 1 for v in variants):
        site = anchor
    elif len(variants) == 1:
        raise ValueError(f"the generation prompt {variants[0]!r} does not contain the adapter's "
                         f"last_context_token {anchor!r} exactly once")
    else:
        prefix = os.path.commonprefix(variants)
        prefix_ids = encode(prefix)
        site = None
        for cut in range(len(prefix)):
            cand = prefix[cut:]
            if _SITE_FORBIDDEN & set(cand):
                continue
            cand_ids = encode(cand)
            if len(cand_ids) != 1:
                continue
            lead = prefix[:cut]
            if (encode(lead) if lead else []) + cand_ids == prefix_ids:
                site = cand
                break
        if site is None:
            raise ValueError(f"the generation prompt variants {variants!r} share no single token that could "
                             f"stand in for last_context_token {anchor!r}")
        if any(v.count(site) != 1 for v in variants):
            raise ValueError(f"substitution site {site!r} occurs more than once in {variants!r}")
    if len(encode(site)) != 1:
        raise ValueError(f"substitution site {site!r} is not a single token")
    prefix = os.path.commonprefix(variants)
    cut = prefix.rfind(site)
    if cut < 0:
        raise ValueError(f"the variants {variants!r} share no prefix containing {site!r}")
    head = prefix[:cut]
    tails = tuple(sorted({v[len(head):] for v in variants}, key=len, reverse=True))
    return SRSite(site=site, head=head, tails=tails)


# ---------------------------------------------------------------- the wrapper
def _lit(s: str) -> str:
    """A Jinja string literal rendering to ``s`` (JSON string syntax is valid Jinja)."""
    return json.dumps(s)


def build_chat_template(base: str, fmt: TemplateFormat, placements: dict[str, Placement], *,
                        sr: SRSite | None = None, audio_marker: str | None = None) -> str:
    """Wrap ``base`` so ``adapter_name`` / ``history_adapters`` place control tokens.

    Without ``adapter_name`` (or with a name that is not an adapter of the
    checkpoint) and without audio parts the output equals the base template's.
    """
    if any(p.mode == "sr" for p in placements.values()) and sr is None:
        raise ValueError("Shadow-Residual placements need the resolved SRSite")
    table = {n: {"token": p.token, "mode": p.mode, "inv": p.invocation_text, "drop": p.drop_chars}
             for n, p in placements.items()}
    mk = _lit(fmt.role_open_marker)
    flatten = fmt.flatten_content
    audio = audio_marker is not None
    t = []
    a = t.append
    a("{#- adapter control-token placement: adapter_name=..., history_adapters=[...] -#}\n")
    a("{%- set _gs_map = " + json.dumps(table) + " %}\n")
    a("{%- set _gs = namespace(tok='', mode='', inv='', drop=0, target=-1, msgs=[]) %}\n")
    a("{%- if adapter_name is defined and adapter_name is string and adapter_name in _gs_map %}"
      "{%- set _gs.tok = _gs_map[adapter_name]['token'] %}"
      "{%- set _gs.mode = _gs_map[adapter_name]['mode'] %}"
      "{%- set _gs.inv = _gs_map[adapter_name]['inv'] %}"
      "{%- set _gs.drop = _gs_map[adapter_name]['drop'] %}"
      "{%- endif %}\n")
    # a probe reads its verdict at the marker: nothing may follow it
    a("{%- if _gs.mode == 'probe' %}{%- set add_generation_prompt = false %}{%- endif %}\n")
    # aLoRA: the last user message containing the invocation text
    a("{%- if _gs.mode == 'alora' %}{%- for _m in messages %}{%- if _m.role == 'user' %}"
      "{%- if _m.content is string %}{%- if _gs.inv in _m.content %}{%- set _gs.target = loop.index0 %}"
      "{%- endif %}"
      "{%- elif _m.content is iterable and _m.content is not mapping %}{%- set _i = loop.index0 %}"
      "{%- for _e in _m.content %}{%- if _e.type is defined and _e.type == 'text' and _gs.inv in _e.text %}"
      "{%- set _gs.target = _i %}{%- endif %}{%- endfor %}"
      "{%- endif %}{%- endif %}{%- endfor %}{%- endif %}\n")
    # message rewrite: content flattening / audio markers / aLoRA insertion
    a("{%- for _m in messages %}{%- set _w = namespace(c=_m.content, changed=false) %}")
    a("{%- if _w.c is not string and _w.c is iterable and _w.c is not mapping %}")
    if flatten:
        # text parts newline-joined, other parts dropped (audio: the marker; the
        # leading system message drops audio like the reference's preamble does)
        a("{%- set _f = namespace(val='') %}{%- set _sys0 = loop.first and _m.role == 'system' %}"
          "{%- for _e in _w.c %}")
        if audio:
            a("{%- if _e.type is defined and 'audio' in _e.type and not _sys0 %}"
              "{%- set _f.val = _f.val ~ " + _lit(audio_marker) + " %}{%- elif")
        else:
            a("{%- if")
        a(" _e.type is defined and _e.type == 'text' %}{%- if _f.val != '' %}{%- set _f.val = _f.val ~ '\\n' %}"
          "{%- endif %}{%- set _f.val = _f.val ~ _e.text %}{%- endif %}{%- endfor %}"
          "{%- set _w.c = _f.val %}{%- set _w.changed = true %}")
    elif audio:
        # the template joins text parts with newlines and drops the rest: an audio
        # marker is appended to the text part before it (or opens one), so the
        # joined text is the parts' texts with each marker where its clip sat
        a("{%- set _p = namespace(parts=[], pend=none, any=false) %}{%- for _e in _w.c %}"
          "{%- if _e.type is defined and 'audio' in _e.type %}{%- set _p.any = true %}"
          "{%- if _p.pend is none %}{%- set _p.pend = {'type': 'text', 'text': " + _lit(audio_marker) + "} %}"
          "{%- else %}{%- set _p.pend = dict(_p.pend, text=_p.pend.text ~ " + _lit(audio_marker) + ") %}"
          "{%- endif %}"
          "{%- elif _e.type is defined and _e.type == 'text' %}"
          "{%- if _p.pend is not none %}{%- set _p.parts = _p.parts + [_p.pend] %}{%- endif %}"
          "{%- set _p.pend = _e %}"
          "{%- else %}{%- set _p.parts = _p.parts + [_e] %}{%- endif %}{%- endfor %}"
          "{%- if _p.pend is not none %}{%- set _p.parts = _p.parts + [_p.pend] %}{%- endif %}"
          "{%- if _p.any %}{%- set _w.c = _p.parts %}{%- set _w.changed = true %}{%- endif %}")
    a("{%- endif %}")
    a("{%- if loop.index0 == _gs.target %}{%- set _w.changed = true %}"
      "{%- if _w.c is string %}{%- set _s = _w.c.rsplit(_gs.inv, 1) %}"
      "{%- set _w.c = _s[0] ~ _gs.tok ~ _gs.inv[_gs.drop:] ~ _s[1] %}"
      "{%- else %}{%- set _q = namespace(last=-1, parts=[]) %}"
      "{%- for _e in _w.c %}{%- if _e.type is defined and _e.type == 'text' and _gs.inv in _e.text %}"
      "{%- set _q.last = loop.index0 %}{%- endif %}{%- endfor %}"
      "{%- for _e in _w.c %}{%- if loop.index0 == _q.last %}{%- set _s = _e.text.rsplit(_gs.inv, 1) %}"
      "{%- set _q.parts = _q.parts + [dict(_e, text=_s[0] ~ _gs.tok ~ _gs.inv[_gs.drop:] ~ _s[1])] %}"
      "{%- else %}{%- set _q.parts = _q.parts + [_e] %}{%- endif %}{%- endfor %}"
      "{%- set _w.c = _q.parts %}{%- endif %}{%- endif %}")
    a("{%- if _w.changed %}{%- set _gs.msgs = _gs.msgs + [dict(_m, content=_w.c)] %}"
      "{%- else %}{%- set _gs.msgs = _gs.msgs + [_m] %}{%- endif %}{%- endfor %}\n")
    a("{%- set messages = _gs.msgs %}\n")
    # the unmodified base template, rendered into a string
    a("{%- set _gs_out %}" + base + "{% endset %}\n")
    # placement in the rendered text
    a("{%- set _gs_mk = " + mk + " %}\n")
    a("{%- if _gs.mode == 'lora' %}{{- _gs.tok ~ _gs_out.replace(_gs_mk, '', 1) }}\n")
    a("{%- elif _gs.mode == 'alora' and _gs.target == -1 %}"
      "{%- if add_generation_prompt and _gs_mk in _gs_out %}{%- set _s = _gs_out.rsplit(_gs_mk, 1) %}"
      "{{- _s[0] ~ _gs.tok ~ _s[1] }}{%- else %}{{- _gs_out ~ _gs.tok }}{%- endif %}\n")
    a("{%- elif _gs.mode == 'probe' %}{{- _gs_out ~ _gs.tok }}\n")
    if sr is not None:
        a(_sr_branch(sr))
    a("{%- else %}{{- _gs_out }}{%- endif %}")
    return "".join(t)


def _sr_branch(sr: SRSite) -> str:
    site, head = _lit(sr.site), _lit(sr.head)
    tails = " or ".join(f"_p.startswith({_lit(x)})" for x in sr.tails)
    n = len(sr.site)
    return (
        "{%- elif _gs.mode == 'sr' %}"
        "{%- set _r = namespace(pre=_gs_out, gp='', out='') %}"
        "{%- if add_generation_prompt and _gs_mk in _gs_out %}{%- set _s = _gs_out.rsplit(_gs_mk, 1) %}"
        "{%- set _r.pre = _s[0] %}{%- set _r.gp = (_gs_mk ~ _s[1]).replace(" + site + ", _gs.tok, 1) %}{%- endif %}"
        # history_adapters: one entry (an SR adapter name or none) per assistant message
        "{%- if history_adapters is defined and history_adapters is not none %}"
        "{%- if history_adapters is string or history_adapters is mapping or history_adapters is not iterable %}"
        "{{- raise_exception('history_adapters must be a list with one adapter name (or none) per assistant "
        "message') }}{%- endif %}"
        "{%- set _na = messages | selectattr('role', 'equalto', 'assistant') | list | length %}"
        "{%- if history_adapters | length != _na %}"
        "{{- raise_exception('history_adapters has ' ~ (history_adapters | length) ~ ' entries for ' ~ _na ~ "
        "' assistant messages') }}{%- endif %}"
        "{%- for _h in history_adapters %}{%- if _h is not none and (_h is not string or _h not in _gs_map or "
        "_gs_map[_h]['mode'] != 'sr') %}"
        "{{- raise_exception('history_adapters names ' ~ _h ~ ', which is not a Shadow Residual adapter of "
        "this checkpoint') }}{%- endif %}{%- endfor %}"
        "{%- set _parts = _r.pre.split(" + head + ") %}"
        "{%- if _parts | length - 1 == _na %}"
        "{%- for _p in _parts %}{%- if loop.first %}{%- set _r.out = _p %}{%- else %}"
        "{%- set _h = history_adapters[loop.index0 - 1] %}"
        "{%- if _h is not none and (" + tails + ") %}"
        "{%- set _r.out = _r.out ~ " + head + " ~ _gs_map[_h]['token'] ~ _p[" + str(n) + ":] %}"
        "{%- else %}{%- set _r.out = _r.out ~ " + head + " ~ _p %}{%- endif %}"
        "{%- endif %}{%- endfor %}{%- set _r.pre = _r.out %}{%- endif %}"
        "{%- endif %}"
        "{{- _r.pre ~ _r.gp }}\n"
    )


__all__ = ["TemplateFormat", "GRANITE_FORMAT", "CHATML_FORMAT", "detect_template_format", "Placement", "SRSite",
           "make_environment", "render", "generation_prompt_variants", "resolve_sr_site", "build_chat_template",
           "MODES", "GENERATION_FLAGS"]
