"""Multi-turn conversations whose turns may each use a different adapter, as token ids.

Why ids: a control token exists only in the token ids a chat-template render
produced; the message texts carry none. Re-rendering a conversation from its
messages therefore drops earlier turns' control tokens, re-routes those
positions to the base model and makes their cached KV unreachable. This module
builds prompts from the ids already sent plus the new turn, so earlier regions
keep their adapter and the server's token-keyed prefix cache keeps hitting.

Public surface (same as the reference, src/granite_switch/conversation.py:98-737):
``Conversation``, ``KVHistoryPolicy``, ``PromptTokenIds``,
``MAX_RETAINED_CONTROL_TOKENS``.

How a turn is built. ``prev`` is the render of the already-sent messages (with
the template kwargs they were sent with), ``full`` the render of all messages
plus a generation prompt with this turn's adapter. When ``full`` extends
``prev`` and this turn's control token lies in the added text, the new ids are
``sent + encode(full - prev)``; the added text must start on a special token
(``<|``) so no tokenizer merge can cross the seam. Otherwise the turn is a
re-prefill (a full render; earlier control tokens are dropped) when a render
without the adapter still extends ``prev`` (the control token just landed in
the sent prefix, as a LoRA token at position 0 does), and an error when the
template itself rewrote history or the kwargs drifted.

``RE_PREFILL`` keeps the conversation in its base form: history is re-rendered
without adapters, but the base-form ids of history already sent are reused
verbatim (lagging one turn), so that prefix still hits the cache.

``MAX_RETAINED_CONTROL_TOKENS`` (188) is the reference's bf16 counting-head
limit. This runtime routes exactly at any count, but the budget is kept so a
conversation built here behaves identically when served by the reference.
"""
from __future__ import annotations

import logging
from enum import Enum

__all__ = ["MAX_RETAINED_CONTROL_TOKENS", "Conversation", "KVHistoryPolicy", "PromptTokenIds"]

logger = logging.getLogger(__name__)

MAX_RETAINED_CONTROL_TOKENS = 188


class KVHistoryPolicy(Enum):
    """``RE_PREFILL``: history re-rendered in base form each turn (the default).
    ``PRESERVE_MIXED_HISTORY``: the ids already sent are kept, control tokens included."""

    RE_PREFILL = "re_prefill"
    PRESERVE_MIXED_HISTORY = "preserve_mixed_history"


class PromptTokenIds(list):
    """``list[int]`` returned by :meth:`Conversation.build_prompt`, tagged with its policy.

    These ids must reach the server as ids (``/v1/completions`` with a token-id
    prompt): a server-side re-render produces a different prefix and silently
    loses the cache reuse.
    """

    __slots__ = ("policy",)

    def __init__(self, ids, policy):
        super().__init__(ids)
        self.policy = policy

    @property
    def requires_token_ids(self) -> bool:
        return True


class Conversation:
    """A conversation that remembers which adapter produced which region of its ids.

    Args:
        tokenizer: tokenizer of a composed checkpoint (control tokens + adapter-aware
            chat template accepting ``adapter_name``).
        policy: :class:`KVHistoryPolicy` (default ``RE_PREFILL``).
        config: the checkpoint config (``adapter_token_ids``); required for
            ``PRESERVE_MIXED_HISTORY`` because the control-token budget reads it.
    """

    def __init__(self, tokenizer, policy=KVHistoryPolicy.RE_PREFILL, config=None):
        self.tokenizer = tokenizer
        self.policy = policy
        self.config = config
        if policy is KVHistoryPolicy.PRESERVE_MIXED_HISTORY and config is None:
            raise ValueError(
                "PRESERVE_MIXED_HISTORY needs config=<the checkpoint config>: its control-token "
                "budget guard reads adapter_token_ids, and without it a long conversation could "
                "exceed what the reference's switch addresses exactly."
            )
        self._control_ids = set(getattr(config, "adapter_token_ids", None) or [])
        self._control_strings = None
        self._msgs: list[dict] = []
        self._n_committed = 0            # messages represented in the sent ids
        self._sent: list[int] = []       # PRESERVE: ids already sent, verbatim
        self._sent_kwargs: dict = {}
        self._pending: list[int] | None = None
        self._pending_kwargs: dict = {}
        self._pending_adapter = None
        self._turn_adapters: list = []
        self._emitted_controls: list = []
        self._reprefills = 0
        # RE_PREFILL reuse: base-form ids of committed history (+ the text they render)
        self._base_ids: list[int] | None = None
        self._base_text: str | None = None
        self._next_base: tuple[list[int] | None, str | None] = (None, None)

    # ------------------------------------------------------------------ transcript
    def user(self, content, **fields):
        self._msgs.append({"role": "user", "content": content, **fields})

    def system(self, content):
        self._msgs.append({"role": "system", "content": content})

    @property
    def messages(self):
        """Role/content dicts (display view; under PRESERVE the ids are what is sent)."""
        return [dict(m) for m in self._msgs]

    @property
    def sent_token_ids(self):
        return list(self._sent)

    @property
    def reprefills(self) -> int:
        """Turns rebuilt as full renders (history's control tokens dropped)."""
        return self._reprefills

    @property
    def generated_control_tokens(self):
        """Per recorded answer: control ids the model emitted ([]), or None if recorded as text."""
        return [None if x is None else list(x) for x in self._emitted_controls]

    # ------------------------------------------------------------------ prompts
    def build_prompt(self, adapter=None, **template_kwargs) -> PromptTokenIds:
        """Token ids for the next assistant turn (``adapter`` = name or None for base).

        Does not change the transcript until :meth:`record_answer`.
        """
        if self.policy is KVHistoryPolicy.RE_PREFILL:
            ids = self._prompt_base_form(adapter, template_kwargs)
        elif not self._sent:
            ids = self._encode(self._render(self._msgs, True, adapter, template_kwargs))
        else:
            ids = self._prompt_preserved(adapter, template_kwargs)
        self._check_budget(ids)
        self._pending = ids
        self._pending_adapter = adapter
        self._pending_kwargs = dict(template_kwargs)
        return PromptTokenIds(ids, self.policy)

    def _prompt_preserved(self, adapter, kw):
        prev = self._render(self._msgs[: self._n_committed], False, None, self._sent_kwargs)
        full = self._render(self._msgs, True, adapter, kw)
        if self._can_append(full, prev):
            added = full[len(prev):]
            self._check_seam(added)
            ids = self._sent + self._encode(added)
            n = self._count_controls(ids)
            if n > MAX_RETAINED_CONTROL_TOKENS:
                ids = self._full_render_reset(adapter, kw, len(ids),
                                              f"{n} control tokens exceed {MAX_RETAINED_CONTROL_TOKENS}")
            return ids
        if self._render(self._msgs, True, None, kw).startswith(prev):
            return self._full_render_reset(adapter, kw, len(self._sent),
                                           "this turn's control token falls inside the sent prefix")
        self._raise_kwargs_drift(kw)
        self._raise_not_append_only()

    def _prompt_base_form(self, adapter, kw):
        committed = self._msgs[: self._n_committed]
        full = self._render(self._msgs, True, adapter, kw)
        if not committed:
            self._next_base = (None, None)
            return self._encode(full)
        base_hist = self._render(committed, False, None, kw)
        if not self._can_append(full, base_hist):
            self._next_base = (None, None)
            return self._encode(full)
        tail = full[len(base_hist):]
        self._check_seam(tail)
        if self._base_text is not None and base_hist.startswith(self._base_text):
            joined = base_hist[len(self._base_text):]
            if joined:
                self._check_seam(joined)
            prefix = self._base_ids + self._encode(joined)
        else:
            prefix = self._encode(base_hist)
        self._next_base = (prefix, base_hist)
        return prefix + self._encode(tail)

    def completion_payload(self, adapter=None, **extra) -> dict:
        """A ``/v1/completions`` body whose ``prompt`` is the token ids of the next turn."""
        return {"prompt": list(self.build_prompt(adapter=adapter)), **extra}

    def record_answer(self, answer, adapter=None) -> str:
        """Record the reply to the last built prompt (token ids preferred over text)."""
        if self._pending is None:
            raise RuntimeError("record_answer() needs a preceding build_prompt(): nothing records what was sent")
        if isinstance(answer, str):
            text, ids = answer, None
        else:
            ids = [int(t) for t in answer]
            text = self.tokenizer.decode(ids, skip_special_tokens=True)
        self._msgs.append({"role": "assistant", "content": text})
        self._turn_adapters.append(adapter)
        self._n_committed = len(self._msgs)
        self._emitted_controls.append(None if ids is None else [t for t in ids if t in self._control_ids])
        if self.policy is KVHistoryPolicy.PRESERVE_MIXED_HISTORY:
            body = ids if ids is not None else self._encode(text)
            self._sent = list(self._pending) + body + self._encode(self._turn_terminator())
            self._sent_kwargs = dict(self._pending_kwargs)
        else:
            self._base_ids, self._base_text = self._next_base
        self._pending = None
        return text

    # ------------------------------------------------------------------ helpers
    def _render(self, msgs, gen, adapter, kw):
        args = dict(kw)
        if adapter:
            args["adapter_name"] = adapter
        return self.tokenizer.apply_chat_template(msgs, add_generation_prompt=gen, tokenize=False, **args)

    def _encode(self, text):
        return list(self.tokenizer(text, add_special_tokens=False)["input_ids"])

    def _full_render_reset(self, adapter, kw, old_len, why):
        ids = self._encode(self._render(self._msgs, True, adapter, kw))
        self._reprefills += 1
        logger.warning("re-prefilled (%s): history's control tokens dropped; %d ids instead of %d "
                       "(re-prefills so far: %d)", why, len(ids), old_len, self._reprefills)
        return ids

    def _count_controls(self, ids):
        return sum(1 for t in ids if t in self._control_ids) if self._control_ids else 0

    def _check_budget(self, ids):
        n = self._count_controls(ids)
        if n > MAX_RETAINED_CONTROL_TOKENS:
            raise RuntimeError(
                f"{n} control tokens in one request exceed {MAX_RETAINED_CONTROL_TOKENS}; this prompt is "
                "already a full render, so the count comes from the current turn or from control-token "
                "text recorded into a message")

    def _control_texts(self):
        if self._control_strings is None:
            out = []
            for tid in sorted(self._control_ids):
                try:
                    s = self.tokenizer.convert_ids_to_tokens(tid)
                except Exception:
                    s = None
                if s:
                    out.append(s)
            self._control_strings = out
        return self._control_strings

    def _can_append(self, full, prev):
        """``full`` extends ``prev`` and this turn's control token (if any) is in the added text."""
        if not full.startswith(prev):
            return False
        where = [full.find(t) for t in self._control_texts()]
        where = [w for w in where if w >= 0]
        return not where or min(where) >= len(prev)

    @staticmethod
    def _check_seam(text):
        if not text.startswith("<|"):
            raise RuntimeError(
                f"the appended turn must start on a special token so tokenizer merges cannot cross the "
                f"join; the template produced {text[:32]!r}. Use KVHistoryPolicy.RE_PREFILL.")

    def _turn_terminator(self):
        probe = [{"role": "user", "content": ""}, {"role": "assistant", "content": ""}]
        both = self._render(probe, False, None, self._pending_kwargs)
        opener = self._render(probe[:1], True, None, self._pending_kwargs)
        if not both.startswith(opener):
            raise RuntimeError(
                "cannot derive the assistant-turn terminator from this chat template (a user+assistant "
                "render does not extend the user render plus generation prompt); use RE_PREFILL")
        return both[len(opener):]

    def _raise_kwargs_drift(self, kw):
        if kw == self._sent_kwargs:
            return
        keys = sorted((set(kw) ^ set(self._sent_kwargs))
                      | {k for k in set(kw) & set(self._sent_kwargs) if kw[k] != self._sent_kwargs[k]})
        raise RuntimeError(
            f"template kwargs changed mid-conversation ({', '.join(keys)}) and re-render turns that were "
            "already sent; pass the same kwargs every turn (e.g. documents=[] from the first turn) or use "
            "KVHistoryPolicy.RE_PREFILL")

    @staticmethod
    def _raise_not_append_only():
        raise RuntimeError(
            "cannot derive a delta: the chat template is not append-only for a growing message list "
            "(earlier turns re-render when a turn is added)")
