"""Synthetic multi-adapter serving workload (chained aLoRA calls over a shared context).

Each conversation arrives by a Poisson process and holds one random context of
``context_len`` tokens, followed by ``calls`` sequential adapter calls. Call
``k`` appends an invocation of U[inv_min, inv_max] tokens whose first token is
the chosen adapter's control token (aLoRA: the control token replaces the
first invocation token) and generates U[gen_min, gen_max] tokens; call ``k+1``
starts when call ``k`` finishes, with its prompt extended by call ``k``'s
output. Served as aLoRA, every call shares the KV of the whole earlier
conversation; served as standard LoRA (``mode="lora"``), each call's prompt
starts with its control token, so its KV cannot be shared across adapters.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field


@dataclass
class CallSpec:
    adapter: int           # 0-based adapter slot
    invocation: list[int]  # tokens after the control token
    gen_len: int


@dataclass
class ConversationSpec:
    cid: int
    arrival: float
    context: list[int]
    calls: list[CallSpec]
    next_call: int = 0
    history: list[int] = field(default_factory=list)  # context + earlier invocations + outputs


@dataclass
class WorkloadConfig:
    num_conversations: int = 256
    rate: float = 8.0            # conversations per second (Poisson); inf = all at t=0
    context_len: int = 4096
    calls: int = 8
    inv_min: int = 16
    inv_max: int = 64
    gen_min: int = 32
    gen_max: int = 128
    vocab: int = 49152
    num_adapters: int = 12
    seed: int = 0
    mode: str = "alora"          # "alora" | "lora"


def make_workload(cfg: WorkloadConfig) -> list[ConversationSpec]:
    rng = random.Random(cfg.seed)
    t = 0.0
    convs = []
    for c in range(cfg.num_conversations):
        if cfg.rate != float("inf"):
            t += rng.expovariate(cfg.rate)
        ctx = [rng.randrange(1, cfg.vocab) for _ in range(cfg.context_len)]
        calls = []
        for _ in range(cfg.calls):
            inv_len = rng.randint(cfg.inv_min, cfg.inv_max)
            calls.append(CallSpec(rng.randrange(cfg.num_adapters),
                                  [rng.randrange(1, cfg.vocab) for _ in range(inv_len - 1)],
                                  rng.randint(cfg.gen_min, cfg.gen_max)))
        convs.append(ConversationSpec(c, t, ctx, calls, history=list(ctx)))
    return convs


def call_prompt(conv: ConversationSpec, control_token_ids: list[int], mode: str = "alora") -> list[int]:
    """Prompt of the conversation's next call (does not advance it)."""
    call = conv.calls[conv.next_call]
    ctrl = control_token_ids[call.adapter]
    if mode == "alora":
        return conv.history + [ctrl] + call.invocation
    return [ctrl] + conv.history + call.invocation


def advance(conv: ConversationSpec, prompt: list[int], output: list[int], mode: str = "alora") -> bool:
    """Record a finished call; returns True while calls remain."""
    if mode == "alora":
        conv.history = prompt + output
    else:
        conv.history = prompt[1:] + output
    conv.next_call += 1
    return conv.next_call < len(conv.calls)
