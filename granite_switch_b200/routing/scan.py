"""Exact per-token adapter routing: "the latest control token wins".

The reference derives each token's adapter with two attention heads over a
Kerdock-coded memory (reference: src/granite_switch/hf/switch/multi.py:336-600,
src/granite_switch/vllm/switch/multi.py:348-525). The value that machinery is
built to produce is defined in closed form:

    adapter_index[t] = expert(last control token at a position <= t of the
                              same request), or 0 if there is none,

with ``expert = slot + 1`` (or ``slot`` when ``adapter_token_ids`` carries a
leading base-reset token, whose expert is 0), clamped to ``[0, num_adapters]``.

Here it is computed exactly as a segmented scan. Within a request the state
carried across chunks is a single integer: the expert of the last control
token seen so far. That carry is a pure function of the token prefix, so it
can be stored per KV-cache block and shared under token-keyed prefix caching.
The same definition is implemented by the native routing kernel
(csrc/routing.cu); this module is its CPU statement and oracle.
"""
from __future__ import annotations

import torch


def expert_table(adapter_token_ids: list[int], num_adapters: int, vocab_hint: int = 0) -> torch.Tensor:
    """``int32[size]``: ``-1`` for ordinary tokens, the expert id for control tokens."""
    size = max(vocab_hint, (max(adapter_token_ids) + 1) if adapter_token_ids else 0)
    tbl = torch.full((max(size, 1),), -1, dtype=torch.int32)
    offset = 0 if len(adapter_token_ids) == num_adapters + 1 else 1
    for slot, tok in enumerate(adapter_token_ids):
        tbl[tok] = min(max(slot + offset, 0), num_adapters)
    return tbl


def probe_slot_mask(adapter_kinds) -> torch.Tensor | None:
    """Which expert ids belong to probe slots: ``bool[len(adapter_kinds) + 1]`` (entry 0 is
    the base), or ``None`` when no slot is a probe.

    This is the persisted ``model.switch.adapter_kind_lut`` buffer of composed
    checkpoints. The native routing kernel reads the same mask (its ``kind_lut``).
    """
    kinds = list(adapter_kinds or [])
    if "probe" not in kinds:
        return None
    return torch.tensor([False] + [kind == "probe" for kind in kinds], dtype=torch.bool)


def split_probe_stream(adapter_index: torch.Tensor, mask: torch.Tensor | None):
    """``(lora_index, probe_index)`` from the routed expert ids.

    A token routed to a probe slot runs no LoRA delta (its LoRA index is 0) and
    carries the slot in the probe stream; every other token keeps its expert in
    the LoRA stream and 0 in the probe stream. Same rule as the routing kernel
    (csrc/routing.cu); reference behaviour: src/granite_switch/probe_routing.py:36-58.
    """
    if mask is None:
        return adapter_index, torch.zeros_like(adapter_index)
    sel = mask.to(adapter_index.device)[adapter_index].to(adapter_index.dtype)
    return adapter_index * (1 - sel), adapter_index * sel


def route_sequence(token_ids: list[int] | torch.Tensor, table: torch.Tensor, carry: int = 0) -> tuple[torch.Tensor, int]:
    """Route one request chunk. Returns ``(adapter_index[int64], new_carry)``."""
    ids = torch.as_tensor(token_ids, dtype=torch.long)
    n = ids.numel()
    if n == 0:
        return torch.zeros(0, dtype=torch.long), carry
    inside = ids < table.numel()
    e = torch.where(inside, table[torch.where(inside, ids, torch.zeros_like(ids))].long(),
                    torch.full_like(ids, -1))
    pos = torch.arange(n)
    last = torch.where(e >= 0, pos, torch.full_like(pos, -1))
    last = torch.cummax(last, dim=0).values
    vals = torch.where(last >= 0, e[last.clamp(min=0)], torch.full_like(ids, carry))
    return vals, int(vals[-1])


def route_batch(input_ids: torch.Tensor, table: torch.Tensor, carries: torch.Tensor | None = None) -> torch.Tensor:
    """Route a padded ``[B, S]`` batch (each row one request chunk)."""
    b = input_ids.shape[0]
    out = torch.zeros_like(input_ids, dtype=torch.long)
    for i in range(b):
        c = int(carries[i]) if carries is not None else 0
        out[i], _ = route_sequence(input_ids[i].cpu(), table, c)
    return out.to(input_ids.device)


def route_flat(token_ids: torch.Tensor, seq_starts: list[int], carries: list[int], table: torch.Tensor) -> tuple[torch.Tensor, list[int]]:
    """Route a flattened batch of request chunks (engine layout).

    ``seq_starts`` has one entry per chunk plus the total length.
    Returns ``(adapter_index[T], new_carries)``.
    """
    ids = token_ids.cpu()
    out = torch.zeros(ids.numel(), dtype=torch.long)
    new = []
    for i in range(len(seq_starts) - 1):
        a, b = seq_starts[i], seq_starts[i + 1]
        out[a:b], c = route_sequence(ids[a:b], table, carries[i])
        new.append(c)
    return out, new
