"""fp32 statement of the reference's coded-memory switch (CPU oracle only).

Two single-head causal attentions (reference:
src/granite_switch/hf/switch/multi.py:391-588):

1. counting head: keys are unmasked (0) at the position-0 anchor and at every
   control token, ``-1e9`` elsewhere; value 1 at the anchor. The output at t is
   ``1/(1+n)`` with n the number of control tokens in ``(0, t]`` (plus one if
   position 0 is itself a control token only when it is also counted as the
   anchor, which it is not), so ``n = round(1/signal - 1)``.
2. memory head: at control tokens the key is ``codebook[n] * gain`` and the
   value the expert id; every query is ``codebook[n]``. Softmax picks the
   control token whose write address equals the reader's count, i.e. the
   most recent one.

The result is rounded and clamped to ``[0, num_adapters]``. This module exists
to check the exact scan in :mod:`.scan` against the algorithm it replaces.
"""
from __future__ import annotations

import torch

from .codebook import recover_count_from_signal

_NEG = -1e9


def coded_switch_route(input_ids: torch.Tensor, adapter_token_ids: list[int], num_adapters: int,
                       codebook: torch.Tensor, memory_gain: float = 28.0) -> torch.Tensor:
    """Route one sequence ``int64[S]`` (positions 0..S-1) with the coded memory."""
    ids = input_ids.long()
    s = ids.numel()
    tok = torch.tensor(adapter_token_ids, dtype=torch.long)
    matches = ids.unsqueeze(1) == tok.unsqueeze(0)
    is_ctrl = matches.any(dim=1)
    offset = 0 if len(adapter_token_ids) == num_adapters + 1 else 1
    expert = torch.where(is_ctrl, matches.long().argmax(dim=1) + offset, torch.zeros_like(ids))
    pos = torch.arange(s)
    anchor = pos == 0
    causal = pos.unsqueeze(0) <= pos.unsqueeze(1)  # [q, k]

    # counting head: q.k = key[k] (0 or -1e9), v = anchor indicator
    key = torch.where(anchor | is_ctrl, torch.zeros(s), torch.full((s,), _NEG)).float()
    logits = key.unsqueeze(0).expand(s, s).clone()
    logits[~causal] = _NEG
    w = torch.softmax(logits, dim=1)
    signal = w @ anchor.float()
    n = recover_count_from_signal(signal, codebook.shape[0])

    codes = codebook.float()[n]  # [S, N]
    mkey = codes * memory_gain * is_ctrl.float().unsqueeze(1)
    mval = expert.float() * is_ctrl.float()
    mlog = codes @ mkey.t()  # [q, k]
    mlog[~causal] = _NEG
    mw = torch.softmax(mlog, dim=1)
    raw = mw @ mval
    return torch.clamp(torch.round(raw).long(), 0, num_adapters)
