"""Control-token -> substitute-token exchange (format-level, backend neutral).

The switch reads the original ids to decide routing and then rewrites every
control id to its substitute id, so the decoder never embeds a control token
(reference: src/granite_switch/token_exchange.py:52-176). The table is a pure
function of ``vocab_size``, ``adapter_token_ids`` and
``adapter_substitute_token_ids``; it is persisted in the checkpoint as
``model.switch.control_to_substitute_lut``.
"""
from __future__ import annotations

import torch


def build_control_to_substitute_lut(config) -> torch.Tensor | None:
    """``int64[max(vocab_size, max_ctrl + 1)]``: ``-1`` except control ids -> substitute.

    The table is sized with ``max`` because the composer builds the switch
    before it resizes the embeddings to cover the appended control ids.
    Returns ``None`` when no mapping is configured.
    """
    if config is None:
        return None
    ctrl = getattr(config, "adapter_token_ids", None)
    subs = getattr(config, "adapter_substitute_token_ids", None)
    if not ctrl or not subs:
        return None
    size = max(int(getattr(config, "vocab_size", 0)), max(ctrl) + 1)
    lut = torch.full((size,), -1, dtype=torch.long)
    lut[torch.tensor(ctrl, dtype=torch.long)] = torch.tensor(subs, dtype=torch.long)
    return lut


def apply_token_exchange(lut: torch.Tensor | None, input_ids: torch.Tensor) -> torch.Tensor:
    """Branch-free rewrite ``lut[id] >= 0 ? lut[id] : id``; ids past the table pass through."""
    if lut is None:
        return input_ids
    lut = lut.to(input_ids.device)
    inside = input_ids < lut.numel()
    looked = lut[torch.where(inside, input_ids, torch.zeros_like(input_ids))]
    return torch.where(inside & (looked >= 0), looked, input_ids)


def validate_control_lut(lut: torch.Tensor | None, config) -> None:
    """Pre-save check: the persisted table must be exactly ``vocab_size`` long.

    (reference: src/granite_switch/composer/validator.py:17-64)
    """
    if lut is None:
        return
    if lut.numel() != int(config.vocab_size):
        raise ValueError(
            f"control_to_substitute_lut has {lut.numel()} entries but vocab_size is "
            f"{config.vocab_size}; rebuild the table after resizing the embeddings."
        )
    ctrl = config.adapter_token_ids or []
    subs = config.adapter_substitute_token_ids or []
    for c, s in zip(ctrl, subs):
        if int(lut[c]) != int(s):
            raise ValueError(f"lut[{c}] = {int(lut[c])}, expected substitute {s}")
