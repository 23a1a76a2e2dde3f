"""Split the adapter stream into a LoRA stream and a probe stream.

Probe slots share the control-token machinery with LoRA slots, but their
positions must not run any LoRA delta; the probe head reads the hidden state
at the probe's control token instead (reference:
src/granite_switch/probe_routing.py:17-58).
"""
from __future__ import annotations

import torch


def build_adapter_kind_lut(config) -> torch.Tensor | None:
    """``bool[num_adapters + 1]`` marking probe slots by adapter index; ``None`` if none."""
    kinds = getattr(config, "adapter_kinds", None) if config is not None else None
    if kinds is None or not any(k == "probe" for k in kinds):
        return None
    lut = torch.zeros(len(kinds) + 1, dtype=torch.bool)
    for slot, kind in enumerate(kinds):
        if kind == "probe":
            lut[slot + 1] = True
    return lut


def split_adapter_indices(kind_lut: torch.Tensor | None, adapter_indices: torch.Tensor):
    """``(lora_indices, probe_indices)``: probe positions zeroed / kept respectively."""
    if kind_lut is None:
        return adapter_indices, torch.zeros_like(adapter_indices)
    is_probe = kind_lut.to(adapter_indices.device)[adapter_indices]
    zeros = torch.zeros_like(adapter_indices)
    return torch.where(is_probe, zeros, adapter_indices), torch.where(is_probe, adapter_indices, zeros)
