"""Device routing + LoRA metadata launch (native) wrapper."""
from __future__ import annotations

import torch

from .._native import native


def route_device(ids, seq_starts, carry_in, expert_tbl, lut, kind_lut, num_adapters, remap,
                 adapter_idx, lora_idx, modified_ids, carry_out=None, row_adapter=None, tile_mask=None):
    native().routing(ids, seq_starts, carry_in, expert_tbl, lut, kind_lut, int(num_adapters), remap,
                     adapter_idx, lora_idx, modified_ids, carry_out, row_adapter, tile_mask)


def tile_masks_reference(row_adapter: torch.Tensor, tile: int = 128) -> torch.Tensor:
    t = row_adapter.numel()
    n = (t + tile - 1) // tile
    out = torch.zeros(n, dtype=torch.int64)
    ra = row_adapter.cpu().tolist()
    for i, a in enumerate(ra):
        if a > 0:
            out[i // tile] |= 1 << (a - 1)
    return out
