"""RMSNorm, embedding + token exchange, RoPE + paged KV write, argmax (native) and oracles."""
from __future__ import annotations

import torch

from .._native import err_buffer, native


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None,
            rows: torch.Tensor | None = None) -> torch.Tensor:
    n = rows.numel() if rows is not None else x.shape[0]
    if out is None:
        out = torch.empty((n, x.shape[1]), dtype=x.dtype, device=x.device)
    native().rmsnorm(x, w, out, rows, float(eps))
    return out


def rmsnorm_reference(x, w, eps, rows=None):
    if rows is not None:
        x = x[rows]
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * h.to(x.dtype).float()).to(x.dtype)


def embed(ids: torch.Tensor, table: torch.Tensor, lut: torch.Tensor | None, mult: float,
          out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device)
    native().embed(ids, table, lut, float(mult), out, err_buffer(ids.device))
    return out


def embed_reference(ids, table, lut, mult):
    if lut is not None:
        inside = ids < lut.numel()
        s = lut[torch.where(inside, ids, torch.zeros_like(ids))]
        ids = torch.where(inside & (s >= 0), s, ids)
    return (table[ids].float() * mult).to(table.dtype)


def rope_cos_sin_table(max_pos: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """``[max_pos, head_dim]`` fp32: cos in the first half, sin in the second (computed in fp64)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    f = torch.arange(max_pos, dtype=torch.float64).unsqueeze(1) * inv.unsqueeze(0)
    return torch.cat([f.cos(), f.sin()], dim=1).float().to(device)


def rope_kv(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, num_q: int, num_kv: int,
            head_dim: int, k_cache=None, v_cache=None, slots=None) -> None:
    native().rope_kv(qkv, positions, cos_sin, k_cache, v_cache, slots, num_q, num_kv, head_dim,
                     err_buffer(qkv.device))


def rope_reference(x, positions, cos_sin):
    """x ``[T, heads, D]``; NeoX rotate-half with the fp32 table."""
    d = x.shape[-1]
    cs = cos_sin[positions]
    c, s = cs[:, : d // 2], cs[:, d // 2:]
    x1, x2 = x[..., : d // 2].float(), x[..., d // 2:].float()
    c, s = c.unsqueeze(1), s.unsqueeze(1)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
    native().argmax(logits, out)
    return out


def residual_axpy(h: torch.Tensor, y: torch.Tensor, scale: float) -> None:
    """``h <- h + y * scale`` (bf16)."""
    native().residual_axpy(h, y, float(scale))
