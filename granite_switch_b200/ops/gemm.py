"""Switched-LoRA GEMM (tcgen05/TMEM/TMA, sm_100a) and its PyTorch oracle.

``switched_gemm`` computes ``x @ w.T`` on the tensor cores and, when LoRA
operands are given, adds per row ``S_a @ B_a.T`` inside the same accumulator
(``S`` = masked shrink output, ``B`` = packed expand weights), then applies a
fused epilogue. ``lora_shrink`` produces ``S`` with the same kernel and an
epilogue that zeroes the columns of adapters other than the row's own.
"""
from __future__ import annotations

import torch

from .._native import err_buffer, native

EPI_STORE = 0
EPI_RESADD = 1
EPI_SWIGLU = 2
EPI_MASK_ADAPTER = 3
EPI_F32 = 4
EPI_MULTIMEM_RED = 5


def pick_bn(m: int, n: int, candidates=(256, 128, 64), two_tile_bn: int | None = 128) -> int:
    """Widest N tile dividing ``n`` that still gives every SM work.

    Small-M (decode) GEMMs are bandwidth bound: narrower tiles put more CTAs
    on the weight stream. Large-M GEMMs prefer the widest tile. Two row tiles
    (129-256 rows, a decode batch plus a few short prefill chunks) take 128-wide
    tiles: every CTA re-reads its rows of ``x`` per N tile, and measured on B200
    at M = 222 / 140 (8B shapes, event-timed, weights rotated past L2) 64-wide
    tiles ran qkv (6144x4096) in 44 vs 26 us and down (4096x12800) in 63 vs 44 us
    (the latter split-K), with o and gate/up within 5%. ``two_tile_bn=None``
    keeps the narrowest-filling rule (the LoRA shrink, whose N is a few hundred).
    """
    m_tiles = (m + 127) // 128
    ok = [bn for bn in candidates if n % bn == 0]
    if not ok:
        raise ValueError(f"N={n} is not a multiple of 64")
    if m_tiles == 2 and two_tile_bn in ok and (n // two_tile_bn) * m_tiles >= 64:
        return two_tile_bn  # as measured: at least 64 output tiles (split-K fills the rest)
    for bn in ok:
        if (n // bn) * m_tiles >= 148:
            return bn
    return ok[-1]


def switched_gemm(
    x: torch.Tensor,
    w: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    epi: int = EPI_STORE,
    residual: torch.Tensor | None = None,
    scale: float = 1.0,
    s: torch.Tensor | None = None,
    lb: torch.Tensor | None = None,
    tile_mask: torch.Tensor | None = None,
    rank: int = 0,
    num_adapters: int = 0,
    slice_bounds: list[int] | None = None,
    row_adapter: torch.Tensor | None = None,
    mask_rank: int = 0,
    mask_num_adapters: int = 0,
    bn: int | None = None,
    mc_out: int = 0,
    tile_expert: torch.Tensor | None = None,
) -> torch.Tensor:
    """``tile_expert`` selects grouped mode: ``w`` is a stack ``[E, N, K]`` and
    128-row tile ``t`` of ``x`` multiplies expert ``tile_expert[t]`` (-1: skipped)."""
    m, _ = x.shape
    n = w.shape[-2]
    if out is None:
        if epi == EPI_SWIGLU:
            out = torch.empty((m, n // 2), dtype=torch.bfloat16, device=x.device)
        elif epi == EPI_F32:
            out = torch.empty((m, n), dtype=torch.float32, device=x.device)
        else:
            out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    if bn is None:
        bn = pick_bn(m, n)
        if slice_bounds is not None and s is not None:
            while any(b % bn for b in slice_bounds[:-1]) and bn > 64:
                bn //= 2
    native().switched_gemm(
        x, w, out, epi, bn, residual, float(scale), s, lb, tile_mask, rank, num_adapters,
        list(slice_bounds) if slice_bounds is not None else [0, n], row_adapter, mask_rank,
        mask_num_adapters, err_buffer(x.device), int(mc_out), tile_expert,
    )
    return out


SMALL_SHRINK_MAX_M = 96  # up to this many tokens the shrink runs on CUDA cores (lora_small.cu)


def lora_shrink(x: torch.Tensor, a_all: torch.Tensor, row_adapter: torch.Tensor, rank: int,
                num_adapters: int, out: torch.Tensor | None = None,
                tile_mask: torch.Tensor | None = None) -> torch.Tensor:
    """``S = mask(x @ a_all.T)``: row ``m`` keeps only its adapter's columns.

    With ``tile_mask`` (adapters present per 128-row tile) only the column
    blocks of present adapters are computed; the expand reads nothing else.
    Up to ``SMALL_SHRINK_MAX_M`` tokens each row's own columns are computed on
    CUDA cores instead (the tensor-core kernel's fixed cost dominates there).
    """
    n = a_all.shape[0]
    if n % 64:
        raise ValueError(f"a_all must have a multiple of 64 rows (pad with zeros), got {n}")
    if x.shape[0] <= SMALL_SHRINK_MAX_M:
        if out is None:
            out = torch.empty(x.shape[0], n, dtype=torch.bfloat16, device=x.device)
        native().lora_shrink_small(x, a_all, row_adapter, out, rank, num_adapters)
        return out
    bn = pick_bn(x.shape[0], n, (128, 64), two_tile_bn=None)
    if bn > rank * num_adapters:
        bn = 64
    return switched_gemm(x, a_all, out, epi=EPI_MASK_ADAPTER, row_adapter=row_adapter,
                         mask_rank=rank, mask_num_adapters=num_adapters, tile_mask=tile_mask, bn=bn)


# ---------------------------------------------------------------- oracle
def switched_gemm_reference(x, w, *, epi=EPI_STORE, residual=None, scale=1.0, s=None, lb=None,
                            rank=0, num_adapters=0, slice_bounds=None, row_adapter=None,
                            mask_rank=0, mask_num_adapters=0, swiglu_tile=None):
    """fp32 PyTorch statement of what the kernel computes (test oracle)."""
    acc = x.float() @ w.float().t()
    n = w.shape[0]
    if s is not None and lb is not None and num_adapters > 0:
        slice_cols = num_adapters * rank
        bounds = slice_bounds or [0, n]
        delta = torch.zeros_like(acc)
        if epi == EPI_SWIGLU:
            half = swiglu_tile // 2
            for t in range(n // swiglu_tile):
                for u in range(2):
                    rows = slice(t * swiglu_tile + u * half, t * swiglu_tile + (u + 1) * half)
                    sb = u * slice_cols
                    delta[:, rows] = s[:, sb:sb + slice_cols].float() @ lb[rows].float().t()
        else:
            for i in range(len(bounds) - 1):
                cols = slice(bounds[i], bounds[i + 1])
                sb = i * slice_cols
                delta[:, cols] = s[:, sb:sb + slice_cols].float() @ lb[cols].float().t()
        acc = acc + delta
    if epi == EPI_STORE:
        return (acc * scale).to(torch.bfloat16)
    if epi == EPI_F32:
        return acc * scale
    if epi == EPI_RESADD:
        return (residual.float() + acc.to(torch.bfloat16).float() * scale).to(torch.bfloat16)
    if epi == EPI_MASK_ADAPTER:
        cols = torch.arange(n, device=x.device)
        a = (cols // mask_rank) % mask_num_adapters + 1
        keep = a.unsqueeze(0) == row_adapter.long().unsqueeze(1)
        return (acc * scale * keep).to(torch.bfloat16)
    if epi == EPI_SWIGLU:
        half = swiglu_tile // 2
        outs = []
        for t in range(n // swiglu_tile):
            g = acc[:, t * swiglu_tile: t * swiglu_tile + half].to(torch.bfloat16).float()
            u = acc[:, t * swiglu_tile + half: (t + 1) * swiglu_tile].to(torch.bfloat16).float()
            outs.append(torch.nn.functional.silu(g) * u)
        return torch.cat(outs, dim=1).to(torch.bfloat16)
    raise ValueError(epi)
