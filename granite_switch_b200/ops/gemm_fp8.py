"""Block-scaled fp8 (e4m3) GEMM with the bf16 switched-LoRA expand fused, its
quantisers and its fp32 oracle.

Scales are powers of two (UE8M0): one per (token row, 128-element K block) of the
activations and one per (128-row, 128-K) block of the weights. They are stored as
512-byte scale-factor atoms, ``[row tile][K tile][512]``; inside an atom byte
``16 (r % 32) + 4 (r // 32) + j`` holds row ``r``'s scale for K sub-block ``j``
(32 elements), the same value for the four sub-blocks. A scale ``2^e`` is the
smallest power of two with ``max|x| / 2^e <= 448`` and the stored value is
``e4m3(x / 2^e)`` (round to nearest, saturating), so dequantisation is exact
multiplication by ``2^e``.
"""
from __future__ import annotations

import torch

from .._native import err_buffer, native

E4M3_MAX = 448.0
EPI_STORE = 0
EPI_RESADD = 1


def _atom_index(device) -> torch.Tensor:
    """Byte offset of row r's sub-block-0 scale inside an atom, r = 0..127."""
    r = torch.arange(128, device=device)
    return 16 * (r % 32) + 4 * (r // 32)


def _exponent(amax: torch.Tensor) -> torch.Tensor:
    """Smallest integer e with amax / 2^e <= 448, clamped to [-127, 126]."""
    r = amax.float() / E4M3_MAX
    m, ex = torch.frexp(r)
    e = torch.where(m == 0.5, ex - 1, ex)
    e = torch.where(r < 2.0 ** -126, torch.full_like(e, -127), e)
    return e.clamp(-127, 126)


def _to_e4m3_bytes(v: torch.Tensor) -> torch.Tensor:
    return v.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def _atoms_from_exponents(e: torch.Tensor, rows_pad: int) -> torch.Tensor:
    """``e [rows, kblocks]`` int -> atoms ``[rows_pad / 128, kblocks, 512]`` uint8."""
    rows, kb = e.shape
    byte = torch.zeros(rows_pad, kb, dtype=torch.uint8, device=e.device)
    byte[:rows] = (e + 127).to(torch.uint8)
    tiles = rows_pad // 128
    atoms = torch.zeros(tiles, kb, 512, dtype=torch.uint8, device=e.device)
    idx = _atom_index(e.device)
    per = byte.view(tiles, 128, kb).permute(0, 2, 1)  # [tiles, kb, 128]
    for j in range(4):
        atoms[:, :, idx + j] = per
    return atoms


def _exponents_from_atoms(atoms: torch.Tensor, rows: int) -> torch.Tensor:
    """Inverse of :func:`_atoms_from_exponents` (sub-block 0): ``[rows, kblocks]`` int."""
    idx = _atom_index(atoms.device)
    per = atoms[:, :, idx]  # [tiles, kb, 128]
    return per.permute(0, 2, 1).reshape(-1, atoms.shape[1])[:rows].long() - 127


def quantize_weight_fp8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``w [N, K]`` -> (``w8 [N, K]`` e4m3 bytes, ``sfb [2 ceil(N / 256), K / 128, 512]``
    atoms) with one scale per 128 x 128 block (load time; plain PyTorch)."""
    n, k = w.shape
    assert k % 128 == 0 and n % 128 == 0, "weight dims must be multiples of 128"
    wb = w.float().view(n // 128, 128, k // 128, 128)
    e = _exponent(wb.abs().amax(dim=(1, 3)))  # [n/128, k/128]
    inv = torch.ldexp(torch.ones_like(e, dtype=torch.float32), -e)
    w8 = _to_e4m3_bytes(wb * inv[:, None, :, None]).view(n, k)
    rows_pad = (n + 255) // 256 * 256
    e_rows = e.repeat_interleave(128, dim=0)  # [n, k/128]
    return w8.contiguous(), _atoms_from_exponents(e_rows, rows_pad)


def quantize_rows_fp8(x: torch.Tensor, x8: torch.Tensor | None = None, sfa: torch.Tensor | None = None):
    """``x [M, K]`` bf16 -> (``x8 [M, K]`` e4m3 bytes, ``sfa [ceil(M / 128), K / 128, 512]``
    atoms), one scale per (row, 128-K block), on the GPU."""
    m, k = x.shape
    if x8 is None:
        x8 = torch.empty(m, k, dtype=torch.uint8, device=x.device)
    if sfa is None:
        sfa = torch.empty((m + 127) // 128, k // 128, 512, dtype=torch.uint8, device=x.device)
    native().quantize_fp8_rows(x, x8, sfa, err_buffer(x.device))
    return x8, sfa


def quantize_rows_reference(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """PyTorch statement of :func:`quantize_rows_fp8` (same bytes)."""
    m, k = x.shape
    xb = x.float().view(m, k // 128, 128)
    e = _exponent(xb.abs().amax(dim=2))  # [m, k/128]
    inv = torch.ldexp(torch.ones_like(e, dtype=torch.float32), -e)
    x8 = _to_e4m3_bytes(xb * inv[:, :, None]).view(m, k)
    return x8, _atoms_from_exponents(e, (m + 127) // 128 * 128)


def dequantize_fp8(q8: torch.Tensor, atoms: torch.Tensor) -> torch.Tensor:
    """fp32 values of e4m3 bytes ``q8 [rows, K]`` with their scale atoms."""
    rows, k = q8.shape
    e = _exponents_from_atoms(atoms, rows)  # [rows, k/128]
    scale = torch.ldexp(torch.ones_like(e, dtype=torch.float32), e)
    v = q8.view(torch.float8_e4m3fn).float().view(rows, k // 128, 128)
    return (v * scale[:, :, None]).view(rows, k)


def fp8_gemm(x8, sfa, w8, sfb, out=None, *, epi: int = EPI_STORE, scale: float = 1.0, residual=None,
             s=None, lb=None, tile_mask=None, rank: int = 0, num_adapters: int = 0, slice_bounds=None):
    """``out [M, N]`` bf16 = epi(scale * (dequant(x8) @ dequant(w8).T + S @ LB.T)); the LoRA
    operands (bf16, ``rank`` a multiple of 32) follow :func:`ops.gemm.switched_gemm`."""
    m, n = x8.shape[0], w8.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x8.device)
    native().fp8_gemm(x8, sfa, w8, sfb, out, int(epi), float(scale), residual, s, lb, tile_mask, int(rank),
                      int(num_adapters), list(slice_bounds) if slice_bounds is not None else [0, n],
                      err_buffer(x8.device))
    return out


def fp8_gemm_reference(x8, sfa, w8, sfb, *, epi: int = EPI_STORE, scale: float = 1.0, residual=None, s=None,
                       lb=None, rank: int = 0, num_adapters: int = 0, slice_bounds=None):
    """fp32 oracle of :func:`fp8_gemm`."""
    acc = dequantize_fp8(x8, sfa) @ dequantize_fp8(w8, sfb).t()
    n = w8.shape[0]
    if s is not None and lb is not None and num_adapters > 0:
        bounds = slice_bounds or [0, n]
        cols = num_adapters * rank
        for i in range(len(bounds) - 1):
            rows = slice(bounds[i], bounds[i + 1])
            acc[:, rows] += s[:, i * cols:(i + 1) * cols].float() @ lb[rows, :cols].float().t()
    if epi == EPI_RESADD:
        return residual.float() + acc.to(torch.bfloat16).float() * scale
    return acc * scale


__all__ = ["quantize_weight_fp8", "quantize_rows_fp8", "quantize_rows_reference", "dequantize_fp8", "fp8_gemm",
           "fp8_gemm_reference", "EPI_STORE", "EPI_RESADD"]
