"""Paged causal GQA attention (native, sm_100a) and its PyTorch oracle."""
from __future__ import annotations

import math

import torch

from .._native import err_buffer, native

NUM_SMS = 148

#: rows per CTA of the tcgen05 prefill attention the engine uses: 128 (one query
#: tile per CTA), 256 (two query tiles per CTA sharing each K/V tile) or 0 (chosen
#: per step by :func:`tc_rows_for`); A/B tests assign it
TC_ROWS = 0


def tc_rows_for(q_lens: list[int], kv_lens: list[int]) -> int:
    """Rows per CTA for a step's prefill chunks when ``TC_ROWS`` is 0.

    256 when at least half of the prefill tokens are in long, mostly fresh chunks
    (q_len >= 1024 over at most as many cached keys), else 128. Measured on B200
    (d=128, 32/8 heads): fresh causal 4k runs at 825 vs 768 TFLOP/s with 256 rows
    (16.5 vs 17.4 ms in an 8B step with two such prompts), while 8 chunks of 512
    over 3.5k cached keys run at 759 vs 775 TFLOP/s.
    """
    if TC_ROWS:
        return TC_ROWS
    total = sum(q_lens)
    long_fresh = sum(q for q, k in zip(q_lens, kv_lens) if q >= 1024 and k - q <= q)
    return 256 if total and 2 * long_fresh >= total else 128


# CTAs a split prefill grid aims at, and the fewest keys a split may hold (A/B knobs of
# split_prefill; the engine uses the defaults).
PREFILL_SPLIT_CTAS = NUM_SMS
PREFILL_MIN_KEYS_PER_SPLIT = 512


def split_prefill(q_lens: list[int], kv_lens: list[int], group: int, num_kv_heads: int,
                  min_kv: int = 1024, rows: int = 128) -> int:
    """Key-range splits for a step's prefill tiles of ``rows`` rows (128: tcgen05; 64: the
    mma.sync layout, which an fp8 cache uses), or 0 for none.

    Short chunks after long cached prefixes (the next call of a conversation:
    tens of new tokens over thousands of cached keys) give the tcgen05 kernel
    a few 128-row tiles that each stream the whole prefix, leaving most SMs
    idle: measured on B200 (8B shape, two 48-token chunks over 4.5k keys) at
    95 us per layer. When the grid would have fewer CTAs than SMs and the
    longest context is at least ``min_kv`` keys, each tile's key range is
    split over CTAs as for decode (``choose_splits``) and the partials merged.
    """
    if not q_lens or max(kv_lens) < min_kv:
        return 0
    n_ctas = sum(-(-q * group // rows) for q in q_lens) * num_kv_heads
    if n_ctas >= NUM_SMS:
        return 0
    ns = choose_splits(n_ctas, max(kv_lens), PREFILL_MIN_KEYS_PER_SPLIT, PREFILL_SPLIT_CTAS)
    return ns if ns > 1 else 0


def build_work(q_lens: list[int], group: int, rows_per_tile: int,
               kv_lens: list[int] | None = None) -> tuple[list[int], list[int]]:
    """(request, first row) per CTA tile; a request contributes ceil(q_len*G / rows) tiles.

    With ``kv_lens`` the tiles are ordered by the number of keys they attend
    (causal), heaviest first, so the last wave of CTAs is short.
    """
    seqs, rows = [], []
    for i, ql in enumerate(q_lens):
        n = ql * group
        for r0 in range(0, n, rows_per_tile):
            seqs.append(i)
            rows.append(r0)
    if kv_lens is not None and len(seqs) > 1:
        def keys(t):
            i, r0 = seqs[t], rows[t]
            last = min(r0 + rows_per_tile, q_lens[i] * group) - 1
            return min(kv_lens[i], kv_lens[i] - q_lens[i] + last // group + 1)

        order = sorted(range(len(seqs)), key=keys, reverse=True)
        seqs = [seqs[t] for t in order]
        rows = [rows[t] for t in order]
    return seqs, rows


# CTAs a split decode grid aims at (choose_splits): about 3.5 waves of the decode layout's
# three resident CTAs per SM
DECODE_SPLIT_CTAS = 1536


def choose_splits(n_ctas: int, max_kv: int, min_keys_per_split: int = 512, target: int | None = None) -> int:
    """Flash-decoding split count: split every (request, KV head) key range while the
    grid has fewer than ``target`` CTAs (default ``DECODE_SPLIT_CTAS``), aiming at about
    ``target`` CTAs, never below ``min_keys_per_split`` keys per split. Measured on B200
    (d=128, 32 q / 8 kv heads, 128 requests x 4.2-4.5k keys, 1,024 CTAs): two splits ran
    the kernel in 349 vs 365 us (L2 flushed; three: 355 us) and a CUDA-graph decode step of
    the 8B shape in 19.6 vs 20.3 ms, the unsplit grid's last partial wave of CTAs being the
    loss; the fp32 partials and the merge cost less than that.
    """
    if target is None:
        target = DECODE_SPLIT_CTAS
    if n_ctas >= target:
        return 1
    want = max(1, (target + n_ctas - 1) // max(n_ctas, 1))
    cap = max(1, max_kv // min_keys_per_split)
    return int(max(1, min(want, cap, 32)))


def paged_attention(q, k_cache, v_cache, block_table, q_start, kv_len, work_seq, work_row0,
                    rows_per_tile: int, num_q_heads: int, scale: float, out, nsplit: int = 1,
                    ws_o=None, ws_lse=None, k_scale=None, v_scale=None):
    """bf16 cache: ``k_cache``/``v_cache`` ``[blocks, Hkv, 16, D]``. fp8 cache (uint8, the
    layout of :func:`kv_write_fp8`): K ``[blocks, Hkv, 16, D]``, V ``[blocks, Hkv, D, 16]``,
    with fp32 ``k_scale``/``v_scale`` ``[blocks, Hkv, 16]``."""
    native().paged_attention(q, k_cache, v_cache, block_table, q_start, kv_len, work_seq, work_row0,
                             rows_per_tile, num_q_heads, float(scale), out, nsplit, ws_o, ws_lse,
                             err_buffer(q.device), k_scale, v_scale)
    return out


def _perm16():
    """Stored position of each element of a 16-element group in the fp8 cache."""
    return [((i >> 1) << 2) + (i & 1) if i < 8 else (((i - 8) >> 1) << 2) + 2 + (i & 1) for i in range(16)]


def kv_write_fp8(qkv, slots, k8, v8, k_scale, v_scale, num_q_heads: int, num_kv_heads: int, head_dim: int):
    """Quantise a step's (already rotated) K and V rows of ``qkv`` into the fp8 cache: one fp32
    scale per (token, KV head) row, ``max|x| / 448``, and e4m3 values. K is stored
    ``[blocks, Hkv, 16, D]`` and V transposed ``[blocks, Hkv, D, 16]``, both with each
    16-element group in the order 0 1 8 9 2 3 10 11 4 5 12 13 6 7 14 15."""
    native().kv_write_fp8(qkv, slots, k8, v8, k_scale, v_scale, num_q_heads, num_kv_heads, head_dim,
                          err_buffer(qkv.device))


def rope_kv_fp8(qkv, positions, cos_sin, slots, k8, v8, k_scale, v_scale, num_q_heads: int, num_kv_heads: int,
                head_dim: int):
    """RoPE on the step's q / k heads of ``qkv`` (in place), then the quantised write of its K / V
    rows into the fp8 cache, in one launch: the result of ``elementwise.rope_kv`` (without a
    cache) followed by :func:`kv_write_fp8`."""
    native().rope_kv_fp8(qkv, positions, cos_sin, slots, k8, v8, k_scale, v_scale, num_q_heads, num_kv_heads,
                         head_dim, err_buffer(qkv.device))


def dequantize_fp8_cache(k8, v8, k_scale, v_scale):
    """fp32 ``[blocks, Hkv, 16, D]`` K and V from the fp8 cache (test oracle, reads the stored order)."""
    perm = torch.tensor(_perm16(), device=k8.device)
    nb, hkv, page, d = k8.shape
    kf = k8.view(torch.float8_e4m3fn).float().view(nb, hkv, page, d // 16, 16)[..., perm].reshape(nb, hkv, page, d)
    vf = v8.view(torch.float8_e4m3fn).float()[..., perm].transpose(2, 3)  # [nb, hkv, 16, d]
    return kf * k_scale.unsqueeze(-1), vf * v_scale.unsqueeze(-1)


def prefill_attention_tc(q, k_cache, v_cache, block_table, q_start, kv_len, work_seq, work_row0,
                         num_q_heads: int, scale: float, out, rows_per_tile: int = 128, nsplit: int = 1,
                         ws_o=None, ws_lse=None):
    """tcgen05 prefill attention; the work tiles must be built with the same ``rows_per_tile``:
    128 (one query tile per CTA, two CTAs per SM) or 256 (two query tiles per CTA sharing each
    K/V tile, 128-key tiles, one CTA per SM). ``nsplit > 1`` (128-row tiles) splits every
    tile's key range over CTAs and merges the partials, with the fp32 workspaces of
    :func:`paged_attention`; only the work tiles' own output rows are written."""
    native().prefill_attention_tc(q, k_cache, v_cache, block_table, q_start, kv_len, work_seq, work_row0,
                                  num_q_heads, float(scale), out, err_buffer(q.device), int(rows_per_tile),
                                  int(nsplit), ws_o, ws_lse)
    return out


def paged_attention_reference(q, k_cache, v_cache, block_table, q_lens, kv_lens, num_q_heads, scale):
    """fp32 oracle. q ``[T, Hq*D]`` (flat, requests back to back); returns ``[T, Hq*D]`` fp32."""
    _, hkv, page, d = k_cache.shape
    g = num_q_heads // hkv
    outs = []
    off = 0
    for i, (ql, kl) in enumerate(zip(q_lens, kv_lens)):
        nblk = (kl + page - 1) // page
        blocks = block_table[i, :nblk].long()
        k = k_cache[blocks].permute(0, 2, 1, 3).reshape(-1, hkv, d)[:kl].float()  # [kl, hkv, d]
        v = v_cache[blocks].permute(0, 2, 1, 3).reshape(-1, hkv, d)[:kl].float()
        qi = q[off:off + ql, : num_q_heads * d].float().view(ql, num_q_heads, d)
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
        att = torch.einsum("qhd,khd->hqk", qi, k) * scale
        pos = torch.arange(kl - ql, kl, device=q.device)
        mask = torch.arange(kl, device=q.device).unsqueeze(0) <= pos.unsqueeze(1)
        att = att.masked_fill(~mask.unsqueeze(0), float("-inf"))
        p = torch.softmax(att, dim=-1)
        o = torch.einsum("hqk,khd->qhd", p, v).reshape(ql, num_q_heads * d)
        outs.append(o)
        off += ql
    return torch.cat(outs, 0)


__all__ = ["paged_attention", "paged_attention_reference", "build_work", "choose_splits", "math"]
