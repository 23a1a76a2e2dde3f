"""The native kernels as ``torch.library`` custom ops (``torch.ops.granite_switch_b200.*``).

Registered ops are opaque to ``torch.compile`` (it traces them through their
fake implementations and calls the kernel at run time) and capture into CUDA
graphs like any other op, so a user model can call the switched-LoRA linear
inside compiled or graph-captured code (reference: the ``granite_switch::``
custom ops, src/granite_switch/vllm/core/lora_ops.py:27-226).

* ``switched_lora_linear(x, w, a_all, lb, row_adapter, tile_mask, rank,
  num_adapters, slice_bounds, epi, scale, residual, swiglu_tile)`` - the whole
  switched-LoRA projection: masked shrink, then the base GEMM with every
  present adapter's expand in the same accumulator and the fused epilogue;
* ``lora_shrink(x, a_all, row_adapter, rank, num_adapters, tile_mask)``;
* ``paged_attention(q, k_cache, v_cache, block_table, q_start, kv_len,
  work_seq, work_row0, rows_per_tile, num_q_heads, scale, out)`` - mutates ``out``.
"""
from __future__ import annotations

import torch

from . import attention as A
from . import gemm as G

NS = "granite_switch_b200"


def _out_shape(x: torch.Tensor, w: torch.Tensor, epi: int) -> tuple[tuple[int, int], torch.dtype]:
    n = w.shape[0]
    if epi == G.EPI_SWIGLU:
        return (x.shape[0], n // 2), torch.bfloat16
    if epi == G.EPI_F32:
        return (x.shape[0], n), torch.float32
    return (x.shape[0], n), torch.bfloat16


@torch.library.custom_op(f"{NS}::lora_shrink", mutates_args=())
def lora_shrink(x: torch.Tensor, a_all: torch.Tensor, row_adapter: torch.Tensor, rank: int, num_adapters: int,
                tile_mask: torch.Tensor | None = None) -> torch.Tensor:
    return G.lora_shrink(x, a_all, row_adapter, rank, num_adapters, tile_mask=tile_mask)


@lora_shrink.register_fake
def _(x, a_all, row_adapter, rank, num_adapters, tile_mask=None):
    return x.new_empty((x.shape[0], a_all.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{NS}::switched_lora_linear", mutates_args=())
def switched_lora_linear(x: torch.Tensor, w: torch.Tensor, a_all: torch.Tensor | None, lb: torch.Tensor | None,
                         row_adapter: torch.Tensor | None, tile_mask: torch.Tensor | None, rank: int,
                         num_adapters: int, slice_bounds: list[int], epi: int = G.EPI_STORE, scale: float = 1.0,
                         residual: torch.Tensor | None = None, swiglu_tile: int = 0) -> torch.Tensor:
    if epi not in (G.EPI_STORE, G.EPI_RESADD, G.EPI_SWIGLU, G.EPI_F32):
        raise ValueError(f"switched_lora_linear: unsupported epilogue {epi}")
    bn = swiglu_tile if epi == G.EPI_SWIGLU else None
    if a_all is None or lb is None or num_adapters == 0:
        return G.switched_gemm(x, w, epi=epi, residual=residual, scale=scale, bn=bn)
    s = G.lora_shrink(x, a_all, row_adapter, rank, num_adapters, tile_mask=tile_mask)
    return G.switched_gemm(x, w, epi=epi, residual=residual, scale=scale, s=s, lb=lb, tile_mask=tile_mask,
                           rank=rank, num_adapters=num_adapters, slice_bounds=list(slice_bounds), bn=bn)


@switched_lora_linear.register_fake
def _(x, w, a_all, lb, row_adapter, tile_mask, rank, num_adapters, slice_bounds, epi=G.EPI_STORE, scale=1.0,
      residual=None, swiglu_tile=0):
    shape, dtype = _out_shape(x, w, epi)
    return x.new_empty(shape, dtype=dtype)


@torch.library.custom_op(f"{NS}::paged_attention", mutates_args=("out",))
def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                    q_start: torch.Tensor, kv_len: torch.Tensor, work_seq: torch.Tensor, work_row0: torch.Tensor,
                    rows_per_tile: int, num_q_heads: int, scale: float, out: torch.Tensor) -> None:
    A.paged_attention(q, k_cache, v_cache, block_table, q_start, kv_len, work_seq, work_row0, rows_per_tile,
                      num_q_heads, scale, out)


@paged_attention.register_fake
def _(q, k_cache, v_cache, block_table, q_start, kv_len, work_seq, work_row0, rows_per_tile, num_q_heads, scale,
      out):
    return None


def ops():
    """The registered op packet: ``torch.ops.granite_switch_b200``."""
    return getattr(torch.ops, NS)


__all__ = ["lora_shrink", "switched_lora_linear", "paged_attention", "ops", "NS"]
