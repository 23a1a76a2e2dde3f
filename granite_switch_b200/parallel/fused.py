"""Fused tensor-parallel collectives over NVSwitch symmetric memory.

Row-parallel projections (o_proj, down) are computed by the switched GEMM with
the ``EPI_MULTIMEM_RED`` epilogue: as each output tile's accumulator drains,
its epilogue adds the tile into a symmetric bf16 buffer ``y`` through the
NVLink multicast address (``multimem.red``), so the NVSwitch sums the ranks'
partials and every rank's copy receives the total while other tiles are still
being computed. Rank 0 folds the residual stream into its contribution. A
bounded peer barrier then orders the reductions before the consumer, and one
kernel moves the sum into the residual stream and applies the next RMSNorm
(``h <- y; x <- RMSNorm(y); y <- 0``).

This replaces the reference's ``tensor_model_parallel_all_reduce`` after the
expand (reference: src/granite_switch/vllm/core/lora.py:568-586) and the
separate residual add / norm kernels. Because the reduction result is
multicast to all ranks, the next column-parallel GEMM (qkv, gate/up) reads its
full input from local memory: the all-gather happens inside the switch.

Requires NVLS multicast (``has_multicast_support``); without it the model keeps
the NCCL all-reduce path. Buffers come from ``torch.distributed._symmetric_memory``.
"""
from __future__ import annotations

import torch

from .._native import err_buffer, native
from ..ops import gemm as G

BARRIER_BUDGET_NS = 5_000_000_000
# largest step (rows) whose reduction rides in the GEMM epilogue, per TP size (default 256)
RED_MAX_TOKENS = {2: 1 << 20, 4: 1024}


def _multicast_supported(device: torch.device) -> bool:
    """NVLink multicast (NVLS) objects can be created on this device."""
    from torch._C._autograd import DeviceType
    from torch._C._distributed_c10d import _SymmetricMemory

    idx = device.index if device.index is not None else torch.cuda.current_device()
    return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, idx))


class FusedTPComm:
    def __init__(self, group, device: torch.device, max_tokens: int, hidden: int, red_max_tokens: int | None = None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device
        # two buffers, alternated per projection: a buffer is zeroed by its consumer
        # one projection (and so one barrier) before any rank adds into it again
        self.max_tokens, self.hidden = max_tokens, hidden
        self.y = symm_mem.empty(2, max_tokens, hidden, dtype=torch.bfloat16, device=device)
        self.y.zero_()
        self.turn = 0
        self.y_handle = symm_mem.rendezvous(self.y, group)
        self.mc = int(self.y_handle.multicast_ptr) if _multicast_supported(device) else 0
        self.y_ptrs = torch.tensor([int(p) for p in self.y_handle.buffer_ptrs], dtype=torch.int64, device=device)
        self.pads = symm_mem.empty(64, dtype=torch.int32, device=device)
        self.pads.zero_()
        self.pad_handle = symm_mem.rendezvous(self.pads, group)
        self.pad_ptrs = torch.tensor(list(self.pad_handle.buffer_ptrs), dtype=torch.int64, device=device)
        # barrier epochs count on the device, so barriers replayed from a CUDA graph
        # and eager ones advance one sequence
        self.epoch_ctr = torch.zeros(1, dtype=torch.int32, device=device)
        # rows up to which the reduction rides in the GEMM epilogue (see row_parallel);
        # from the collective sweep: always at TP=2, small steps only at TP=4 / 8
        self.red_max_tokens = red_max_tokens if red_max_tokens is not None else RED_MAX_TOKENS.get(self.world, 256)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    @property
    def supported(self) -> bool:
        return self.mc != 0

    def barrier(self, budget_ns: int = BARRIER_BUDGET_NS) -> None:
        native().peer_barrier(self.pad_ptrs, self.rank, self.world, self.epoch_ctr, budget_ns,
                              err_buffer(self.device))

    def row_parallel(self, model, pl, x: torch.Tensor, h: torch.Tensor, mult: float) -> torch.Tensor:
        """Reduce ``x @ W_shard^T * mult`` (+ ``h`` once) over the group into ``y``; returns ``y[:m]``.

        Up to ``red_max_tokens`` rows the GEMM epilogue adds each finished tile
        into every rank's copy through the multicast address (``multimem.red``):
        the reduction overlaps the GEMM and there is one barrier. That makes
        every GPU's memory absorb all N partials, which stops paying at large
        steps on many GPUs (measured at TP=8: 26 vs 43 us at 8 tokens, 0.82 vs
        0.30 ms at 8192 tokens against NCCL), so larger steps store the partial
        and all-reduce it with NCCL.
        """
        m = x.shape[0]
        b = self.turn
        self.turn ^= 1
        y = self.y[b, :m]
        resid = h if self.rank == 0 else None
        mc = self.mc + b * self.max_tokens * self.hidden * 2
        if m <= self.red_max_tokens:
            model._proj(pl, x, y, epi=G.EPI_MULTIMEM_RED, residual=resid, scale=mult, mc_out=mc)
            self.barrier()
        else:
            if resid is not None:
                model._proj(pl, x, y, epi=G.EPI_RESADD, residual=resid, scale=mult)
            else:
                model._proj(pl, x, y, epi=G.EPI_STORE, scale=mult)
            torch.distributed.all_reduce(y, group=self.group)
        return y

    def finish(self, y: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor, x: torch.Tensor, eps: float) -> None:
        """``h <- y; x <- RMSNorm(y) * norm_w; y <- 0``."""
        native().rmsnorm_residual_from(y, h, norm_w, x, float(eps))


def attach_fused_comm(model, group) -> bool:
    """Attach a :class:`FusedTPComm` to a native model; False (NCCL path kept) without multicast."""
    if getattr(model, "dual", False) or getattr(model, "has_moe", False):
        return False  # Shadow-Residual and expert-bank models reduce over NCCL
    comm = FusedTPComm(group, model.device, model.max_tokens, model.hidden)
    if not comm.supported:
        return False
    model.comm = comm
    return True
