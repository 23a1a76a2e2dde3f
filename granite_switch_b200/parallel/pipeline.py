"""Pipeline parallelism: process groups and the stage-to-stage hand-off.

World = ``tp * pp`` processes, one per GPU; global rank ``r`` is pipeline stage
``r // tp`` and tensor-parallel rank ``r % tp`` inside it. Each stage holds a
contiguous range of decoder layers (and the KV cache of those layers only).
Every rank runs the same scheduler (SPMD). Per step the first stage embeds,
each stage runs its layers and sends the hidden state to the same TP rank of
the next stage with NCCL point-to-point; every stage recomputes the routing
metadata from the step's token ids instead of receiving it; the last stage
computes logits, samples, and broadcasts the sampled ids to every rank so
all schedulers stay in lockstep. This mirrors the reference's vLLM pipeline
contract (reference: src/granite_switch/vllm/granite_switch_model.py:279-318,
:413-418, :492-505): hidden state crosses stages, routing metadata is
recomputed per rank.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class Pipeline:
    rank: int              # stage index
    size: int              # number of stages
    prev: int | None       # global rank this stage receives from
    next: int | None       # global rank this stage sends to
    last_src: int          # global rank that broadcasts the sampled ids (last stage, TP rank 0)

    def send(self, *tensors) -> None:
        for t in tensors:
            if t is not None:
                dist.send(t.contiguous(), self.next)

    def recv(self, *tensors) -> None:
        for t in tensors:
            if t is not None:
                dist.recv(t, self.prev)

    def broadcast_tokens(self, tokens: torch.Tensor) -> None:
        dist.broadcast(tokens, src=self.last_src)


def init_parallel_groups(tp: int, pp: int):
    """Create the TP groups (one per stage) on an initialised world of ``tp * pp`` ranks.

    Returns ``(tp_rank, tp_group or None, Pipeline or None)``. Every rank calls
    ``new_group`` for every stage, as torch.distributed requires.
    """
    world = dist.get_world_size() if dist.is_initialized() else 1
    if world != tp * pp:
        raise ValueError(f"world size {world} != tensor_parallel_size {tp} x pipeline_parallel_size {pp}")
    rank = dist.get_rank() if dist.is_initialized() else 0
    stage, tp_rank = divmod(rank, tp)
    tp_group = None
    if tp > 1:
        for s in range(pp):
            g = dist.new_group(list(range(s * tp, (s + 1) * tp)))
            if s == stage:
                tp_group = g
    pipeline = None
    if pp > 1:
        pipeline = Pipeline(rank=stage, size=pp, prev=rank - tp if stage > 0 else None,
                            next=rank + tp if stage < pp - 1 else None, last_src=(pp - 1) * tp)
    return tp_rank, tp_group, pipeline


__all__ = ["Pipeline", "init_parallel_groups"]
