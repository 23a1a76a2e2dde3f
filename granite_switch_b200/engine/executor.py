"""Model executors: turn a scheduler step into model inputs, run it, sample.

``NativeExecutor`` runs :class:`~granite_switch_b200.models.native.NativeGraniteSwitch`
on a B200: step inputs are staged in pinned host memory, copied to persistent
device buffers (fixed addresses, so decode steps can be captured in CUDA
graphs), and the sampled ids are copied back once per step.

``ReferenceExecutor`` runs the same step with the HF-style PyTorch modules over
a paged fp32 cache. It is the CPU oracle for the engine (scheduler, paging,
prefix caching and chunked prefill are checked against plain ``generate``).
"""
from __future__ import annotations

import math

import torch

from ..routing.scan import route_flat
from .kv_cache import BLOCK_SIZE
from .scheduler import SchedulerOutput


class HostBatch:
    """Flattened host-side description of one step."""

    def __init__(self, out: SchedulerOutput):
        ids, pos, slots, starts, carry, kv_lens, rows, q_lens = [], [], [], [0], [], [], [], []
        self.chunks = out.chunks
        for c in out.chunks:
            r = c.req
            toks = r.all_ids[c.start:c.start + c.num_tokens]
            ids.extend(toks)
            for p in range(c.start, c.start + c.num_tokens):
                pos.append(p)
                slots.append(r.block_ids[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE)
            starts.append(starts[-1] + c.num_tokens)
            carry.append(r.carry)
            kv_lens.append(c.start + c.num_tokens)
            q_lens.append(c.num_tokens)
            if c.needs_sample:
                rows.append(starts[-1] - 1)
        self.ids, self.pos, self.slots, self.starts = ids, pos, slots, starts
        self.carry, self.kv_lens, self.rows, self.q_lens = carry, kv_lens, rows, q_lens
        self.block_lists = [c.req.block_ids for c in out.chunks]


class NativeExecutor:
    def __init__(self, model, max_model_len: int, tp_group=None, tp_size: int = 1, use_cuda_graphs: bool = False):
        self.model = model
        self.device = model.device
        self.tp_group, self.tp_size = tp_group, tp_size
        self.max_blocks = (max_model_len + BLOCK_SIZE - 1) // BLOCK_SIZE
        t, s = model.max_tokens, model.max_seqs
        pin = dict(pin_memory=True)
        self.h_i64 = torch.empty(3 * t, dtype=torch.long, **pin)          # ids | positions | slots
        self.h_i32 = torch.empty(3 * s + 1, dtype=torch.int32, **pin)     # starts | carry | kv_lens
        self.h_bt = torch.zeros(s, self.max_blocks, dtype=torch.int32, **pin)
        self.h_rows = torch.empty(s, dtype=torch.long, **pin)
        self.h_out = torch.empty(s, dtype=torch.long, **pin)
        dev = self.device
        self.d_i64 = torch.empty(3 * t, dtype=torch.long, device=dev)
        self.d_i32 = torch.empty(3 * s + 1, dtype=torch.int32, device=dev)
        self.d_bt = torch.zeros(s, self.max_blocks, dtype=torch.int32, device=dev)
        self.d_rows = torch.empty(s, dtype=torch.long, device=dev)
        self.d_work = torch.empty(4, 4 * t + 4 * s, dtype=torch.int32, device=dev)
        self.h_work = torch.empty(4, 4 * t + 4 * s, dtype=torch.int32, **pin)
        self.d_tokens = torch.empty(s, dtype=torch.long, device=dev)
        self.copy_event = torch.cuda.Event()
        self.h2d_event = torch.cuda.Event()
        self.h2d_pending = False
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.gather_buf = None

    def _stage(self, hb: HostBatch):
        from ..models.native import AttnPlan, StepBatch

        t, s = len(hb.ids), len(hb.starts) - 1
        m = self.model
        if t > m.max_tokens or s > m.max_seqs:
            raise ValueError(f"step of {t} tokens / {s} seqs exceeds buffers ({m.max_tokens}/{m.max_seqs})")
        # host staging (pinned): the previous step's async copies must have landed
        if self.h2d_pending:
            self.h2d_event.synchronize()
        self.h_i64[:t] = torch.tensor(hb.ids, dtype=torch.long)
        self.h_i64[t:2 * t] = torch.tensor(hb.pos, dtype=torch.long)
        self.h_i64[2 * t:3 * t] = torch.tensor(hb.slots, dtype=torch.long)
        self.h_i32[: s + 1] = torch.tensor(hb.starts, dtype=torch.int32)
        self.h_i32[s + 1:2 * s + 1] = torch.tensor(hb.carry, dtype=torch.int32)
        self.h_i32[2 * s + 1:3 * s + 1] = torch.tensor(hb.kv_lens, dtype=torch.int32)
        width = max(len(b) for b in hb.block_lists)
        bt = torch.zeros(s, width, dtype=torch.int32)
        for i, bl in enumerate(hb.block_lists):
            bt[i, : len(bl)] = torch.tensor(bl, dtype=torch.int32)
        self.h_bt[:s, :width] = bt
        nb = len(hb.rows)
        self.h_rows[:nb] = torch.tensor(hb.rows, dtype=torch.long)
        plans_host = m.attention_plans(hb.q_lens, hb.kv_lens)
        for pi, (ws, wr, rows, ns) in enumerate(plans_host):
            self.h_work[2 * pi, : len(ws)] = torch.tensor(ws, dtype=torch.int32)
            self.h_work[2 * pi + 1, : len(wr)] = torch.tensor(wr, dtype=torch.int32)
        # H2D (one copy per staging buffer)
        self.d_i64[: 3 * t].copy_(self.h_i64[: 3 * t], non_blocking=True)
        self.d_i32[: 3 * s + 1].copy_(self.h_i32[: 3 * s + 1], non_blocking=True)
        self.d_bt[:s, :width].copy_(self.h_bt[:s, :width], non_blocking=True)
        self.d_rows[:nb].copy_(self.h_rows[:nb], non_blocking=True)
        nw = max((len(p[0]) for p in plans_host), default=0)
        if plans_host:
            self.d_work[: 2 * len(plans_host), :nw].copy_(self.h_work[: 2 * len(plans_host), :nw], non_blocking=True)
        self.h2d_event.record()
        self.h2d_pending = True
        self.h2d_bytes += 8 * 3 * t + 4 * (3 * s + 1) + 4 * s * width + 8 * nb + 4 * 2 * len(plans_host) * nw
        plans = [AttnPlan(self.d_work[2 * pi, : len(ws)], self.d_work[2 * pi + 1, : len(ws)], rows, ns)
                 for pi, (ws, wr, rows, ns) in enumerate(plans_host)]
        return StepBatch(num_tokens=t, num_seqs=s, ids=self.d_i64[:t], positions=self.d_i64[t:2 * t],
                         slots=self.d_i64[2 * t:3 * t], seq_starts=self.d_i32[: s + 1],
                         carry_in=self.d_i32[s + 1:2 * s + 1], kv_lens=self.d_i32[2 * s + 1:3 * s + 1],
                         block_table=self.d_bt[:s, :width], logit_rows=self.d_rows[:nb], plans=plans)

    def _gather_logits(self, logits: torch.Tensor) -> torch.Tensor:
        if self.tp_size == 1:
            return logits[:, : self.model.vocab]
        b, per = logits.shape
        full = torch.empty(self.tp_size, b, per, dtype=logits.dtype, device=logits.device)
        torch.distributed.all_gather_into_tensor(full, logits.contiguous(), group=self.tp_group)
        return full.permute(1, 0, 2).reshape(b, self.tp_size * per)[:, : self.model.vocab]

    def compute_logits(self, out: SchedulerOutput):
        """Run the step; returns ``(HostBatch, fp32 logits [B, vocab])`` for rows that sample."""
        hb = HostBatch(out)
        batch = self._stage(hb)
        logits = self.model.forward(batch)
        if not hb.rows or logits is None:
            return hb, None
        return hb, self._gather_logits(logits)

    def execute(self, out: SchedulerOutput) -> list[int]:
        from ..ops import elementwise as E
        from .sampling import sample

        hb, logits = self.compute_logits(out)
        nb = len(hb.rows)
        if nb == 0:
            return []
        params = [c.req.sampling for c in hb.chunks if c.needs_sample]
        toks = self.d_tokens[:nb]
        if all(p.greedy for p in params):
            E.argmax(logits, out=toks)
        else:
            sample(logits, params, [c.req for c in hb.chunks if c.needs_sample], out=toks)
        self.h_out[:nb].copy_(toks, non_blocking=True)
        self.copy_event.record()
        self.copy_event.synchronize()
        self.d2h_bytes += 8 * nb
        return self.h_out[:nb].tolist()


class ReferenceExecutor:
    """Paged-cache step on the HF-style PyTorch modules (CPU oracle)."""

    def __init__(self, ref_model, num_blocks: int, dtype=torch.float32):
        self.m = ref_model
        cfg = ref_model.config
        self.cfg = cfg
        d = cfg.head_dim_eff
        self.kv = torch.zeros(cfg.num_decoder_layers, 2, num_blocks, cfg.num_key_value_heads, BLOCK_SIZE, d,
                              dtype=dtype)
        sw = ref_model.model.switch
        self.table = sw._table if sw is not None else None
        self.h2d_bytes = self.d2h_bytes = 0

    @torch.no_grad()
    def execute(self, out: SchedulerOutput) -> list[int]:
        hb, logits = self.compute_logits(out)
        if logits is None:
            return []
        params = [c.req.sampling for c in hb.chunks if c.needs_sample]
        if all(p.greedy for p in params):
            return logits.argmax(dim=-1).tolist()
        from .sampling import sample_reference

        return sample_reference(logits, params, [c.req for c in hb.chunks if c.needs_sample]).tolist()

    @torch.no_grad()
    def compute_logits(self, out: SchedulerOutput):
        from ..models.layers import apply_rope, rope_cos_sin
        from ..ops.attention import paged_attention_reference
        from ..routing.token_exchange import apply_token_exchange

        cfg = self.cfg
        hb = HostBatch(out)
        ids = torch.tensor(hb.ids, dtype=torch.long)
        if self.table is not None:
            idx, _ = route_flat(ids, hb.starts, hb.carry, self.table)
            lora_idx, _ = self.m.model.switch.split_indices(idx)
            lut = self.m.model.switch.control_to_substitute_lut
        else:
            lora_idx = torch.zeros_like(ids)
            lut = None
        mod = apply_token_exchange(lut, ids)
        pos = torch.tensor(hb.pos, dtype=torch.long)
        slots = torch.tensor(hb.slots, dtype=torch.long)
        h = self.m.model.embed_tokens(mod) * cfg.embedding_multiplier
        cos, sin = rope_cos_sin(pos.unsqueeze(0), cfg.head_dim_eff, cfg.rope_theta, h.dtype)
        width = max(len(b) for b in hb.block_lists)
        bt = torch.zeros(len(hb.block_lists), width, dtype=torch.int32)
        for i, bl in enumerate(hb.block_lists):
            bt[i, : len(bl)] = torch.tensor(bl, dtype=torch.int32)
        blk, off = slots // BLOCK_SIZE, slots % BLOCK_SIZE
        for li, layer in enumerate(self.m.model.layers):
            att = layer.self_attn
            x = layer.input_layernorm(h)
            q, k, v = att.project_qkv(x.unsqueeze(0), lora_idx.unsqueeze(0), cos, sin)
            q, k, v = q[0], k[0], v[0]
            self.kv[li, 0, blk, :, off] = k.to(self.kv.dtype)
            self.kv[li, 1, blk, :, off] = v.to(self.kv.dtype)
            o = paged_attention_reference(q.reshape(len(hb.ids), -1), self.kv[li, 0], self.kv[li, 1], bt,
                                          hb.q_lens, hb.kv_lens, cfg.num_attention_heads, att.scaling)
            h = h + att.out(o.to(h.dtype).unsqueeze(0), lora_idx.unsqueeze(0))[0] * layer.residual_multiplier
            x = layer.post_attention_layernorm(h)
            h = h + layer.mlp(x.unsqueeze(0), lora_idx.unsqueeze(0))[0] * layer.residual_multiplier
        if not hb.rows:
            return hb, None
        hf = self.m.model.norm(h[torch.tensor(hb.rows)])
        return hb, self.m.lm_head(hf).float() / cfg.logits_scaling


__all__ = ["NativeExecutor", "ReferenceExecutor", "HostBatch", "math"]
