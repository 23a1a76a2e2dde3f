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
import types
import time

import numpy as np
import torch

from ..routing.scan import route_flat
from ..utils.tracing import nvtx_range
from .kv_cache import BLOCK_SIZE
from .scheduler import SchedulerOutput


def _req_tokens(r, upto: int) -> np.ndarray:
    """int64 mirror of ``r.all_ids`` with at least ``upto`` valid entries (extended in place)."""
    a, n = r._np_tok, r._np_tok_n
    if a is None or a.shape[0] < upto:
        cap = max(upto, len(r.prompt_ids) + r.sampling.max_tokens)
        b = np.empty(cap, np.int64)
        if a is not None and n:
            b[:n] = a[:n]
        a = r._np_tok = b
    if n < upto:
        a[n:upto] = r.all_ids[n:upto]
        r._np_tok_n = upto
    return a


def _req_blocks(r) -> tuple[np.ndarray, int]:
    """int32 mirror of ``r.block_ids`` (appended incrementally; rebuilt when the list is replaced)."""
    src = r.block_ids
    a = r._np_bt
    n = r._np_bt_n if r._np_bt_src is src else 0
    r._np_bt_src = src
    ln = len(src)
    if a is None or a.shape[0] < ln:
        b = np.empty(max(ln, 64, 2 * (a.shape[0] if a is not None else 0)), np.int32)
        if a is not None and n:
            b[:n] = a[:n]
        a = r._np_bt = b
    if n < ln:
        a[n:ln] = src[n:ln]
    r._np_bt_n = ln
    return a, ln


class HostBatch:
    """Flattened host-side description of one step (numpy arrays).

    ``ids``/``pos``/``slots`` are per token; ``starts`` (chunk offsets plus the
    total), ``carry``, ``q_lens``, ``kv_lens`` per chunk; ``bt`` is the step's
    block table ``[chunks, width]``; ``rows`` the flat rows that sample. Token
    ids and block ids come from per-request numpy mirrors that grow with the
    request, so packing costs a few vector operations per chunk instead of a
    Python loop per token.
    """

    def __init__(self, out: SchedulerOutput):
        chunks = out.chunks
        self.chunks = chunks
        s = len(chunks)
        start = np.fromiter((c.start for c in chunks), np.int64, s)
        count = np.fromiter((c.num_tokens for c in chunks), np.int64, s)
        cu = np.zeros(s + 1, np.int64)
        np.cumsum(count, out=cu[1:])
        t = int(cu[-1])
        ids = np.empty(t, np.int64)
        blocks = []
        width = 1
        fb_dst, fb_src = [], []
        for i, c in enumerate(chunks):
            r = c.req
            end = c.start + c.num_tokens
            ids[cu[i]:cu[i + 1]] = _req_tokens(r, end)[c.start:end]
            if r.pending >= 0:  # its last sampled token is still on the device
                pos = len(r.prompt_ids) + r.pending
                if c.start <= pos < end:
                    fb_dst.append(int(cu[i]) + pos - c.start)
                    fb_src.append(r.pending_row)
            bl = _req_blocks(r)
            blocks.append(bl)
            width = max(width, bl[1])
        # token rows whose id is the previous step's sample: (row in this step, row of that step's samples)
        self.fb_dst = np.asarray(fb_dst, np.int64)
        self.fb_src = np.asarray(fb_src, np.int64)
        bt = np.zeros((s, width), np.int32)
        for i, (bl, ln) in enumerate(blocks):
            bt[i, :ln] = bl[:ln]
        seq_of = np.repeat(np.arange(s), count)
        pos = np.arange(t, dtype=np.int64) - cu[:-1][seq_of] + start[seq_of]
        slots = bt[seq_of, pos // BLOCK_SIZE].astype(np.int64) * BLOCK_SIZE + pos % BLOCK_SIZE
        sample = np.fromiter((c.needs_sample for c in chunks), bool, s)
        self.ids, self.pos, self.slots, self.bt = ids, pos, slots, bt
        self.starts = cu
        self.carry = np.fromiter((c.req.carry for c in chunks), np.int64, s)
        self.q_lens = count.tolist()
        self.kv_lens = (start + count).tolist()
        self.rows = (cu[1:] - 1)[sample]


GRAPH_BUCKETS = (8, 16, 32, 64, 128, 256, 512)


class StepHandle:
    """A launched step: its sampled ids land in buffer ``buf`` (``nb`` rows) when ``event`` completes."""

    def __init__(self, out: SchedulerOutput, nb: int, buf: int, event, tokens=None):
        self.out, self.nb, self.buf, self.event, self.tokens = out, nb, buf, event, tokens


class _DecodeGraph:
    """One captured decode step for a padded batch of ``size`` single-token rows."""

    def __init__(self, size: int, graph, logits, launches: int, work):
        self.size, self.graph, self.logits, self.launches, self.work = size, graph, logits, launches, work


class NativeExecutor:
    """Stages a scheduler step into persistent device buffers and runs the native model.

    With ``use_cuda_graphs``, decode-only steps (every chunk one token) replay a
    CUDA graph captured per padded batch size (8, 16, ... up to ``max_seqs``): the
    inputs are staged into the same device buffers, padding rows point at a scratch
    KV page and are not sampled, and the whole forward (routing, every layer, LM
    head) is one graph launch. Under tensor parallelism a bucket is captured only
    when every row-parallel reduction rides in the fused GEMM epilogue (the peer
    barrier counts its epochs on the device); the logits all-gather runs after the
    replay. Other steps, and pipeline-parallel ones, run eagerly.
    """

    def __init__(self, model, max_model_len: int, tp_group=None, tp_size: int = 1, use_cuda_graphs: bool = False,
                 pp_microbatches: bool = True):
        self.model = model
        self.device = model.device
        self.tp_group, self.tp_size = tp_group, tp_size
        self.max_blocks = (max_model_len + BLOCK_SIZE - 1) // BLOCK_SIZE
        t, s = model.max_tokens, model.max_seqs
        pin = dict(pin_memory=True)
        # pinned staging, two sets: a pipelined step stages its second micro-batch while the
        # first one's copies may still wait behind the previous step on the stream
        self._staging = [self._make_staging(t, s) for _ in range(2 if model.pipeline is not None else 1)]
        # sampled ids and the device error word (bits, bad-index site, index) of the last two
        # launched steps: a step's inputs may take the previous step's ids on the device
        self.h_out = torch.empty(2, s, dtype=torch.long, **pin)
        self.h_err = torch.zeros(2, 3, dtype=torch.int32, **pin)
        self.d_err = torch.zeros(3, dtype=torch.int32, device=model.device)

        dev = self.device
        self.d_i64 = torch.empty(3 * t, dtype=torch.long, device=dev)
        self.d_i32 = torch.empty(3 * s + 1, dtype=torch.int32, device=dev)
        self.d_bt = torch.zeros(s, self.max_blocks, dtype=torch.int32, device=dev)
        self.d_rows = torch.empty(s, dtype=torch.long, device=dev)
        self.d_work = torch.empty(4, 4 * t + 4 * s, dtype=torch.int32, device=dev)

        self.d_tokens = torch.empty(2, s, dtype=torch.long, device=dev)
        self.d_fb = torch.empty(2, s, dtype=torch.long, device=dev)
        self.buf = 0           # buffer of the next launched step
        self.prev_buf = None   # buffer of the last launched step (source of fed-back ids)
        self._use_staging(0)
        self.copy_events = (torch.cuda.Event(), torch.cuda.Event())

        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.gather_buf = None
        # under tensor parallelism only steps whose reductions all ride in the fused GEMM
        # epilogue are captured (no NCCL call inside a graph); see _graph_bucket
        self.use_cuda_graphs = bool(use_cuda_graphs) and model.pipeline is None
        # pipeline parallelism: a step of two or more sequences runs as two micro-batches
        self.pp_microbatches = bool(pp_microbatches) and model.pipeline is not None
        self.routing_trace = None  # utils.tracing.RoutingTrace: per-step routing records
        self.nvtx = False          # NVTX range per step (regions: model.prof = NvtxRanges())
        self.graphs: dict[int, _DecodeGraph] = {}
        self.graph_replays = 0
        # host seconds: staging inputs, enqueueing the forward, waiting for the step's results
        self.host_stage_s = 0.0
        self.host_enqueue_s = 0.0
        self.host_wait_s = 0.0

    def _make_staging(self, t: int, s: int):
        pin = dict(pin_memory=True)
        st = types.SimpleNamespace(
            h_i64=torch.empty(3 * t, dtype=torch.long, **pin),          # ids | positions | slots
            h_i32=torch.empty(3 * s + 1, dtype=torch.int32, **pin),     # starts | carry | kv_lens
            h_bt=torch.zeros(s, self.max_blocks, dtype=torch.int32, **pin),
            h_rows=torch.empty(s, dtype=torch.long, **pin),
            h_fb=torch.empty(2, s, dtype=torch.long, **pin),
            h_work=torch.empty(4, 4 * t + 4 * s, dtype=torch.int32, **pin),
            h2d_event=torch.cuda.Event(), h2d_pending=False)
        # numpy views of the pinned buffers (same memory)
        st.np_i64, st.np_i32 = st.h_i64.numpy(), st.h_i32.numpy()
        st.np_bt, st.np_rows, st.np_work = st.h_bt.numpy(), st.h_rows.numpy(), st.h_work.numpy()
        return st

    def _use_staging(self, slot: int) -> None:
        """Point the staging attributes at pinned set ``slot`` (its copy event travels with it)."""
        if getattr(self, "_slot", None) is not None:
            cur = self._staging[self._slot]
            cur.h2d_pending = self.h2d_pending
        st = self._staging[slot]
        self._slot = slot
        for k in ("h_i64", "h_i32", "h_bt", "h_rows", "h_fb", "h_work", "np_i64", "np_i32", "np_bt", "np_rows",
                  "np_work", "h2d_event"):
            setattr(self, k, getattr(st, k))
        self.h2d_pending = st.h2d_pending

    # ------------------------------------------------------------------ CUDA graphs
    def _graph_bucket(self, out: SchedulerOutput) -> int | None:
        if not self.use_cuda_graphs or not out.is_decode_only:
            return None
        n = len(out.chunks)
        m = self.model
        for b in GRAPH_BUCKETS:
            if n <= b <= m.max_seqs and b <= m.max_tokens:
                if self.tp_size > 1:
                    # every row-parallel reduction must be the fused epilogue + device-counted
                    # peer barrier, never an NCCL all-reduce
                    comm = getattr(m, "comm", None)
                    if comm is None or b > comm.red_max_tokens or getattr(m, "dual", False) or m.has_moe:
                        return None
                return b
        return None

    def _stage_graph(self, hb: HostBatch, p: int) -> None:
        """Stage a decode step padded to ``p`` rows at the fixed offsets the graphs read."""
        s = len(hb.ids)
        m = self.model
        if self._slot != 0:
            self._use_staging(0)
        if self.h2d_pending:
            self.h2d_event.synchronize()
        i64, i32 = self.np_i64, self.np_i32
        scratch = m.scratch_block * BLOCK_SIZE
        i64[:s] = hb.ids
        i64[s:p] = 0
        i64[p:p + s] = hb.pos
        i64[p + s:2 * p] = 0
        i64[2 * p:2 * p + s] = hb.slots
        i64[2 * p + s:3 * p] = scratch
        i32[: p + 1] = np.arange(p + 1, dtype=np.int32)
        i32[p + 1:p + 1 + s] = hb.carry
        i32[p + 1 + s:2 * p + 1] = 0
        i32[2 * p + 1:2 * p + 1 + s] = hb.kv_lens
        i32[2 * p + 1 + s:3 * p + 1] = 1
        width = hb.bt.shape[1]
        if width > self.max_blocks:
            raise ValueError(f"block table width {width} exceeds max_model_len blocks {self.max_blocks}")
        self.np_bt[:s, :width] = hb.bt
        self.np_bt[:s, width:] = 0
        self.np_bt[s:p, :] = m.scratch_block
        self.np_rows[:p] = np.arange(p)
        self.d_i64[: 3 * p].copy_(self.h_i64[: 3 * p], non_blocking=True)
        self.d_i32[: 3 * p + 1].copy_(self.h_i32[: 3 * p + 1], non_blocking=True)
        self.d_bt[:p].copy_(self.h_bt[:p], non_blocking=True)
        self.d_rows[:p].copy_(self.h_rows[:p], non_blocking=True)
        self._feed_back(hb, self.d_i64[:s])
        self.h2d_event.record()
        self.h2d_pending = True
        self.h2d_bytes += 8 * 3 * p + 4 * (3 * p + 1) + 4 * p * self.max_blocks + 8 * p

    def _feed_back(self, hb: HostBatch, ids: torch.Tensor) -> None:
        """Rows whose token was sampled by the previous (still running) step take it from that
        step's device buffer: one H2D copy of the row pairs and one gather."""
        n = len(hb.fb_dst)
        if n == 0:
            return
        if self.prev_buf is None:
            raise RuntimeError("a step feeds back sampled ids but no step was launched before it")
        hf = self.h_fb.numpy()
        hf[0, :n] = hb.fb_dst
        hf[1, :n] = hb.fb_src
        self.d_fb[:, :n].copy_(self.h_fb[:, :n], non_blocking=True)
        ids.index_copy_(0, self.d_fb[0, :n], self.d_tokens[self.prev_buf].index_select(0, self.d_fb[1, :n]))
        self.h2d_bytes += 16 * n

    def _graph_batch(self, p: int, work):
        from ..models.native import AttnPlan, StepBatch

        return StepBatch(num_tokens=p, num_seqs=p, ids=self.d_i64[:p], positions=self.d_i64[p:2 * p],
                         slots=self.d_i64[2 * p:3 * p], seq_starts=self.d_i32[: p + 1],
                         carry_in=self.d_i32[p + 1:2 * p + 1], kv_lens=self.d_i32[2 * p + 1:3 * p + 1],
                         block_table=self.d_bt[:p], logit_rows=self.d_rows[:p],
                         plans=[AttnPlan(work[0], work[1], self.model.fp8_decode_rows if self.model.kv_fp8 else 16,
                                         work[2])])

    def _run_graph(self, hb: HostBatch, p: int) -> torch.Tensor:
        from .. import _native
        from ..ops import attention as A

        self._stage_graph(hb, p)
        g = self.graphs.get(p)
        if g is None:
            m = self.model
            ws, wr = A.build_work([1] * p, m.num_q // m.num_kv, m.fp8_decode_rows if m.kv_fp8 else 16)
            ns = A.choose_splits(p * m.num_kv, self.max_blocks * BLOCK_SIZE)
            if ns > 1 and p > m.ws_tokens:
                ns = 1
            work = (torch.tensor(ws, dtype=torch.int32, device=self.device),
                    torch.tensor(wr, dtype=torch.int32, device=self.device), ns)
            batch = self._graph_batch(p, work)
            m.forward(batch)  # eager warm-up: one-time kernel set-up happens outside the capture
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            before = _native.launch_count()
            with torch.cuda.graph(graph):
                logits = m.forward(batch)
            launches = _native.launch_count() - before
            g = self.graphs[p] = _DecodeGraph(p, graph, logits, launches, work)
        g.graph.replay()
        _native.add_launches(g.launches)
        self.graph_replays += 1
        return g.logits[: len(hb.rows)]

    def _stage(self, hb: HostBatch, slot: int = 0):
        from ..models.native import AttnPlan, StepBatch

        if slot != self._slot:
            self._use_staging(slot)

        t, s = len(hb.ids), len(hb.starts) - 1
        m = self.model
        if t > m.max_tokens or s > m.max_seqs:
            raise ValueError(f"step of {t} tokens / {s} seqs exceeds buffers ({m.max_tokens}/{m.max_seqs})")
        # host staging (pinned): the previous step's async copies must have landed
        if self.h2d_pending:
            self.h2d_event.synchronize()
        i64, i32 = self.np_i64, self.np_i32
        i64[:t] = hb.ids
        i64[t:2 * t] = hb.pos
        i64[2 * t:3 * t] = hb.slots
        i32[: s + 1] = hb.starts
        i32[s + 1:2 * s + 1] = hb.carry
        i32[2 * s + 1:3 * s + 1] = hb.kv_lens
        width = hb.bt.shape[1]
        if width > self.max_blocks:
            raise ValueError(f"block table width {width} exceeds max_model_len blocks {self.max_blocks}")
        self.np_bt[:s, :width] = hb.bt
        nb = len(hb.rows)
        self.np_rows[:nb] = hb.rows
        plans_host = m.attention_plans(hb.q_lens, hb.kv_lens)
        for pi, (ws, wr, rows, ns) in enumerate(plans_host):
            self.np_work[2 * pi, : len(ws)] = ws
            self.np_work[2 * pi + 1, : len(wr)] = wr
        # H2D (one copy per staging buffer)
        self.d_i64[: 3 * t].copy_(self.h_i64[: 3 * t], non_blocking=True)
        self.d_i32[: 3 * s + 1].copy_(self.h_i32[: 3 * s + 1], non_blocking=True)
        self.d_bt[:s, :width].copy_(self.h_bt[:s, :width], non_blocking=True)
        self.d_rows[:nb].copy_(self.h_rows[:nb], non_blocking=True)
        nw = max((len(p[0]) for p in plans_host), default=0)
        if plans_host:
            self.d_work[: 2 * len(plans_host), :nw].copy_(self.h_work[: 2 * len(plans_host), :nw], non_blocking=True)
        self._feed_back(hb, self.d_i64[:t])
        self.h2d_event.record()
        self.h2d_pending = True
        self.h2d_bytes += 8 * 3 * t + 4 * (3 * s + 1) + 4 * s * width + 8 * nb + 4 * 2 * len(plans_host) * nw
        plans = [AttnPlan(self.d_work[2 * pi, : len(ws)], self.d_work[2 * pi + 1, : len(ws)], rows, ns)
                 for pi, (ws, wr, rows, ns) in enumerate(plans_host)]
        probe_groups = probe_all = None
        if m.probe_w is not None:
            marks = probe_markers(m.cfg, hb)
            if marks:
                # rare (probe calls only): small synchronous copies
                read = m.cfg.probe_read_layers or [None] * m.cfg.num_adapters
                dev = self.device
                groups = {}
                for j, r, slot in marks:
                    groups.setdefault(read[slot - 1], []).append((j, r, slot))
                probe_groups = []
                for layer, ms in groups.items():
                    rows = [r for _, r, _ in ms] if layer is not None else [j for j, _, _ in ms]
                    probe_groups.append((layer, torch.tensor(rows, dtype=torch.int32, device=dev),
                                         torch.tensor([sl for _, _, sl in ms], dtype=torch.int32, device=dev),
                                         torch.tensor([j for j, _, _ in ms], dtype=torch.int32, device=dev)))
                probe_all = (torch.tensor([j for j, _, _ in marks], dtype=torch.int32, device=dev),
                             torch.tensor([sl for _, _, sl in marks], dtype=torch.int32, device=dev))
                self.h2d_bytes += 4 * 5 * len(marks)
        return StepBatch(num_tokens=t, num_seqs=s, ids=self.d_i64[:t], positions=self.d_i64[t:2 * t],
                         slots=self.d_i64[2 * t:3 * t], seq_starts=self.d_i32[: s + 1],
                         carry_in=self.d_i32[s + 1:2 * s + 1], kv_lens=self.d_i32[2 * s + 1:3 * s + 1],
                         block_table=self.d_bt[:s, :width], logit_rows=self.d_rows[:nb], plans=plans,
                         probe_groups=probe_groups, probe_all=probe_all)

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
        with nvtx_range(f"step {len(hb.ids)} tokens", self.nvtx):
            p = self._graph_bucket(out)
            parts = self._pp_parts(out) if p is None else None
            if parts is not None:
                return hb, self._forward_parts(parts)
            if p is not None:
                t0 = time.perf_counter()
                logits = self._run_graph(hb, p)
                self.host_enqueue_s += time.perf_counter() - t0
            else:
                t0 = time.perf_counter()
                batch = self._stage(hb)
                t1 = time.perf_counter()
                logits = self.model.forward(batch)
                self.host_stage_s += t1 - t0
                self.host_enqueue_s += time.perf_counter() - t1
                if not len(hb.rows):
                    logits = None
            if self.routing_trace is not None:
                self._trace(hb)
            if logits is None:
                return hb, None
            return hb, self._gather_logits(logits)

    # smallest step split into micro-batches: below it the projections stream their weights
    # (bandwidth-bound), and two micro-batches would read every weight twice per stage
    PP_SPLIT_MIN_TOKENS = 1024

    def _pp_parts(self, out: SchedulerOutput):
        """Two micro-batches of about half the step's tokens each (whole sequences), so that
        stage s + 1 runs the first while stage s runs the second; None when the step is not
        split (no pipeline, one sequence, fewer than ``PP_SPLIT_MIN_TOKENS`` tokens, probe
        steps, routing trace on)."""
        m = self.model
        if (not self.pp_microbatches or m.probe_w is not None or self.routing_trace is not None
                or len(out.chunks) < 2 or out.num_tokens < self.PP_SPLIT_MIN_TOKENS):
            return None
        total, acc, k = out.num_tokens, 0, 0
        for k, c in enumerate(out.chunks):
            acc += c.num_tokens
            if 2 * acc >= total:
                break
        k = min(max(k + 1, 1), len(out.chunks) - 1)
        return [SchedulerOutput(chunks=out.chunks[:k]), SchedulerOutput(chunks=out.chunks[k:])]

    def _forward_parts(self, parts) -> torch.Tensor | None:
        """Run the micro-batches in order on this stage's stream. Each hands its hidden state
        to the next stage as soon as its layers finish, so the stages overlap; the last stage
        keeps each part's logits (the next part's forward rewrites the logits buffer) and
        returns them in the step's row order."""
        outs = []
        for i, part in enumerate(parts):
            hbp = HostBatch(part)
            t0 = time.perf_counter()
            batch = self._stage(hbp, slot=i)
            t1 = time.perf_counter()
            lg = self.model.forward(batch)
            self.host_stage_s += t1 - t0
            self.host_enqueue_s += time.perf_counter() - t1
            if lg is not None and len(hbp.rows):
                outs.append(self._gather_logits(lg).clone())
        return torch.cat(outs) if outs else None

    def _trace(self, hb: HostBatch) -> None:
        """Record this step's routing from the model's static buffers (valid after a graph replay too)."""
        t = len(hb.ids)
        m = self.model
        if m.n_maps:
            adapter = m.adapter_idx[:t].to("cpu", torch.int64)
            lora = m.lora_idx[:t].to("cpu", torch.int64)
        else:
            adapter = lora = torch.zeros(t, dtype=torch.int64)
        rec = self.routing_trace.record([c.req.request_id for c in hb.chunks], hb.ids, hb.pos, adapter, lora,
                                        torch.where(adapter != lora, adapter, 0))
        rec["spans"] = [(int(hb.starts[i]), int(hb.starts[i + 1])) for i in range(len(hb.chunks))]

    def execute(self, out: SchedulerOutput) -> list[int]:
        """Run one step and return its sampled ids (blocking)."""
        return self.collect(self.launch(out))

    def launch(self, out: SchedulerOutput) -> StepHandle:
        """Stage and enqueue one step (forward, sampling, copies of the ids and the error word)
        without waiting for it. Rows whose input is the previous launched step's sample read it
        on the device (``HostBatch.fb_dst``)."""
        from ..ops import elementwise as E
        from .sampling import sample

        hb, logits = self.compute_logits(out)
        nb = len(hb.rows)
        buf = self.buf
        toks = self.d_tokens[buf, :nb]
        if nb:
            pipe = self.model.pipeline
            if pipe is None or self.model.last_stage:
                params = [c.req.sampling for c in hb.chunks if c.needs_sample]
                if all(p.greedy for p in params):
                    E.argmax(logits, out=toks)
                else:
                    sample(logits, params, [c.req for c in hb.chunks if c.needs_sample], out=toks)
            if pipe is not None:
                pipe.broadcast_tokens(toks)  # every stage's scheduler sees the sampled ids
        self._stage_error_word(buf)
        if nb:
            self.h_out[buf, :nb].copy_(toks, non_blocking=True)
        ev = self.copy_events[buf]
        ev.record()
        self.d2h_bytes += 8 * nb + 12
        self.prev_buf, self.buf = buf, buf ^ 1
        return StepHandle(out, nb, buf, ev)

    def collect(self, h: StepHandle) -> list[int]:
        """Wait for a launched step's ids (raises :class:`DeviceError` if a kernel reported one)."""
        t0 = time.perf_counter()
        h.event.synchronize()
        self.host_wait_s += time.perf_counter() - t0
        self._raise_device_error(h.buf)
        return self.h_out[h.buf, :h.nb].tolist()

    def _stage_error_word(self, buf: int) -> None:
        """Queue the copy of the device error word next to the sampled ids.

        Under tensor or pipeline parallelism the word is max-reduced over the
        model's ranks first, so every rank sees a failure in the same step and
        the ranks stay in lock step when the engine aborts that step.
        """
        from .._native import err_buffer

        err = err_buffer(self.device)
        self.d_err.copy_(err[:3])
        group = None
        if self.model.pipeline is not None:
            group = torch.distributed.group.WORLD
        elif self.tp_size > 1:
            group = self.tp_group
        if group is not None:
            torch.distributed.all_reduce(self.d_err, op=torch.distributed.ReduceOp.MAX, group=group)
        self.h_err[buf].copy_(self.d_err, non_blocking=True)

    def _raise_device_error(self, buf: int) -> None:
        """After the step's copies landed: raise :class:`DeviceError` if a kernel reported one
        (and clear the device word, so the engine can go on with other requests)."""
        word = int(self.h_err[buf, 0])
        if not word:
            return
        from .._native import DeviceError, err_buffer, site_name

        site, idx = int(self.h_err[buf, 1]), int(self.h_err[buf, 2])
        err_buffer(self.device).zero_()
        self.h_err.zero_()
        raise DeviceError(word, site_name(site), idx if site else None)


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
        self.routing_trace = None
        self.last_tokens = np.zeros(0, np.int64)  # the last launched step's sampled ids

    def launch(self, out: SchedulerOutput) -> StepHandle:
        """Run the step now (CPU); rows fed back from the previous step read its ids here."""
        toks = self.execute(out)
        self.last_tokens = np.asarray(toks, np.int64)
        return StepHandle(out, len(toks), 0, None, toks)

    def collect(self, h: StepHandle) -> list[int]:
        return h.tokens

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
        from ..models.layers import rope_cos_sin
        from ..ops.attention import paged_attention_reference
        from ..routing.token_exchange import apply_token_exchange

        cfg = self.cfg
        hb = HostBatch(out)
        if len(hb.fb_dst):
            hb.ids[hb.fb_dst] = self.last_tokens[hb.fb_src]
        ids = torch.from_numpy(hb.ids)
        if self.table is not None:
            idx, _ = route_flat(ids, hb.starts.tolist(), hb.carry.tolist(), self.table)
            lora_idx, probe_idx = self.m.model.switch.split_indices(idx)
            lut = self.m.model.switch.control_to_substitute_lut
        else:
            idx = lora_idx = probe_idx = torch.zeros_like(ids)
            lut = None
        if self.routing_trace is not None:
            rec = self.routing_trace.record([c.req.request_id for c in hb.chunks], hb.ids, hb.pos, idx, lora_idx,
                                            probe_idx)
            rec["spans"] = [(int(hb.starts[i]), int(hb.starts[i + 1])) for i in range(len(hb.chunks))]
        mod = apply_token_exchange(lut, ids)
        pos = torch.from_numpy(hb.pos)
        slots = torch.from_numpy(hb.slots)
        h = self.m.model.embed_tokens(mod) * cfg.embedding_multiplier
        cos, sin = rope_cos_sin(pos.unsqueeze(0), cfg.head_dim_eff, cfg.rope_theta, h.dtype)
        bt = torch.from_numpy(hb.bt)
        blk, off = slots // BLOCK_SIZE, slots % BLOCK_SIZE
        markers = probe_markers(cfg, hb, probe_idx)
        verdict = {}
        head = self.m.model.probe_head
        read = cfg.probe_read_layers or [None] * cfg.num_adapters

        def score(layer, hidden):
            for j, r, slot in markers:
                if read[slot - 1] == layer:
                    verdict[j] = head(hidden[r].unsqueeze(0), torch.tensor([slot]))[0]

        n = len(hb.ids)
        li_b = lora_idx.unsqueeze(0)
        dual = bool(cfg.dual_stream)
        hbase = h if dual else None

        def attend(q, li, att):
            return paged_attention_reference(q[0].reshape(n, -1), self.kv[li, 0], self.kv[li, 1], bt, hb.q_lens,
                                             hb.kv_lens, cfg.num_attention_heads, att.scaling)

        for li, layer in enumerate(self.m.model.layers):
            att = layer.self_attn
            rm = layer.residual_multiplier
            if dual:
                # Shadow Residual: the base stream writes K/V; the adapter stream's
                # queries attend to that base K/V (its own K/V are never used)
                xb = layer.input_layernorm(hbase).unsqueeze(0)
                xa = layer.input_layernorm(h).unsqueeze(0)
                qb, k, v = att.project_qkv(xb, None, cos, sin)
                qa, _, _ = att.project_qkv(xa, li_b, cos, sin)
                self.kv[li, 0, blk, :, off] = k[0].to(self.kv.dtype)
                self.kv[li, 1, blk, :, off] = v[0].to(self.kv.dtype)
                ob, oa = attend(qb, li, att), attend(qa, li, att)
                hbase = hbase + att.out(ob.to(h.dtype).unsqueeze(0), None)[0] * rm
                h = h + att.out(oa.to(h.dtype).unsqueeze(0), li_b)[0] * rm
                xb = layer.post_attention_layernorm(hbase).unsqueeze(0)
                xa = layer.post_attention_layernorm(h).unsqueeze(0)
                routing = layer.block_sparse_moe.route(xb) if layer.block_sparse_moe is not None else None
                hbase = hbase + layer.mlp(xb, None, routing)[0] * rm
                h = h + layer.mlp(xa, li_b, routing)[0] * rm
                h = h + layer.cross_stream(hbase.unsqueeze(0), li_b)[0]
            else:
                x = layer.input_layernorm(h)
                q, k, v = att.project_qkv(x.unsqueeze(0), li_b, cos, sin)
                self.kv[li, 0, blk, :, off] = k[0].to(self.kv.dtype)
                self.kv[li, 1, blk, :, off] = v[0].to(self.kv.dtype)
                o = attend(q, li, att)
                h = h + att.out(o.to(h.dtype).unsqueeze(0), li_b)[0] * rm
                x = layer.post_attention_layernorm(h)
                h = h + layer.mlp(x.unsqueeze(0), li_b)[0] * rm
            score(li, h)
        if not len(hb.rows):
            return hb, None
        hf = self.m.model.norm(h[torch.from_numpy(hb.rows)])
        logits = self.m.lm_head(hf).float() / cfg.logits_scaling
        for j, _r, slot in markers:
            if read[slot - 1] is None:
                verdict[j] = head(hf[j].unsqueeze(0), torch.tensor([slot]))[0]
            labels = cfg.probe_label_token_ids[slot - 1]
            logits[j] = float("-inf")
            logits[j, torch.tensor(labels)] = verdict[j][: len(labels)].float()
        return hb, logits


def probe_markers(cfg, hb: HostBatch, probe_idx=None) -> list[tuple[int, int, int]]:
    """``(logit row j, flat token row, probe slot)`` for sampled rows that hold a probe control token.

    A probe's control token must be its request's last token, so a marker is
    always a row that samples (reference: src/granite_switch/hf/modeling_granite_switch.py:482-531).
    """
    ids = cfg.probe_control_token_ids or []
    if not ids or not len(hb.rows):
        return []
    tok = hb.ids[hb.rows]
    hit = np.flatnonzero(np.isin(tok, np.asarray(ids)))
    if not hit.size:
        return []
    off = len(cfg.adapter_token_ids or []) - cfg.num_adapters
    slot_of = {int(t): i - off + 1 for i, t in enumerate(cfg.adapter_token_ids or []) if i >= off}
    return [(int(j), int(hb.rows[j]), slot_of[int(tok[j])]) for j in hit]


__all__ = ["NativeExecutor", "ReferenceExecutor", "HostBatch", "probe_markers", "math"]
