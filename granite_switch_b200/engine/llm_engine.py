"""Serving engine: continuous batching over a paged, prefix-cached KV cache.

``LLMEngine`` is the step loop (add requests, ``step()``, collect finished
requests). ``LLM`` is the offline entry point: ``LLM(model_dir).generate(...)``.
Both run the same scheduler on every tensor-parallel rank (SPMD); ranks stay in
lockstep because every input to a scheduling decision (arrivals, sampled
tokens) is identical on all ranks.
"""
from __future__ import annotations

import logging
import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .._native import DeviceError, native
from ..config import GraniteSwitchConfig
from ..routing.scan import expert_table
from .kv_cache import BLOCK_SIZE, BlockManager
from .request import Request, RequestOutput, RequestStatus, SamplingParams
from .scheduler import Scheduler


_log = logging.getLogger(__name__)

# Engine steps a cold request may be passed over under cache-affinity admission
# before it goes first (about a minute of 8B-shape steps on one B200).
DEFAULT_MAX_WAIT_STEPS = 2000


@dataclass
class EngineConfig:
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    max_model_len: int = 8192
    num_kv_blocks: int | None = None       # None: size from free GPU memory
    gpu_memory_utilization: float = 0.88
    enable_prefix_caching: bool = True
    enable_chunked_prefill: bool = True
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    use_cuda_graphs: bool = True           # decode-only steps replay a captured graph (TP: fused reductions only)
    dtype: str = "bfloat16"
    seed: int = 0
    fused_tp_comm: bool = False            # symmetric-memory fused GEMM + reduction kernels
    scheduling_policy: str = "cache_affinity"  # or "fcfs" (admission order, see engine.scheduler)
    max_wait_steps: int | None = DEFAULT_MAX_WAIT_STEPS  # cache_affinity: steps before a cold request
    #                                                    goes first; None = unbounded
    kv_cache_dtype: str = "bfloat16"       # or "fp8_e4m3": e4m3 K/V with a per-(token, KV head) scale
    # launch step i+1 before reading step i's sampled ids (they reach step i+1's inputs on
    # the device), so scheduling and bookkeeping overlap the GPU
    async_scheduling: bool = True
    # pipeline parallelism: run each step as two micro-batches so consecutive stages overlap
    pipeline_microbatches: bool = True
    # launch the decode-sized GEMMs as programmatic dependents of the kernel before them:
    # they set up and start streaming weights while that kernel finishes (process-wide)
    programmatic_launch: bool = True
    # a step with decode rows and prefill chunks runs the prefill attention on a second
    # stream beside the decode attention
    overlap_attention: bool = True


@dataclass
class EngineStats:
    steps: int = 0
    prompt_tokens: int = 0
    generated_tokens: int = 0
    finished: int = 0
    ttfts: list = field(default_factory=list)
    latencies: list = field(default_factory=list)
    device_errors: int = 0   # steps aborted because a kernel reported an error
    prefill_tokens: int = 0  # tokens computed in prefill chunks (prompt tokens not served from cache)
    decode_rows: int = 0     # single-token decode rows
    # host seconds per phase (the GPU idles during schedule / stage / post unless work is queued)
    host_schedule_s: float = 0.0
    host_post_s: float = 0.0


class HostRouter:
    """Host copy of the routing rule, used to carry routing state across chunks.

    Long chunks (prefill) are scanned with a vectorised lookup table; short
    ones (decode) with a dict.
    """

    def __init__(self, config: GraniteSwitchConfig):
        self.map = {}
        self.lut = None
        if config.num_adapters > 0 and config.adapter_token_ids:
            tbl = expert_table(config.adapter_token_ids, config.num_adapters)
            for tok in config.adapter_token_ids:
                self.map[tok] = int(tbl[tok])
            self.lut = tbl.numpy().astype(np.int64)

    def __call__(self, ids, carry: int) -> int:
        m = self.map
        if not m:
            return carry
        if len(ids) > 32:
            a = np.asarray(ids, dtype=np.int64)
            lut = self.lut
            inside = a < lut.shape[0]
            e = np.where(inside, lut[np.where(inside, a, 0)], -1)
            hit = np.flatnonzero(e >= 0)
            return int(e[hit[-1]]) if hit.size else carry
        for t in reversed(ids):
            e = m.get(int(t))
            if e is not None:
                return e
        return carry


class LLMEngine:
    def __init__(self, config: GraniteSwitchConfig, executor, num_blocks: int, engine_config: EngineConfig | None = None):
        self.config = config
        self.ecfg = engine_config or EngineConfig()
        self.executor = executor
        self.blocks = BlockManager(num_blocks, self.ecfg.enable_prefix_caching)
        self.router = HostRouter(config)
        self.scheduler = Scheduler(self.blocks, self.ecfg.max_num_seqs, self.ecfg.max_num_batched_tokens,
                                   self.ecfg.enable_chunked_prefill, route_fn=self.router,
                                   policy=self.ecfg.scheduling_policy, max_wait_steps=self.ecfg.max_wait_steps)
        self.stats = EngineStats()
        self.requests: dict[str, Request] = {}
        self.eos = config.eos_token_id if isinstance(config.eos_token_id, int) else None
        self.on_finish = None  # optional callback(req)
        self.health = None     # optional parallel.health.Heartbeat (multi-rank)
        # async steps need an executor that launches without waiting, and no probe
        # control tokens (a probe marker is found from the sampled row's token id on the host)
        self.async_steps = (self.ecfg.async_scheduling and hasattr(executor, "launch")
                            and not (getattr(config, "probe_control_token_ids", None) or []))
        self._inflight = None  # StepHandle of the launched step whose ids are not read yet

    # -------------------------------------------------------------- requests
    def add_request(self, prompt_ids: list[int], sampling: SamplingParams | None = None,
                    request_id: str | None = None, arrival_time: float | None = None, user_data=None) -> Request:
        if len(prompt_ids) == 0:
            raise ValueError("empty prompt")
        sp = sampling or SamplingParams()
        if len(prompt_ids) + sp.max_tokens > self.ecfg.max_model_len:
            raise ValueError(f"prompt ({len(prompt_ids)}) + max_tokens ({sp.max_tokens}) exceeds "
                             f"max_model_len {self.ecfg.max_model_len}")
        req = Request(list(prompt_ids), sp, eos_token_id=self.eos, user_data=user_data)
        if request_id is not None:
            req.request_id = request_id
        if arrival_time is not None:
            req.arrival_time = arrival_time
        self.requests[req.request_id] = req
        self.scheduler.add(req)
        self.stats.prompt_tokens += len(prompt_ids)
        return req

    def abort_request(self, request_id: str) -> bool:
        r = self.requests.get(request_id)
        ok = self.scheduler.abort(request_id)
        if ok and r is not None:
            r.drop_pending()  # a token of the running step is discarded with the request
        return ok

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work() or self._inflight is not None

    # -------------------------------------------------------------- step
    def step(self) -> list[Request]:
        if self.async_steps:
            return self._step_async()
        t0 = time.perf_counter()
        out = self.scheduler.schedule()
        self.stats.host_schedule_s += time.perf_counter() - t0
        if not out.chunks:
            return []
        if self.health is not None:
            self.health.check()  # a dead peer is reported here, not inside a collective
        for c in out.chunks:
            if c.num_tokens > 1 or c.req.prefilling:
                self.stats.prefill_tokens += c.num_tokens
            else:
                self.stats.decode_rows += c.num_tokens
        try:
            tokens = self.executor.execute(out)
        except DeviceError as e:
            self._abort_step(out, e)
            raise
        if self.health is not None:
            self.health.beat()
        now = time.perf_counter()
        t_post = now
        finished = []
        j = 0
        for c in out.chunks:
            r = c.req
            end = c.start + c.num_tokens
            toks = r._np_tok[c.start:end] if r._np_tok_n >= end else r.all_ids[c.start:end]
            r.carry = self.router(toks, r.carry)
            r.num_computed = c.start + c.num_tokens
            self.blocks.register_full_blocks(r)
            if not c.needs_sample:
                continue
            tok = int(tokens[j])
            j += 1
            r.output_ids.append(tok)
            self.stats.generated_tokens += 1
            if r.first_token_time is None:
                r.first_token_time = now
            reason = self._stop_reason(r, tok)
            if reason:
                r.finish_time = now
                self.scheduler.finish(r, reason)
                finished.append(r)
                self.stats.finished += 1
                if r.ttft() is not None:
                    self.stats.ttfts.append(r.ttft())
                self.stats.latencies.append(r.finish_time - r.arrival_time)
                self.requests.pop(r.request_id, None)
                if self.on_finish is not None:
                    self.on_finish(r)
        self.stats.steps += 1
        self.stats.host_post_s += time.perf_counter() - t_post
        return finished

    def _count_mix(self, out) -> None:
        for c in out.chunks:
            if c.num_tokens > 1 or c.req.prefilling:
                self.stats.prefill_tokens += c.num_tokens
            else:
                self.stats.decode_rows += c.num_tokens

    def _step_async(self) -> list[Request]:
        """One pipelined step: finish the bookkeeping of the running step that needs no
        sampled values (positions, routing carry, published blocks, a placeholder per
        sampled row), schedule and launch the next step (its decode rows take the running
        step's ids on the device), then wait for the running step's ids and resolve them
        (stop checks, finished requests). A request whose last token stops it was scheduled
        once more; that row's result is dropped. Returns the requests finished by the
        step whose ids were resolved."""
        inflight = self._inflight  # the launched step's handle, or None
        self._inflight = None       # owned by this call from here on
        t0 = time.perf_counter()
        sampled = self._advance(inflight) if inflight is not None else None
        handle = None
        out = None
        try:
            out = self.scheduler.schedule()
            self.stats.host_schedule_s += time.perf_counter() - t0
            if out.chunks:
                if self.health is not None:
                    self.health.check()
                self._count_mix(out)
                handle = self.executor.launch(out)
        except DeviceError as e:
            self._abort_step(out, e, extra=inflight.out if inflight is not None else None)
            raise
        except BaseException:
            # the running step was advanced above: resolve it now so no step is lost or
            # advanced twice; the step that failed to launch is scheduled again next time
            if inflight is not None:
                self._resolve(sampled, self.executor.collect(inflight))
            raise
        finished = []
        if inflight is not None:
            try:
                toks = self.executor.collect(inflight)
            except DeviceError as e:
                if handle is not None:
                    try:
                        self.executor.collect(handle)  # drain it; its ids are discarded
                    except DeviceError:
                        pass
                self._abort_step(inflight.out, e, extra=out)
                raise
            if self.health is not None:
                self.health.beat()
            t_post = time.perf_counter()
            finished = self._resolve(sampled, toks)
            self.stats.host_post_s += time.perf_counter() - t_post
            self.stats.steps += 1
        self._inflight = handle
        return finished

    def _advance(self, handle) -> list:
        """Bookkeeping of a launched step that needs no sampled value; appends a placeholder
        for every sampled row and returns them, ``(request, output index, row)``, for
        :meth:`_resolve`."""
        sampled = []
        row = 0
        for c in handle.out.chunks:
            r = c.req
            ns = c.needs_sample
            if r.status == RequestStatus.FINISHED:
                row += ns
                continue
            end = c.start + c.num_tokens
            toks = r._np_tok[c.start:end] if r._np_tok_n >= end else r.all_ids[c.start:end]
            r.carry = self.router(toks, r.carry)
            r.num_computed = end
            self.blocks.register_full_blocks(r)
            if ns:
                r.set_pending(row)
                sampled.append((r, r.pending, row))
                if len(r.output_ids) >= r.sampling.max_tokens:
                    r.finishing = True
                row += 1
        return sampled

    def _resolve(self, sampled, toks) -> list[Request]:
        now = time.perf_counter()
        finished = []
        for r, idx, row in sampled:
            if r.status == RequestStatus.FINISHED or r.pending != idx:
                continue  # aborted while its step ran
            tok = int(toks[row])
            r.resolve_pending(tok)
            self.stats.generated_tokens += 1
            if r.first_token_time is None:
                r.first_token_time = now
            reason = self._stop_reason(r, tok)
            if reason:
                self._finish(r, reason, now)
                finished.append(r)
        return finished

    def _finish(self, r: Request, reason: str, now: float) -> None:
        r.finish_time = now
        r.finishing = False
        self.scheduler.finish(r, reason)
        self.stats.finished += 1
        if r.ttft() is not None:
            self.stats.ttfts.append(r.ttft())
        self.stats.latencies.append(r.finish_time - r.arrival_time)
        self.requests.pop(r.request_id, None)
        if self.on_finish is not None:
            self.on_finish(r)

    def _abort_step(self, out, err, extra=None) -> None:
        """A kernel of this step reported an error: its outputs cannot be trusted.

        Every request the step carried is finished with reason ``"error"`` (its
        blocks freed, never published), and the prefix cache is dropped: a bad
        index is replaced by entry 0 on the device, so a cached page may have
        been overwritten. Other waiting and running requests go on.
        """
        now = time.perf_counter()
        self.stats.device_errors += 1
        chunks = (list(out.chunks) if out is not None else []) + (list(extra.chunks) if extra is not None else [])
        for c in chunks:
            r = c.req
            if r.status == RequestStatus.FINISHED:
                continue
            r.drop_pending()
            r.finishing = False
            r.finish_time = now
            self.scheduler.finish(r, "error")
            self.requests.pop(r.request_id, None)
        for r in list(self.scheduler.running):  # their pages are suspect too: recompute them
            self.scheduler.preempt(r)
        self.blocks.reset_prefix_cache()
        _log.error("engine step aborted %d request(s): %s", len(chunks), err)

    def _stop_reason(self, r: Request, tok: int) -> str | None:
        sp = r.sampling
        n = len(r.output_ids)
        if n >= sp.max_tokens:
            return "length"
        if n >= sp.min_tokens:
            if tok in sp.stop_token_ids:
                return "stop"
            if not sp.ignore_eos and r.eos_token_id is not None and tok == r.eos_token_id:
                return "stop"
        return None

    # -------------------------------------------------------------- metrics
    def prefix_cache_hit_rate(self) -> float:
        return self.blocks.hits / max(1, self.blocks.queries)

    def metrics(self) -> dict:
        return {
            "num_requests_running": len(self.scheduler.running),
            "num_requests_waiting": self.scheduler.num_waiting,
            "prefix_cache_queries_total": self.blocks.queries,
            "prefix_cache_hits_total": self.blocks.hits,
            "generation_tokens_total": self.stats.generated_tokens,
            "prompt_tokens_total": self.stats.prompt_tokens,
            "kv_cache_usage_perc": self.blocks.usage(),
            "num_preemptions_total": self.scheduler.num_preemptions,
        }


def _to_output(r: Request) -> RequestOutput:
    return RequestOutput(r.request_id, r.prompt_ids, r.output_ids, r.finish_reason, r.num_cached_tokens,
                         r.ttft(), None if r.finish_time is None else r.finish_time - r.arrival_time)


class LLM:
    """Offline generation over a composed checkpoint (or a random-init config).

    ``LLM(path)`` loads a composed Granite Switch directory; on a CUDA device it
    runs the native kernels, on CPU the PyTorch reference executor.
    """

    def __init__(self, model: str | GraniteSwitchConfig, device: str | None = None,
                 engine_config: EngineConfig | None = None, random_init: dict | None = None,
                 tp_rank: int = 0, tp_group=None, pipeline=None):
        ecfg = engine_config or EngineConfig()
        self.ecfg = ecfg
        if device is None:
            device = "cuda" if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        if isinstance(model, GraniteSwitchConfig):
            config, path = model, None
        else:
            config, path = GraniteSwitchConfig.from_pretrained(model), model
        self.config = config
        tp = ecfg.tensor_parallel_size
        if self.device.type == "cuda":
            from ..models.native import NativeGraniteSwitch, default_num_kv_blocks
            from .executor import NativeExecutor

            max_tokens = max(ecfg.max_num_batched_tokens, ecfg.max_num_seqs)
            nb = ecfg.num_kv_blocks or 64
            if path is not None:
                from ..checkpoint import LazyCheckpoint

                # tensors are read one at a time from the memory-mapped shards, each rank
                # keeping only its shard; the loader audits that none went unused
                ckpt = LazyCheckpoint(path)
                nm = NativeGraniteSwitch.from_state_dict(config, ckpt, self.device, max_tokens, 1, tp_rank, tp,
                                                         tp_group, ecfg.max_num_seqs, pipeline)
                ckpt.close()
            else:
                ri = dict(random_init or {})
                nm = NativeGraniteSwitch.from_random(config, self.device, max_tokens, 1, tp_rank=tp_rank,
                                                     tp_size=tp, tp_group=tp_group, max_seqs=ecfg.max_num_seqs,
                                                     pipeline=pipeline, **ri)
            if ecfg.kv_cache_dtype not in ("bfloat16", "fp8_e4m3"):
                raise ValueError(f"kv_cache_dtype must be 'bfloat16' or 'fp8_e4m3', got {ecfg.kv_cache_dtype!r}")
            nm.kv_fp8 = ecfg.kv_cache_dtype == "fp8_e4m3"
            native().set_pdl(bool(ecfg.programmatic_launch))
            nm.overlap_attention = bool(ecfg.overlap_attention)
            if ecfg.num_kv_blocks is None:
                torch.cuda.synchronize()
                nb = default_num_kv_blocks(0, config, tp, ecfg.gpu_memory_utilization, self.device,
                                           num_layers=nm.num_layers, kv_fp8=nm.kv_fp8)
            nm.num_kv_blocks = nb
            nm._alloc_buffers()
            self.model = nm
            executor = NativeExecutor(nm, ecfg.max_model_len, tp_group, tp, ecfg.use_cuda_graphs,
                                      ecfg.pipeline_microbatches)
            if ecfg.fused_tp_comm and tp > 1 and pipeline is None:
                from ..parallel.fused import attach_fused_comm

                attach_fused_comm(nm, tp_group)
        else:
            from ..models.reference import GraniteSwitchForCausalLM
            from .executor import ReferenceExecutor

            if path is None:
                raise ValueError("the CPU executor needs a checkpoint directory")
            ref = GraniteSwitchForCausalLM.from_pretrained(path).eval()
            nb = ecfg.num_kv_blocks or 256
            executor = ReferenceExecutor(ref, nb)
            self.model = ref
        self.engine = LLMEngine(config, executor, nb, ecfg)
        # tracing toggles: NVTX ranges per step and forward region; per-step routing records
        if os.environ.get("GSB_NVTX", "0") == "1" and hasattr(executor, "nvtx"):
            from ..utils.tracing import NvtxRanges

            executor.nvtx = True
            executor.model.prof = NvtxRanges(executor.model.prof)
        if os.environ.get("GSB_ROUTING_TRACE"):
            self.enable_routing_trace(os.environ["GSB_ROUTING_TRACE"])

    def enable_routing_trace(self, path: str | None = None):
        """Record each step's routing (ids, positions, adapter / LoRA / probe index per token);
        returns the :class:`~granite_switch_b200.utils.tracing.RoutingTrace`."""
        from ..utils.tracing import RoutingTrace

        self.engine.executor.routing_trace = RoutingTrace(path)
        return self.engine.executor.routing_trace

    def generate(self, prompts: list[list[int]], sampling: SamplingParams | list[SamplingParams] | None = None,
                 audios: list | None = None, audio_processor=None) -> list[RequestOutput]:
        """Generate for token-id prompts.

        ``audios[i]`` (with ``audio_processor``, an
        :class:`~granite_switch_b200.audio.AudioPromptProcessor`) lists prompt
        ``i``'s clips; each ``<|audio|>`` marker is replaced by its transcript.
        """
        if audios is not None:
            if audio_processor is None:
                raise ValueError("audios given without an audio_processor")
            prompts = [audio_processor.expand(p, a) for p, a in zip(prompts, audios)]
        sps = sampling if isinstance(sampling, list) else [sampling or SamplingParams()] * len(prompts)
        reqs = [self.engine.add_request(p, sp) for p, sp in zip(prompts, sps)]
        while self.engine.has_unfinished():
            self.engine.step()
        return [_to_output(r) for r in reqs]


__all__ = ["LLM", "LLMEngine", "EngineConfig", "SamplingParams", "BLOCK_SIZE", "DEFAULT_MAX_WAIT_STEPS", "os"]
