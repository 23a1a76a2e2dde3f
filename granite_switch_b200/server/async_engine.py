"""Thread-backed asynchronous front end of :class:`~granite_switch_b200.engine.LLMEngine`.

One background thread owns the engine and runs ``step()`` while work exists;
HTTP handlers submit requests through a lock-protected inbox and await an
``asyncio`` future (or an async token stream) resolved from that thread. The
engine itself is single-threaded, so nothing else touches it.
"""
from __future__ import annotations

import asyncio
import threading
import time
from dataclasses import dataclass, field

from .._native import DeviceError
from ..engine.request import Request, SamplingParams


@dataclass
class _Pending:
    prompt_ids: list[int]
    sampling: SamplingParams
    loop: asyncio.AbstractEventLoop
    future: asyncio.Future
    stream: asyncio.Queue | None = None
    request_id: str | None = None
    submitted: float = field(default_factory=time.perf_counter)


class Histogram:
    """Prometheus-style cumulative histogram (seconds)."""

    def __init__(self, buckets):
        self.buckets = list(buckets)
        self.counts = [0] * (len(self.buckets) + 1)
        self.total = 0.0
        self.n = 0

    def observe(self, v: float):
        self.total += v
        self.n += 1
        for i, b in enumerate(self.buckets):
            if v <= b:
                self.counts[i] += 1
                return
        self.counts[-1] += 1

    def lines(self, name: str, labels: str) -> list[str]:
        out, cum = [], 0
        for b, c in zip(self.buckets, self.counts):
            cum += c
            out.append(f'{name}_bucket{{{labels},le="{b}"}} {cum}')
        cum += self.counts[-1]
        out.append(f'{name}_bucket{{{labels},le="+Inf"}} {cum}')
        out.append(f"{name}_sum{{{labels}}} {self.total}")
        out.append(f"{name}_count{{{labels}}} {self.n}")
        return out


_LAT_BUCKETS = (0.001, 0.005, 0.01, 0.02, 0.04, 0.06, 0.08, 0.1, 0.25, 0.5, 0.75, 1.0, 2.5, 5.0, 7.5, 10.0,
                20.0, 40.0, 80.0)


class StepSync:
    """Lock-step control channel of a multi-rank engine (tensor / pipeline parallel).

    Every rank runs the same scheduler, so every rank must see the same
    requests in the same order before each step: rank 0 (the one serving
    HTTP) publishes, over a CPU process group, the requests it added and
    aborted since the last step and whether to step; the other ranks replay
    that in :func:`follow` and step with it, so the collectives inside the step
    line up. An idle rank 0 publishes a heartbeat every ``heartbeat_s``.
    """

    def __init__(self, group, heartbeat_s: float = 1.0):
        import torch.distributed as dist

        self.group = group
        self.src = dist.get_global_rank(group, 0) if group is not None else 0
        self.heartbeat_s = heartbeat_s
        self.adds: list[tuple] = []
        self.aborts: list[str] = []
        self.last = time.perf_counter()

    def add(self, req: Request) -> None:
        from dataclasses import asdict

        self.adds.append((list(req.prompt_ids), asdict(req.sampling), req.request_id, req.arrival_time))

    def abort(self, request_id: str) -> None:
        self.aborts.append(request_id)

    def publish(self, step: bool, stop: bool = False) -> None:
        import torch.distributed as dist

        pkt = [{"add": self.adds, "abort": self.aborts, "step": step, "stop": stop}]
        dist.broadcast_object_list(pkt, src=self.src, group=self.group)
        self.adds, self.aborts = [], []
        self.last = time.perf_counter()

    def idle(self) -> None:
        if time.perf_counter() - self.last >= self.heartbeat_s:
            self.publish(step=False)


def follow(engine, group) -> None:
    """Loop of a rank other than 0: replay rank 0's request changes and step with it until told to stop."""
    import torch.distributed as dist

    src = dist.get_global_rank(group, 0) if group is not None else 0
    while True:
        pkt = [None]
        dist.broadcast_object_list(pkt, src=src, group=group)
        p = pkt[0]
        for ids, sp, rid, arrival in p["add"]:
            engine.add_request(ids, SamplingParams(**sp), request_id=rid, arrival_time=arrival)
        for rid in p["abort"]:
            engine.abort_request(rid)
        if p["stop"]:
            return
        if p["step"]:
            try:
                engine.step()
            except DeviceError:
                # every rank sees the same (max-reduced) error word and aborts the same
                # step; rank 0 then publishes the aborts of its remaining requests
                pass


class AsyncEngine:
    def __init__(self, engine, model_name: str = "granite-switch", sync: StepSync | None = None):
        self.engine = engine
        self.model_name = model_name
        self.sync = sync
        self._inbox: list[_Pending] = []
        self._lock = threading.Lock()
        self._wake = threading.Event()
        self._live: dict[str, _Pending] = {}
        self._stop = False
        self.ttft = Histogram(_LAT_BUCKETS)
        self.e2e = Histogram(_LAT_BUCKETS)
        self.prompt_tokens = Histogram((1, 16, 64, 256, 1024, 4096, 16384, 65536))
        self.errors = 0
        self._thread = threading.Thread(target=self._run, name="gsb-engine", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------ submission
    async def generate(self, prompt_ids: list[int], sampling: SamplingParams) -> Request:
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        with self._lock:
            self._inbox.append(_Pending(list(prompt_ids), sampling, loop, fut))
        self._wake.set()
        return await fut

    async def stream(self, prompt_ids: list[int], sampling: SamplingParams):
        """Yield lists of new token ids as they are produced; the last item is the Request."""
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        q: asyncio.Queue = asyncio.Queue()
        with self._lock:
            self._inbox.append(_Pending(list(prompt_ids), sampling, loop, fut, stream=q))
        self._wake.set()
        while True:
            item = await q.get()
            yield item
            if isinstance(item, Request):
                return

    def shutdown(self):
        self._stop = True
        self._wake.set()
        self._thread.join(timeout=10)
        if self.sync is not None:
            self.sync.publish(step=False, stop=True)  # release the follower ranks

    # ------------------------------------------------------------ engine thread
    def _run(self):
        emitted: dict[str, int] = {}
        while not self._stop:
            with self._lock:
                inbox, self._inbox = self._inbox, []
            for p in inbox:
                try:
                    req = self.engine.add_request(p.prompt_ids, p.sampling, arrival_time=p.submitted)
                    p.request_id = req.request_id
                    self._live[req.request_id] = p
                    if self.sync is not None:
                        self.sync.add(req)
                    self.prompt_tokens.observe(len(p.prompt_ids))
                except Exception as e:  # invalid request: fail only this one
                    self.errors += 1
                    p.loop.call_soon_threadsafe(_set_exc, p.future, e)
            if not self.engine.has_unfinished():
                if self.sync is not None:
                    self.sync.idle()
                self._wake.wait(timeout=0.05)
                self._wake.clear()
                continue
            try:
                if self.sync is not None:
                    self.sync.publish(step=True)
                finished = self.engine.step()
            except Exception as e:  # a failing step aborts the requests it carried
                self.errors += 1
                for rid, p in list(self._live.items()):
                    self.engine.abort_request(rid)
                    if self.sync is not None:
                        self.sync.abort(rid)
                    p.loop.call_soon_threadsafe(_set_exc, p.future, e)
                self._live.clear()
                continue
            for rid, p in list(self._live.items()):
                if p.stream is None:
                    continue
                r = self._find(rid, finished)
                if r is None:
                    continue
                n = emitted.get(rid, 0)
                if len(r.output_ids) > n:
                    p.loop.call_soon_threadsafe(p.stream.put_nowait, list(r.output_ids[n:]))
                    emitted[rid] = len(r.output_ids)
            for r in finished:
                p = self._live.pop(r.request_id, None)
                emitted.pop(r.request_id, None)
                if p is None:
                    continue
                if r.ttft() is not None:
                    self.ttft.observe(r.ttft())
                if r.finish_time is not None:
                    self.e2e.observe(r.finish_time - r.arrival_time)
                if p.stream is not None:
                    p.loop.call_soon_threadsafe(p.stream.put_nowait, r)
                p.loop.call_soon_threadsafe(_set_result, p.future, r)

    def _find(self, rid, finished):
        for r in finished:
            if r.request_id == rid:
                return r
        return self.engine.requests.get(rid)

    # ------------------------------------------------------------ metrics
    def metrics_text(self) -> str:
        m = self.engine.metrics()
        lab = f'model_name="{self.model_name}"'
        lines = []
        for prefix in ("vllm:", "gsb:"):
            lines += [
                f"# TYPE {prefix}num_requests_running gauge",
                f"{prefix}num_requests_running{{{lab}}} {m['num_requests_running']}",
                f"# TYPE {prefix}num_requests_waiting gauge",
                f"{prefix}num_requests_waiting{{{lab}}} {m['num_requests_waiting']}",
                f"# TYPE {prefix}kv_cache_usage_perc gauge",
                f"{prefix}kv_cache_usage_perc{{{lab}}} {m['kv_cache_usage_perc']}",
                f"# TYPE {prefix}prefix_cache_queries_total counter",
                f"{prefix}prefix_cache_queries_total{{{lab}}} {m['prefix_cache_queries_total']}",
                f"# TYPE {prefix}prefix_cache_hits_total counter",
                f"{prefix}prefix_cache_hits_total{{{lab}}} {m['prefix_cache_hits_total']}",
                f"# TYPE {prefix}generation_tokens_total counter",
                f"{prefix}generation_tokens_total{{{lab}}} {m['generation_tokens_total']}",
                f"# TYPE {prefix}prompt_tokens_total counter",
                f"{prefix}prompt_tokens_total{{{lab}}} {m['prompt_tokens_total']}",
                f"# TYPE {prefix}num_preemptions_total counter",
                f"{prefix}num_preemptions_total{{{lab}}} {m['num_preemptions_total']}",
                f"# TYPE {prefix}time_to_first_token_seconds histogram",
                *self.ttft.lines(f"{prefix}time_to_first_token_seconds", lab),
                f"# TYPE {prefix}e2e_request_latency_seconds histogram",
                *self.e2e.lines(f"{prefix}e2e_request_latency_seconds", lab),
                f"# TYPE {prefix}request_prompt_tokens histogram",
                *self.prompt_tokens.lines(f"{prefix}request_prompt_tokens", lab),
            ]
        return "\n".join(lines) + "\n"


def _set_result(fut, v):
    if not fut.done():
        fut.set_result(v)


def _set_exc(fut, e):
    if not fut.done():
        fut.set_exception(e)
