"""Continuous batching with chunked prefill (one token budget per step).

Each step: running requests first (one decode token, or their next prefill
chunk), then waiting requests while the token budget, the sequence cap and
free KV blocks allow. A new request first acquires its longest cached prefix.
When a running request cannot get a block, the most recently admitted running
request is preempted (its blocks are freed; it recomputes later, largely from
the prefix cache).

Admission order (``policy``):

* ``"fcfs"``: arrival order (vLLM's default policy).
* ``"cache_affinity"``: requests whose first KV block is in the prefix cache
  when they arrive (the next call of a conversation, a preempted request, a
  prompt sharing a cached system prompt) are admitted before cold ones, in
  arrival order within each class. Under overload this finishes the
  conversations whose context is resident instead of prefilling new contexts
  that evict it, so each generated token costs less prefill; an idle or
  lightly loaded server admits everything at once either way. This is the
  longest-prefix-first idea of cache-aware schedulers reduced to one O(1)
  probe per request at arrival, so scheduling cost does not grow with the
  queue. ``max_wait_steps`` bounds how long a cold request can be passed
  over: once the oldest cold request has waited that many engine steps, it
  is admitted ahead of warm ones. The bound counts steps, not seconds, so
  every tensor-parallel rank takes the same decision.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from .kv_cache import BlockManager
from .request import Request, RequestStatus


@dataclass
class ScheduledChunk:
    req: Request
    start: int        # first token position computed in this step
    num_tokens: int

    @property
    def needs_sample(self) -> bool:
        return self.start + self.num_tokens >= self.req.num_tokens


@dataclass
class SchedulerOutput:
    chunks: list[ScheduledChunk] = field(default_factory=list)
    preempted: list[Request] = field(default_factory=list)

    @property
    def num_tokens(self) -> int:
        return sum(c.num_tokens for c in self.chunks)

    @property
    def is_decode_only(self) -> bool:
        return all(c.num_tokens == 1 and not c.req.prefilling for c in self.chunks)


POLICIES = ("fcfs", "cache_affinity")


class Scheduler:
    def __init__(self, blocks: BlockManager, max_num_seqs: int = 256, max_num_batched_tokens: int = 8192,
                 enable_chunked_prefill: bool = True, route_fn=None, policy: str = "fcfs",
                 max_wait_steps: int | None = None):
        if policy not in POLICIES:
            raise ValueError(f"unknown scheduling policy {policy!r} (expected one of {POLICIES})")
        self.policy = policy
        self.blocks = blocks
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.chunked = enable_chunked_prefill
        self.waiting: deque[Request] = deque()  # cold requests (every request under "fcfs")
        self.warm: deque[Request] = deque()     # "cache_affinity": first block cached at arrival
        self.running: list[Request] = []
        self.route_fn = route_fn  # (ids, carry) -> carry after ids
        self.num_preemptions = 0
        self.max_wait_steps = max_wait_steps
        self.steps = 0
        self.num_admitted = 0       # requests admitted from the waiting queues (first admissions)
        self.num_admitted_cold = 0  # ... of which no prompt block was found in the prefix cache

    def add(self, req: Request) -> None:
        req.status = RequestStatus.WAITING
        req.enqueue_step = self.steps
        if self.policy == "cache_affinity" and self.blocks.first_block_cached(req.prompt_ids):
            self.warm.append(req)
        else:
            self.waiting.append(req)

    @property
    def num_waiting(self) -> int:
        return len(self.waiting) + len(self.warm)

    def has_work(self) -> bool:
        return bool(self.waiting or self.warm or self.running)

    def _preempt(self, req: Request, out: SchedulerOutput | None) -> None:
        self.running.remove(req)
        self.blocks.free_request(req)
        req.num_computed = 0
        req.carry = 0
        req.matched = False
        req.status = RequestStatus.PREEMPTED
        # resumes first: its computed blocks stay cached until evicted
        (self.warm if self.policy == "cache_affinity" else self.waiting).appendleft(req)
        if out is not None:
            out.preempted.append(req)
        self.num_preemptions += 1

    def preempt(self, req: Request) -> None:
        """Free a running request's blocks and queue it to recompute from its prompt and
        generated tokens (ahead of other waiting requests)."""
        self._preempt(req, None)

    def _next_queue(self) -> deque:
        if not self.warm:
            return self.waiting
        if (self.max_wait_steps is not None and self.waiting
                and self.steps - self.waiting[0].enqueue_step >= self.max_wait_steps):
            return self.waiting  # the oldest cold request has waited long enough
        return self.warm

    def schedule(self) -> SchedulerOutput:
        self.steps += 1
        out = SchedulerOutput()
        budget = self.max_num_batched_tokens
        scheduled = set()
        # ---- running requests
        i = 0
        while i < len(self.running) and budget > 0:
            req = self.running[i]
            if req.finishing:  # its last token is still on the device
                i += 1
                continue
            remaining = req.num_tokens - req.num_computed
            n = min(remaining, budget) if self.chunked else remaining
            if n <= 0 or n > budget:
                i += 1
                continue
            while not self.blocks.allocate(req, req.num_computed + n):
                victim = self.running[-1]
                if victim is req:
                    self._preempt(req, out)
                    req = None
                    break
                self._preempt(victim, out)
            if req is None:
                continue
            out.chunks.append(ScheduledChunk(req, req.num_computed, n))
            scheduled.add(id(req))
            budget -= n
            i += 1
        # ---- waiting requests
        while budget > 0 and len(self.running) < self.max_num_seqs:
            queue = self._next_queue()
            if not queue:
                break
            req = queue[0]
            if not req.matched:
                req.matched = True
                hit = self.blocks.match_prefix(req)
                req.num_computed = hit
                req.num_cached_tokens = hit
                self.num_admitted += 1
                self.num_admitted_cold += int(hit == 0)
                req.carry = self.route_fn(req.prompt_ids[:hit], 0) if (self.route_fn and hit) else 0
            remaining = req.num_tokens - req.num_computed
            n = min(remaining, budget) if self.chunked else remaining
            if n > budget or not self.blocks.allocate(req, req.num_computed + n):
                break  # keep the admission order; retry next step
            queue.popleft()
            req.status = RequestStatus.RUNNING
            self.running.append(req)
            out.chunks.append(ScheduledChunk(req, req.num_computed, n))
            budget -= n
        return out

    def finish(self, req: Request, reason: str) -> None:
        req.status = RequestStatus.FINISHED
        req.finish_reason = reason
        if req in self.running:
            self.running.remove(req)
        else:  # preempted while its last step ran (async steps)
            for q in (self.warm, self.waiting):
                if req in q:
                    q.remove(req)
        self.blocks.free_request(req)

    def abort(self, request_id: str) -> bool:
        for q in (self.running, self.warm, self.waiting):
            for r in list(q):
                if r.request_id == request_id:
                    q.remove(r)
                    self.blocks.free_request(r)
                    r.status = RequestStatus.FINISHED
                    r.finish_reason = "abort"
                    return True
        return False
