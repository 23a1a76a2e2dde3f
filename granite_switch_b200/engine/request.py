"""Request state and sampling parameters of the serving engine."""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field

_ids = itertools.count()


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0          # 0 = greedy
    top_k: int = 0                    # 0 = off
    top_p: float = 1.0
    seed: int | None = None
    stop_token_ids: tuple[int, ...] = ()
    ignore_eos: bool = False
    min_tokens: int = 0

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0


class RequestStatus(enum.Enum):
    WAITING = 0
    RUNNING = 1
    PREEMPTED = 2
    FINISHED = 3


PENDING_TOKEN = -1  # placeholder id of a sampled token not yet copied to the host


@dataclass
class Request:
    prompt_ids: list[int]
    sampling: SamplingParams = field(default_factory=SamplingParams)
    request_id: str = field(default_factory=lambda: f"req-{next(_ids)}")
    arrival_time: float = field(default_factory=time.perf_counter)
    eos_token_id: int | None = None
    output_ids: list[int] = field(default_factory=list)
    status: RequestStatus = RequestStatus.WAITING
    enqueue_step: int = 0              # scheduler step at which it (re)entered a waiting queue
    num_computed: int = 0              # tokens whose KV is in the cache
    block_ids: list[int] = field(default_factory=list)
    block_hashes: list[int] = field(default_factory=list)  # chained hashes of full blocks
    num_registered_blocks: int = 0     # full blocks published to the prefix cache
    num_cached_tokens: int = 0         # prefix-cache hit at admission
    carry: int = 0                     # routing carry after num_computed tokens
    matched: bool = False              # prefix cache consulted for the current admission
    # async steps: index in output_ids of a sampled token whose value is still on the
    # device (PENDING_TOKEN there), its row in that step's sampled-token buffer, and
    # whether that token completes max_tokens (then the request is not scheduled again)
    pending: int = -1
    pending_row: int = -1
    finishing: bool = False
    first_token_time: float | None = None
    finish_time: float | None = None
    finish_reason: str | None = None
    user_data: object = None
    _all: list = field(default=None, init=False, repr=False, compare=False)
    # host step-packing mirrors (numpy), maintained by engine.executor.HostBatch
    _np_tok: object = field(default=None, init=False, repr=False, compare=False)
    _np_tok_n: int = field(default=0, init=False, repr=False, compare=False)
    _np_bt: object = field(default=None, init=False, repr=False, compare=False)
    _np_bt_n: int = field(default=0, init=False, repr=False, compare=False)
    _np_bt_src: object = field(default=None, init=False, repr=False, compare=False)

    @property
    def all_ids(self) -> list[int]:
        """Prompt followed by the generated tokens (a maintained list; do not mutate).

        Kept incrementally instead of concatenating on every access: the engine
        reads a slice of it for every scheduled chunk of every step.
        """
        a = self._all
        p = len(self.prompt_ids)
        if a is None or len(a) < p:
            a = self._all = list(self.prompt_ids)
        k = len(a) - p
        n_out = len(self.output_ids)
        if k != n_out:
            if k > n_out:
                del a[p + n_out:]
            else:
                a.extend(self.output_ids[k:])
        return a

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)

    def set_pending(self, row: int) -> None:
        """Append a sampled token whose value is still on the device (row ``row`` of its step)."""
        self.output_ids.append(PENDING_TOKEN)
        self.pending = len(self.output_ids) - 1
        self.pending_row = row

    def resolve_pending(self, tok: int) -> None:
        """Write the pending token's value here and into the maintained id mirrors."""
        i = self.pending
        if i < 0:
            return
        self.output_ids[i] = tok
        j = len(self.prompt_ids) + i
        if self._all is not None and len(self._all) > j:
            self._all[j] = tok
        if self._np_tok is not None and self._np_tok_n > j:
            self._np_tok[j] = tok
        self.pending = self.pending_row = -1

    def drop_pending(self) -> None:
        """Forget a pending token (the request was aborted while its step ran)."""
        if self.pending < 0:
            return
        del self.output_ids[self.pending:]
        self._np_tok_n = min(self._np_tok_n, len(self.prompt_ids) + len(self.output_ids))
        self.pending = self.pending_row = -1

    @property
    def prefilling(self) -> bool:
        return self.num_computed < len(self.prompt_ids)

    @property
    def finished(self) -> bool:
        return self.status == RequestStatus.FINISHED

    def ttft(self) -> float | None:
        return None if self.first_token_time is None else self.first_token_time - self.arrival_time


@dataclass
class RequestOutput:
    request_id: str
    prompt_ids: list[int]
    output_ids: list[int]
    finish_reason: str | None
    num_cached_tokens: int
    ttft: float | None
    latency: float | None
