"""Tracing: NVTX ranges per step and per layer region, and a per-step routing trace.

* :class:`NvtxRanges` - a region hook for the native model (``model.prof``):
  every forward region (``qkv``, ``attention``, ``o+reduce``, ...) becomes an
  NVTX range, and the executor wraps each step in one, so an Nsight timeline
  reads layer by layer. Composes with the CUDA-event ``StepProfiler``.
* :class:`RoutingTrace` - after each engine step, the token ids, positions and
  the per-token adapter / LoRA / probe indices the routing kernel wrote are
  copied to the host and kept (optionally appended to a JSONL file). The
  indices are read from the model's static device buffers after the step, so
  the trace also works when the step was replayed from a CUDA graph (the
  reference records the same data only in eager mode:
  src/granite_switch/vllm/switch/multi.py:466-473, hf/modeling_granite_switch.py:679-762).

``GSB_NVTX=1`` and ``GSB_ROUTING_TRACE=<path.jsonl>`` switch them on for
:class:`~granite_switch_b200.engine.LLM`.
"""
from __future__ import annotations

import contextlib
import json

import torch


class NvtxRanges:
    """Region hook pushing an NVTX range per region; ``inner`` (e.g. a StepProfiler) is nested."""

    def __init__(self, inner=None):
        self.inner = inner

    @contextlib.contextmanager
    def region(self, name: str):
        torch.cuda.nvtx.range_push(name)
        try:
            if self.inner is not None:
                with self.inner.region(name):
                    yield
            else:
                yield
        finally:
            torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def nvtx_range(name: str, enabled: bool = True):
    if not enabled:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class RoutingTrace:
    """Per-step routing records: ``{"step", "request_ids", "ids", "positions", "adapter", "lora", "probe"}``."""

    def __init__(self, path: str | None = None, keep: int = 1 << 16):
        self.path = path
        self.keep = keep
        self.records: list[dict] = []
        self.step = 0

    def record(self, request_ids: list[str], ids, positions, adapter, lora, probe=None) -> dict:
        def host(x):
            if x is None:
                return None
            if isinstance(x, torch.Tensor):
                return x.detach().to("cpu").tolist()
            return [int(v) for v in x]

        rec = {"step": self.step, "request_ids": list(request_ids), "ids": host(ids), "positions": host(positions),
               "adapter": host(adapter), "lora": host(lora), "probe": host(probe)}
        self.step += 1
        self.flush()
        self.records.append(rec)
        if len(self.records) > self.keep:
            del self.records[: len(self.records) - self.keep]
        return rec

    def flush(self) -> None:
        """Append the last record (complete once the executor added its spans) to the JSONL file."""
        if self.path and self.records and not self.records[-1].get("_written"):
            rec = self.records[-1]
            rec["_written"] = True
            with open(self.path, "a") as f:
                f.write(json.dumps({k: v for k, v in rec.items() if k != "_written"}) + "\n")

    def of_request(self, request_id: str, field: str = "adapter") -> list[int]:
        """One request's per-token values of ``field`` (``adapter``, ``lora``, ``probe``, ``ids``,
        ``positions``) over the recorded steps, in order (the executor adds each step's ``spans``)."""
        out: list[int] = []
        for r in self.records:
            for rid, (a, b) in zip(r["request_ids"], r.get("spans", [])):
                if rid == request_id:
                    out += r[field][a:b]
        return out


__all__ = ["NvtxRanges", "nvtx_range", "RoutingTrace"]
