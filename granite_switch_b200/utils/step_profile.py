"""Per-op device time of one representative engine step (CUDA events, no profiler).

``python -m granite_switch_b200.utils.step_profile [--preset granite-8b] [--prefill 4096 4096]
[--prefill-ctx 0] [--decode 120 --decode-ctx 4400]``; under torchrun (one process per GPU) it
runs the tensor-parallel model, with the fused NVSwitch collectives unless
``--no-fused-comm``.

The step is built the way the serving engine builds one: prefill chunks (a
fresh prompt, or a chunk after a cached prefix) next to single-token decode
rows, flattened into one batch, KV pages from the block manager. After
warm-up steps, each op of the forward is bracketed by CUDA events (one pair
per launch group) over ``--steps`` steps; the table gives the mean device
milliseconds per step for each op summed over layers, and the share of the
event-timed step. ``step_ms`` is the step without the per-op events and
``host_enqueue_ms`` the host time to stage the inputs and enqueue every
launch of the step. Rank 0 prints one JSON line; with several ranks every op
is the max over ranks.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
from collections import defaultdict

import torch


class StepProfiler:
    """Collects (name, start event, end event) for regions of the forward."""

    def __init__(self):
        self.events = []

    @contextlib.contextmanager
    def region(self, name: str):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        try:
            yield
        finally:
            b.record()
            self.events.append((name, a, b))

    def totals(self) -> dict[str, float]:
        torch.cuda.synchronize()
        out = defaultdict(float)
        for name, a, b in self.events:
            out[name] += a.elapsed_time(b)
        self.events = []
        return dict(out)


def build_step(engine, prefill: list[int], decode: int, decode_ctx: int, vocab: int, seed: int = 0,
               prefill_ctx: int = 0):
    """Scheduler output with ``prefill`` chunks (each after ``prefill_ctx`` cached tokens)
    and ``decode`` single-token rows."""
    from ..engine.request import Request, SamplingParams
    from ..engine.scheduler import ScheduledChunk, SchedulerOutput

    g = torch.Generator().manual_seed(seed)
    bm = engine.blocks
    out = SchedulerOutput()
    for n in prefill:
        r = Request(torch.randint(0, vocab, (prefill_ctx + n,), generator=g).tolist(), SamplingParams(max_tokens=8))
        assert bm.allocate(r, prefill_ctx + n)
        r.num_computed = prefill_ctx
        out.chunks.append(ScheduledChunk(r, prefill_ctx, n))
    for _ in range(decode):
        r = Request(torch.randint(0, vocab, (decode_ctx,), generator=g).tolist(), SamplingParams(max_tokens=8))
        r.output_ids.append(1)
        assert bm.allocate(r, decode_ctx + 1)
        r.num_computed = decode_ctx
        out.chunks.append(ScheduledChunk(r, decode_ctx, 1))
    return out


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--preset", default="granite-8b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--prefill", type=int, nargs="*", default=[4096, 3968])
    p.add_argument("--decode", type=int, default=128)
    p.add_argument("--decode-ctx", type=int, default=4400)
    p.add_argument("--prefill-ctx", type=int, default=0, help="cached tokens before each prefill chunk")
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--no-fused-comm", dest="fused", action="store_false")
    p.add_argument("--lora", nargs="*", default=["qkv", "o"], help="projections with adapters")
    p.add_argument("--kv-cache-dtype", choices=["bfloat16", "fp8_e4m3"], default="bfloat16")
    p.add_argument("--prefill-split-ctas", type=int, default=None,
                   help="CTAs a split prefill grid aims at (A/B of ops.attention.PREFILL_SPLIT_CTAS)")
    p.add_argument("--prefill-min-keys", type=int, default=None,
                   help="fewest keys per prefill split (A/B of ops.attention.PREFILL_MIN_KEYS_PER_SPLIT)")
    p.add_argument("--no-attn-overlap", dest="attn_overlap", action="store_false",
                   help="run a mixed step's prefill attention after its decode attention, on one stream")
    p.add_argument("--small-shrink-max-m", type=int, default=None,
                   help="largest token count whose LoRA shrink runs on CUDA cores (A/B of ops.gemm.SMALL_SHRINK_MAX_M)")
    p.add_argument("--decode-split-ctas", type=int, default=None,
                   help="CTAs a split decode grid aims at (A/B of ops.attention.DECODE_SPLIT_CTAS)")
    p.add_argument("--attn-decode-stages", type=int, default=None, choices=[2, 3],
                   help="decode attention layout: 2 = short rings, three CTAs per SM; 3 = deep rings, two")
    p.add_argument("--fp8-decode-rows", type=int, default=8, choices=[8, 16],
                   help="decode tile rows over an fp8 cache: 8 (keys on the MMA's row side) or 16 (row-major)")
    p.add_argument("--attn-fp8t-stages", type=int, default=None, choices=[2, 3],
                   help="stages of the fp8 decode kernel with 8-row tiles (3: four CTAs per SM, 2: five)")
    p.add_argument("--no-pdl", dest="pdl", action="store_false",
                   help="launch the GEMMs in plain stream order (not as programmatic dependents)")
    args = p.parse_args()

    import torch.distributed as dist

    from .. import _native
    from ..engine import LLM, EngineConfig
    from .timing import local_rank

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(local_rank())
    group = None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank()))
        group = dist.group.WORLD
    _native.native()
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench

    bargs = argparse.Namespace(preset=args.preset, layers=args.layers)
    config, base = bench.model_config(bargs)
    tokens = sum(args.prefill) + args.decode
    need_blocks = (sum((args.prefill_ctx + n + 15) // 16 for n in args.prefill)
                   + args.decode * ((args.decode_ctx + 16) // 16) + 64)
    ecfg = EngineConfig(max_num_seqs=max(8, len(args.prefill) + args.decode), max_num_batched_tokens=tokens,
                        max_model_len=max([args.prefill_ctx + n for n in args.prefill] + [args.decode_ctx + 1]) + 16,
                        tensor_parallel_size=world,
                        num_kv_blocks=need_blocks, fused_tp_comm=args.fused, kv_cache_dtype=args.kv_cache_dtype)
    ecfg.programmatic_launch = args.pdl
    ecfg.overlap_attention = args.attn_overlap
    from ..ops import attention as A

    from ..ops import gemm as G

    if args.small_shrink_max_m is not None:
        G.SMALL_SHRINK_MAX_M = args.small_shrink_max_m
    if args.attn_fp8t_stages:
        _native.native().attn_fp8t_stages(args.attn_fp8t_stages)
    if args.attn_decode_stages:
        _native.native().attn_decode_stages(args.attn_decode_stages)
    if args.decode_split_ctas:
        A.DECODE_SPLIT_CTAS = args.decode_split_ctas
    if args.prefill_split_ctas:
        A.PREFILL_SPLIT_CTAS = args.prefill_split_ctas
    if args.prefill_min_keys:
        A.PREFILL_MIN_KEYS_PER_SPLIT = args.prefill_min_keys
    llm = LLM(config, device=f"cuda:{local_rank()}", engine_config=ecfg,
              random_init=dict(lora_modules=tuple(args.lora), rank=32), tp_rank=rank, tp_group=group)
    eng = llm.engine
    llm.model.fp8_decode_rows = args.fp8_decode_rows
    out = build_step(eng, args.prefill, args.decode, args.decode_ctx, base["vocab_size"], prefill_ctx=args.prefill_ctx)
    ex = eng.executor
    model = llm.model
    for _ in range(args.warmup):
        ex.compute_logits(out)
    torch.cuda.synchronize()
    # host time to enqueue one step (no profiler regions): staging + every launch
    import time

    host_ms = 0.0
    for _ in range(args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ex.compute_logits(out)
        host_ms += (time.perf_counter() - t0) * 1e3
    host_ms /= args.steps
    torch.cuda.synchronize()
    plain = 0.0
    for _ in range(args.steps):
        if group is not None:
            dist.barrier(group=group)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ex.compute_logits(out)
        b.record()
        b.synchronize()
        plain += a.elapsed_time(b)
    plain /= args.steps
    prof = StepProfiler()
    sums = defaultdict(float)
    step_ms = 0.0
    for _ in range(args.steps):
        if group is not None:
            dist.barrier(group=group)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        model.prof = prof
        a.record()
        ex.compute_logits(out)
        b.record()
        model.prof = None
        for k, v in prof.totals().items():
            sums[k] += v
        step_ms += a.elapsed_time(b)
    ops = {k: v / args.steps for k, v in sums.items()}
    step_ms /= args.steps
    if group is not None:
        names = sorted(ops)
        t = torch.tensor([ops[n] for n in names] + [step_ms, plain, host_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        ops = dict(zip(names, t[:-3].tolist()))
        step_ms, plain, host_ms = float(t[-3]), float(t[-2]), float(t[-1])
    if rank == 0:
        table = {k: dict(ms=round(v, 3), share=round(v / step_ms, 3)) for k, v in sorted(ops.items(), key=lambda kv: -kv[1])}
        print(json.dumps(dict(preset=args.preset, tp=world, fused_comm=bool(getattr(model, "comm", None)),
                              tokens=tokens, prefill=args.prefill, prefill_ctx=args.prefill_ctx,
                              decode=args.decode, decode_ctx=args.decode_ctx, pdl=args.pdl,
                              attn_overlap=args.attn_overlap, prefill_split_ctas=A.PREFILL_SPLIT_CTAS,
                              prefill_min_keys=A.PREFILL_MIN_KEYS_PER_SPLIT, small_shrink_max_m=G.SMALL_SHRINK_MAX_M,
                              decode_split_ctas=A.DECODE_SPLIT_CTAS,
                              attn_decode_stages=_native.native().attn_decode_stages(-1),
                              kv_cache_dtype=args.kv_cache_dtype, fp8_decode_rows=args.fp8_decode_rows,
                              attn_fp8t_stages=_native.native().attn_fp8t_stages(-1),
                              step_ms=round(plain, 3), step_ms_with_regions=round(step_ms, 3),
                              host_enqueue_ms=round(host_ms, 3), ops=table)), flush=True)
    if group is not None:
        dist.barrier(group=group)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
