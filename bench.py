#!/usr/bin/env python
"""Headline benchmark: multi-aLoRA serving throughput on the Granite-8B shape.

Metric (the headline benchmark): output tok/s + p50 TTFT for the multi-adapter
Granite-8B-shape workload (40 layers, d_model 4096, 32 q / 8 kv heads,
head_dim 128, FFN 12800, vocab 49152, random init; 12 aLoRA adapters of rank 32
on q/k/v/o), with the KV prefix-hit rate. Conversations arrive by a Poisson
process; each holds a 4096-token context followed by 8 chained adapter calls
(16-64-token invocation, 32-128 generated tokens).

``python bench.py --gpus N --steps K --warmup W`` serves the workload with
tensor parallelism over N GPUs (one process per GPU under torchrun). A step is
one engine iteration (one batched forward over every running request). After
an untimed ramp that fills the server to its steady concurrency, W untimed
warm-up steps run, then exactly K steps are timed with CUDA events bracketed
by a barrier and a device synchronise; the reported time is the max over
ranks. ``value`` is whole-job generated tokens per second over the timed
steps. ``e2e`` is the same metric measured by the host clock around the same
K steps of the public engine API, whose every step copies its inputs from
pinned host memory and reads the sampled ids back.

The engine admits requests under its default ``cache_affinity`` policy:
a call whose context is already in the prefix cache (a conversation's next
call) is admitted before new conversations, and a cold request waits at most
``--max-wait-steps`` engine steps; ``--scheduling-policy fcfs`` admits in
arrival order, as the reference's vLLM engine does. The line reports p50 / p90
TTFT over every request that arrived since the ramp began, queue wait
included (a request still waiting at the end counts at its wait so far), the
p50 of conversations' first calls, the window's token mix (prefill tokens and
decode rows per step, fraction of cold admissions) and the count of device
errors (steps whose kernels reported a bounded wait that ran out or a bad
index); the run exits non-zero if there was any.

``--impl reference`` runs the unmodified reference (granite-switch's vLLM
plugin from baseline/_ref) on the same workload and prints the same line.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))

DEFAULT_MAX_WAIT_STEPS = 2000  # the engine's default (engine.llm_engine.DEFAULT_MAX_WAIT_STEPS)
METRIC = "output tok/s + p50 TTFT, multi-aLoRA 8B-shape, TP1/2/4/8; KV prefix-hit rate"
BASELINE_VALUE = None  # the reference publishes no number for this workload on any B200


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=120)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["native", "reference"], default="native")
    p.add_argument("--preset", default="granite-8b")
    p.add_argument("--layers", type=int, default=None, help="override layer count (debug only; invalid for the metric)")
    p.add_argument("--rate", type=float, default=16.0, help="conversation arrivals per second (Poisson)")
    p.add_argument("--conversations", type=int, default=2048)
    p.add_argument("--context-len", type=int, default=4096)
    p.add_argument("--calls", type=int, default=8)
    p.add_argument("--max-num-seqs", type=int, default=128)
    p.add_argument("--max-num-batched-tokens", type=int, default=8192)
    p.add_argument("--ramp-steps", type=int, default=400, help="max untimed steps to reach steady concurrency")
    p.add_argument("--mode", choices=["alora", "lora"], default="alora")
    p.add_argument("--no-fused-comm", dest="fused_comm", action="store_false",
                   help="use NCCL all-reduce instead of the fused GEMM+multimem collectives for TP")
    p.add_argument("--scheduling-policy", choices=["cache_affinity", "fcfs"], default="cache_affinity",
                   help="engine admission order (the reference arm's vLLM engine is FCFS)")
    p.add_argument("--max-wait-steps", type=int, default=DEFAULT_MAX_WAIT_STEPS,
                   help="cache_affinity: engine steps after which a waiting cold request goes first (negative: none)")
    p.add_argument("--kv-cache-dtype", choices=["bfloat16", "fp8_e4m3"], default="bfloat16",
                   help="KV cache storage; the headline metric is defined on the bf16 cache")
    p.add_argument("--pp", type=int, default=1,
                   help="pipeline stages (the GPUs are split into pp stages of gpus / pp tensor-parallel ranks)")
    p.add_argument("--no-pp-microbatches", dest="pp_microbatches", action="store_false",
                   help="pipeline parallelism: run each step whole instead of as two micro-batches")
    p.add_argument("--no-async", dest="async_scheduling", action="store_false",
                   help="blocking engine steps (read each step's ids before scheduling the next)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kv-blocks", type=int, default=None)
    return p.parse_args()


def _pct(xs, q):
    s = sorted(xs)
    return s[min(len(s) - 1, int(q * len(s)))]


def emit(obj):
    print(json.dumps(obj), flush=True)


# ----------------------------------------------------------------------------- config
def model_config(args):
    sys.path.insert(0, ROOT)
    from granite_switch_b200.composer.synthetic import base_config
    from granite_switch_b200.config import GraniteSwitchConfig

    base = base_config(args.preset)
    if args.layers:
        base["num_hidden_layers"] = args.layers
    na = 12
    v = base["vocab_size"]
    cfg = dict(base)
    cfg.update(num_adapters=na, adapter_token_ids=list(range(v, v + na)),
               adapter_substitute_token_ids=[1] * na, adapter_names=[f"adapter_{i}" for i in range(na)],
               adapter_ranks=[32] * na, max_lora_rank=32, lora_target_modules=["qkv_proj", "o_proj"],
               num_hidden_layers=base["num_hidden_layers"] + 2, vocab_size=v + na)
    return GraniteSwitchConfig(**cfg), base


# ----------------------------------------------------------------------------- native arm
def run_native(args):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from granite_switch_b200 import _native
    from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams
    from granite_switch_b200.utils.timing import ClockSampler, local_rank, max_over_ranks
    from granite_switch_b200.utils.workload import WorkloadConfig, advance, call_prompt, make_workload

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank())
    group = None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank()))
        group = dist.group.WORLD
        # host-side agreement (arrivals) over gloo: a broadcast on the GPU stream plus a host
        # read would wait for the step just launched and serialise the pipelined steps
        cpu_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
    if world % args.pp:
        raise SystemExit(f"--pp {args.pp} does not divide {world} GPUs")
    tp = world // args.pp
    tp_rank, tp_group, pipe = rank, group, None
    if args.pp > 1:
        from granite_switch_b200.parallel.pipeline import init_parallel_groups

        tp_rank, tp_group, pipe = init_parallel_groups(tp, args.pp)
    _native.native()
    config, base = model_config(args)
    ecfg = EngineConfig(max_num_seqs=args.max_num_seqs, max_num_batched_tokens=args.max_num_batched_tokens,
                        max_model_len=args.context_len + args.calls * 200 + 256, tensor_parallel_size=tp,
                        pipeline_parallel_size=args.pp, pipeline_microbatches=args.pp_microbatches,
                        num_kv_blocks=args.kv_blocks, fused_tp_comm=args.fused_comm, seed=args.seed,
                        scheduling_policy=args.scheduling_policy,
                        max_wait_steps=args.max_wait_steps if args.max_wait_steps >= 0 else None,
                        kv_cache_dtype=args.kv_cache_dtype, async_scheduling=args.async_scheduling)
    llm = LLM(config, device=f"cuda:{local_rank()}", engine_config=ecfg,
              random_init=dict(lora_modules=("qkv", "o"), rank=32, seed=args.seed), tp_rank=tp_rank, tp_group=tp_group,
              pipeline=pipe)
    eng = llm.engine
    wl = WorkloadConfig(num_conversations=args.conversations, rate=args.rate, context_len=args.context_len,
                        calls=args.calls, vocab=base["vocab_size"], num_adapters=12, seed=args.seed, mode=args.mode)
    convs = make_workload(wl)
    ctrl = config.adapter_token_ids
    by_req = {}
    first_calls = set()  # request ids of conversations' first calls (cold contexts)

    submitted = []  # every request, for TTFT over all arrivals (queue wait included)

    def submit(conv, now):
        prompt = call_prompt(conv, ctrl, args.mode)
        gen = conv.calls[conv.next_call].gen_len
        r = eng.add_request(prompt, SamplingParams(max_tokens=gen, ignore_eos=True), arrival_time=now)
        submitted.append(r)
        by_req[r.request_id] = conv
        if conv.next_call == 0:
            first_calls.add(r.request_id)

    def on_finish(req):
        conv = by_req.pop(req.request_id)
        if advance(conv, req.prompt_ids, req.output_ids, args.mode):
            submit(conv, time.perf_counter())

    eng.on_finish = on_finish
    t0 = time.perf_counter()
    t_start = t0
    next_conv = 0
    arrived = torch.zeros(1, dtype=torch.long)

    def admit():
        nonlocal next_conv
        now = time.perf_counter() - t0
        if (rank == 0 and not eng.has_unfinished() and next_conv < len(convs)
                and convs[next_conv].arrival > now):
            time.sleep(convs[next_conv].arrival - now)  # idle server: wait for the next arrival
            now = time.perf_counter() - t0
        n = next_conv
        while n < len(convs) and convs[n].arrival <= now:
            n += 1
        if world > 1:
            arrived.fill_(n)
            dist.broadcast(arrived, src=0, group=cpu_group)
            n = int(arrived.item())
        while next_conv < n:
            submit(convs[next_conv], time.perf_counter())
            next_conv += 1

    finished_log = []
    eng_step = eng.step

    def step():
        admit()
        try:
            fin = eng_step()
        except _native.DeviceError as e:  # the engine aborted that step's requests; counted below
            print(f"rank {rank}: {e}", file=sys.stderr, flush=True)
            fin = []
        finished_log.extend(fin)
        return fin

    # ---- ramp: fill the server to steady concurrency
    ramp = 0
    target = int(0.9 * args.max_num_seqs)
    while ramp < args.ramp_steps:
        step()
        ramp += 1
        decoding = sum(1 for r in eng.scheduler.running if r.first_token_time is not None)
        if decoding >= target:
            break
    # ---- warm-up
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(group=group)
    gen0 = eng.stats.generated_tokens
    q0, h0 = eng.blocks.queries, eng.blocks.hits
    pf0, dr0 = eng.stats.prefill_tokens, eng.stats.decode_rows
    adm0, cold0 = eng.scheduler.num_admitted, eng.scheduler.num_admitted_cold
    ex = eng.executor
    h2d0, d2h0 = ex.h2d_bytes, ex.d2h_bytes
    host0 = (eng.stats.host_schedule_s, ex.host_stage_s, ex.host_enqueue_s, ex.host_wait_s, eng.stats.host_post_s)
    launches0 = _native.launch_count()
    start_ev, end_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank()) as clocks:
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        start_ev.record()
        for _ in range(args.steps):
            step()
        end_ev.record()
        torch.cuda.synchronize()
        w1 = time.perf_counter()
    if world > 1:
        dist.barrier(group=group)
    dev_ms = max_over_ranks(start_ev.elapsed_time(end_ev), group)
    wall_s = max_over_ranks(w1 - w0, group)
    gen = eng.stats.generated_tokens - gen0
    launches = _native.launch_count() - launches0
    host1 = (eng.stats.host_schedule_s, ex.host_stage_s, ex.host_enqueue_s, ex.host_wait_s, eng.stats.host_post_s)
    host_ms = {k: round((b - a) * 1e3 / args.steps, 3)
               for k, a, b in zip(("schedule", "stage", "enqueue", "wait_for_gpu", "post"), host0, host1)}
    ttft = ttft_summary(submitted, first_calls, t_start, w0, w1)
    dq, dh = eng.blocks.queries - q0, eng.blocks.hits - h0
    adm, cold = eng.scheduler.num_admitted - adm0, eng.scheduler.num_admitted_cold - cold0
    device_errors = eng.stats.device_errors + _native.read_errors(torch.device("cuda", local_rank()))
    value = gen / (dev_ms / 1e3)
    e2e = gen / wall_s
    clk = clocks.summary()
    if rank == 0:
        emit({
            "metric": METRIC, "value": round(value, 2), "unit": "output tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": (round(value / BASELINE_VALUE, 4) if BASELINE_VALUE else None),
            "dtype": "bf16", "data": "synthetic (random prompts, random-init base and adapter weights)",
            "impl": "native",
            **ttft,
            "prefix_hit_rate": round(dh / dq, 4) if dq else None,
            "prefix_hit_rate_overall": round(eng.prefix_cache_hit_rate(), 4),
            "config": {"model": f"{args.preset}-shape" + (f"-L{args.layers}" if args.layers else ""),
                       "global_batch": args.max_num_seqs, "seq_len": args.context_len,
                       "parallelism": f"tp{tp}" + (f"pp{args.pp}" + ("" if args.pp_microbatches else " (whole steps)")
                                                    if args.pp > 1 else ""),
                       "adapters": "12 aLoRA r32 q/k/v/o",
                       "workload": f"poisson {args.rate}/s, {args.calls} chained calls, inv 16-64, gen 32-128",
                       "mode": args.mode, "max_num_batched_tokens": args.max_num_batched_tokens,
                       "scheduling_policy": args.scheduling_policy, "max_wait_steps": ecfg.max_wait_steps,
                       "kv_cache_dtype": args.kv_cache_dtype, "async_scheduling": eng.async_steps,
                       "ramp_steps": ramp, "l2": "inputs larger than L2 (each step streams all weights)",
                       "fused_comm": bool(getattr(llm.model, "comm", None) is not None)},
            "e2e": {"value": round(e2e, 2), "unit": "output tok/s", "h2d_bytes_per_step": (ex.h2d_bytes - h2d0) // args.steps,
                    "d2h_bytes_per_step": (ex.d2h_bytes - d2h0) // args.steps},
            "gpu_launches": launches,
            "clocks": clk,
            "kv_blocks": eng.blocks.num_blocks,
            "running_at_end": len(eng.scheduler.running),
            "window_mix": {"prefill_tokens_per_step": round((eng.stats.prefill_tokens - pf0) / args.steps, 1),
                           "decode_rows_per_step": round((eng.stats.decode_rows - dr0) / args.steps, 1),
                           "admitted": adm, "cold_admission_fraction": round(cold / adm, 4) if adm else None},
            "device_errors": device_errors,
            # rank 0's host time per step by phase (wall clock): the GPU has no queued work
            # during schedule, stage and post
            "host_ms_per_step": host_ms,
        })
    if world > 1:
        dist.barrier(group=group)
        dist.destroy_process_group()
    if device_errors:
        raise SystemExit(f"{device_errors} device error(s) during the run")


def ttft_summary(reqs, first_calls, t_start, w0, w1) -> dict:
    """TTFT over every request that arrived from the start of the ramp to the end of the
    timed window, queue wait included: a request with no first token by ``w1`` counts at
    its wait so far (``waiting_at_end`` of them). Also the p50 of conversations' first calls
    and, for comparison with window-only figures, TTFTs of first tokens inside [w0, w1]."""
    all_t, first_t, win = [], [], []
    waiting = 0
    for r in reqs:
        if r.arrival_time < t_start or r.arrival_time > w1:
            continue
        ft = r.first_token_time
        if ft is not None and ft <= w1:
            t = ft - r.arrival_time
            if ft >= w0:
                win.append(t)
        else:
            t = w1 - r.arrival_time
            waiting += 1
        all_t.append(t)
        if r.request_id in first_calls:
            first_t.append(t)

    def p(xs, q):
        return round(_pct(xs, q), 4) if xs else None

    return {"p50_ttft_s": p(all_t, 0.5), "p90_ttft_s": p(all_t, 0.9), "ttft_samples": len(all_t),
            "ttft_waiting_at_end": waiting, "ttft_scope": "every request arrived since the ramp began; "
            "requests without a first token count at their wait so far",
            "first_call_p50_ttft_s": p(first_t, 0.5), "first_call_ttft_samples": len(first_t),
            "window_p50_ttft_s": p(win, 0.5), "window_ttft_samples": len(win)}


# ----------------------------------------------------------------------------- reference arm
def find_reference() -> tuple[str | None, list[str]]:
    """Locate the installed reference package: the ``pip --target baseline/_ref`` layout
    (``baseline/_ref/granite_switch``), a source tree (``baseline/_ref/src/granite_switch``)
    or an installed distribution. Returns ``(directory to put on sys.path, paths checked)``."""
    import importlib.util

    ref = os.path.join(ROOT, "baseline", "_ref")
    checked = []
    for root in (ref, os.path.join(ref, "src")):
        pkg = os.path.join(root, "granite_switch", "__init__.py")
        checked.append(pkg)
        if os.path.isfile(pkg):
            return root, checked
    checked.append("importlib: granite_switch")
    spec = importlib.util.find_spec("granite_switch")
    if spec is not None and spec.origin:
        return os.path.dirname(os.path.dirname(spec.origin)), checked
    return None, checked


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    where, checked = find_reference()
    if where is None:
        if rank == 0:
            emit({"impl": "reference", "unavailable": "the reference package is not installed; checked: "
                  + ", ".join(checked)})
        return
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    from reference_arm import run as ref_run  # baseline/reference_arm.py

    ref_run(args, emit, METRIC, where)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
