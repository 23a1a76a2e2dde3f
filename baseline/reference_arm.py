"""Reference arm of bench.py: the unmodified granite-switch vLLM plugin on the same workload.

Runs granite-switch (installed in baseline/_ref) through its own public entry
point, vLLM's engine with the granite-switch plugin, on a composed checkpoint of
the Granite-8B benchmark shape with random weights (written once to /tmp).
Only rank 0 drives vLLM (which starts its own tensor-parallel workers); the
other torchrun ranks wait. Prints the same JSON line as the native arm with
``"impl": "reference"``, or ``{"impl": "reference", "unavailable": ...}``.
"""
from __future__ import annotations

import os
import sys
import time
import traceback

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")
_TORCHRUN_VARS = ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK",
                  "ROLE_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT", "TORCHELASTIC_RUN_ID", "GROUP_WORLD_SIZE",
                  "TORCHELASTIC_RESTART_COUNT", "TORCHELASTIC_MAX_RESTARTS", "TORCH_NCCL_ASYNC_ERROR_HANDLING")


def _wait_for_rank0(flag):
    t0 = time.time()
    while not os.path.exists(flag) and time.time() - t0 < 3600:
        time.sleep(2)


def run(args, emit, metric, ref_path=REF):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    flag = f"/tmp/gs_ref_done_{os.environ.get('MASTER_PORT', 'x')}"
    if rank != 0:
        _wait_for_rank0(flag)
        return
    try:
        _run(args, emit, metric, world, ref_path)
    except Exception as e:  # the line must still be printed
        tb = traceback.format_exc().strip().splitlines()
        emit({"impl": "reference", "unavailable": f"{type(e).__name__}: {str(e)[:300]}",
              "where": tb[-3:] if tb else None})
    finally:
        with open(flag, "w") as f:
            f.write("done")


def _run(args, emit, metric, world, ref_path):
    for k in _TORCHRUN_VARS:
        os.environ.pop(k, None)
    os.environ["PYTHONPATH"] = ref_path + os.pathsep + os.environ.get("PYTHONPATH", "")
    sys.path.insert(0, ref_path)
    sys.path.insert(0, ROOT)
    import torch

    import bench
    from granite_switch_b200.composer.synthetic import write_random_checkpoint
    from granite_switch_b200.utils.workload import WorkloadConfig, advance, call_prompt, make_workload

    config, base = bench.model_config(args)
    ckpt = f"/tmp/gs_ref_ckpt_{args.preset}_L{config.num_decoder_layers}"
    if not os.path.exists(os.path.join(ckpt, "config.json")):
        write_random_checkpoint(ckpt, config, device="cuda:0", seed=args.seed)
        torch.cuda.empty_cache()
    import granite_switch  # noqa: F401  (the reference package)
    from granite_switch.vllm import register

    register()
    from vllm import LLM, SamplingParams

    llm = LLM(model=ckpt, skip_tokenizer_init=True, tensor_parallel_size=world, enable_prefix_caching=True,
              max_num_seqs=args.max_num_seqs, max_num_batched_tokens=args.max_num_batched_tokens,
              max_model_len=args.context_len + args.calls * 200 + 256, dtype="bfloat16",
              gpu_memory_utilization=0.88, seed=args.seed,
              kv_cache_dtype="auto" if getattr(args, "kv_cache_dtype", "bfloat16") == "bfloat16" else "fp8_e4m3")
    engine = llm.llm_engine
    wl = WorkloadConfig(num_conversations=args.conversations, rate=args.rate, context_len=args.context_len,
                        calls=args.calls, vocab=base["vocab_size"], num_adapters=12, seed=args.seed, mode=args.mode)
    convs = make_workload(wl)
    ctrl = config.adapter_token_ids
    live = {}
    stats = {"gen": 0, "prompt": 0, "cached": 0}
    seen = {}
    first_tok = {}
    first_calls = set()
    counter = [0]

    from types import SimpleNamespace

    submitted = {}  # rid -> record with arrival / first-token times (bench.ttft_summary)

    def submit(conv, now):
        prompt = call_prompt(conv, ctrl, args.mode)
        rid = f"r{counter[0]}"
        counter[0] += 1
        submitted[rid] = SimpleNamespace(request_id=rid, arrival_time=now, first_token_time=None)
        sp = SamplingParams(max_tokens=conv.calls[conv.next_call].gen_len, temperature=0.0, ignore_eos=True)
        engine.add_request(rid, {"prompt_token_ids": prompt}, sp)
        live[rid] = (conv, prompt, now)
        if conv.next_call == 0:
            first_calls.add(rid)

    t0 = time.perf_counter()
    t_start = t0
    nxt = [0]

    def step():
        now = time.perf_counter() - t0
        if not engine.has_unfinished_requests() and nxt[0] < len(convs) and convs[nxt[0]].arrival > now:
            time.sleep(convs[nxt[0]].arrival - now)
            now = time.perf_counter() - t0
        while nxt[0] < len(convs) and convs[nxt[0]].arrival <= now:
            submit(convs[nxt[0]], time.perf_counter())
            nxt[0] += 1
        outs = engine.step()
        tnow = time.perf_counter()
        for o in outs:
            if o.request_id not in live:
                continue
            conv, prompt, sub = live[o.request_id]
            toks = list(o.outputs[0].token_ids) if o.outputs else []
            stats["gen"] += max(0, len(toks) - seen.get(o.request_id, 0))
            seen[o.request_id] = len(toks)
            if toks and o.request_id not in first_tok:
                first_tok[o.request_id] = tnow
                submitted[o.request_id].first_token_time = tnow
            if o.finished:
                seen.pop(o.request_id, None)
                stats["prompt"] += len(prompt)
                stats["cached"] += int(getattr(o, "num_cached_tokens", 0) or 0)
                del live[o.request_id]
                if advance(conv, prompt, toks, args.mode):
                    submit(conv, tnow)
        return outs

    ramp = 0
    target = int(0.9 * args.max_num_seqs)
    while ramp < args.ramp_steps:
        step()
        ramp += 1
        decoding = sum(1 for rid in live if rid in first_tok)
        if decoding >= target:
            break
    for _ in range(args.warmup):
        step()
    tok_before = stats["gen"]
    p0, c0 = stats["prompt"], stats["cached"]
    w0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    w1 = time.perf_counter()
    tok_after = stats["gen"]
    gen = tok_after - tok_before
    ttft = bench.ttft_summary(list(submitted.values()), first_calls, t_start, w0, w1)
    dp, dc = stats["prompt"] - p0, stats["cached"] - c0
    hit = None
    try:  # vLLM's own prefix-cache counters, when this version exposes them
        for mt in llm.get_metrics():
            if mt.name in ("vllm:prefix_cache_hits", "vllm:prefix_cache_queries"):
                hit = hit or {}
                hit[mt.name] = getattr(mt, "value", None)
    except Exception:
        pass
    emit({"metric": metric, "value": round(gen / (w1 - w0), 2), "unit": "output tok/s", "n_gpus": world,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round((w1 - w0) * 1e3 / args.steps, 3),
          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
          "data": "synthetic (random prompts, random-init base and adapter weights)", "impl": "reference",
          "timing": "host clock (vLLM runs the model in its own engine process)",
          **ttft,
          "prefix_hit_rate": round(dc / dp, 4) if dp else None, "vllm_prefix_cache_counters": hit,
          "config": {"model": f"{args.preset}-shape", "global_batch": args.max_num_seqs, "seq_len": args.context_len,
                     "parallelism": f"tp{world}", "adapters": "12 aLoRA r32 q/k/v/o",
                     "workload": f"poisson {args.rate}/s, {args.calls} chained calls, inv 16-64, gen 32-128",
                     "mode": args.mode, "scheduling_policy": "fcfs (vLLM default)", "ramp_steps": ramp,
                     "kv_cache_dtype": getattr(args, "kv_cache_dtype", "bfloat16"),
                     "vllm": _vllm_version()}})


def _vllm_version():
    try:
        import vllm

        return vllm.__version__
    except Exception:
        return None
