"""Offline batch benchmark on one GPU: the Granite-3B-shape aLoRA batch of the benchmark configs.

``python -m granite_switch_b200.utils.offline_bench [--impl native|reference] [--requests 256]``

Model: 40 layers, d_model 2048, 32 query / 8 KV heads, head_dim 64, SwiGLU
FFN 8192, vocab 49152, random init N(0, 0.02); twelve aLoRA adapters of rank
32 on q/k/v. Batch: ``--requests`` prompts of ``--prompt-len`` random tokens
whose last tokens are a uniformly chosen adapter's invocation (its control
token followed by ``--inv-len - 1`` invocation tokens), each generating
``--gen-len`` tokens (greedy, EOS ignored). All requests are submitted at once
and the engine runs until every one finishes.

Prints one JSON line: generated tokens per second over the whole batch (host
clock around ``generate``, inputs copied from pinned memory and sampled ids
read back every step), total (prompt + generated) tokens per second, and the
device-timed share (CUDA events around the same loop). ``--impl reference``
runs the unmodified reference (granite-switch's vLLM plugin from
baseline/_ref) on a composed random checkpoint of the same shape.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def model_config(layers: int | None = None):
    sys.path.insert(0, ROOT)
    from ..composer.synthetic import base_config
    from ..config import GraniteSwitchConfig

    base = base_config("granite-3b")
    if layers:
        base["num_hidden_layers"] = layers
    na = 12
    v = base["vocab_size"]
    cfg = dict(base)
    cfg.update(num_adapters=na, adapter_token_ids=list(range(v, v + na)), adapter_substitute_token_ids=[1] * na,
               adapter_names=[f"adapter_{i}" for i in range(na)], adapter_ranks=[32] * na, max_lora_rank=32,
               lora_target_modules=["qkv_proj"], num_hidden_layers=base["num_hidden_layers"] + 2,
               vocab_size=v + na)
    return GraniteSwitchConfig(**cfg), base


def make_prompts(n: int, prompt_len: int, inv_len: int, vocab: int, ctrl: list[int], seed: int = 0):
    rng = random.Random(seed)
    prompts = []
    for _ in range(n):
        a = rng.randrange(len(ctrl))
        body = [rng.randrange(1, vocab) for _ in range(prompt_len - inv_len)]
        inv = [ctrl[a]] + [rng.randrange(1, vocab) for _ in range(inv_len - 1)]
        prompts.append(body + inv)
    return prompts


def run_native(args):
    import torch

    from .. import _native
    from ..engine import LLM, EngineConfig, SamplingParams

    _native.native()
    config, base = model_config(args.layers)
    prompts = make_prompts(args.requests, args.prompt_len, args.inv_len, base["vocab_size"],
                           config.adapter_token_ids, args.seed)
    ecfg = EngineConfig(max_num_seqs=args.max_num_seqs, max_num_batched_tokens=args.max_num_batched_tokens,
                        max_model_len=args.prompt_len + args.gen_len + 16, use_cuda_graphs=args.cuda_graphs)
    llm = LLM(config, device="cuda:0", engine_config=ecfg, random_init=dict(lora_modules=("qkv",), rank=32))
    sp = SamplingParams(max_tokens=args.gen_len, ignore_eos=True)
    # warm-up: a small batch through the same engine (kernels configured, allocator warm)
    llm.generate(prompts[: min(8, len(prompts))], SamplingParams(max_tokens=4, ignore_eos=True))
    llm.engine.blocks.reset_prefix_cache()
    torch.cuda.synchronize()
    launches0 = _native.launch_count()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    outs = llm.generate(prompts, sp)
    b.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    dev_s = a.elapsed_time(b) / 1e3
    gen = sum(len(o.output_ids) for o in outs)
    total = gen + sum(len(p) for p in prompts)
    ex = llm.engine.executor
    return dict(impl="native", value=round(gen / wall, 1), unit="generated tok/s", wall_s=round(wall, 3),
                device_s=round(dev_s, 3), total_tok_s=round(total / wall, 1), generated=gen,
                steps=llm.engine.stats.steps, gpu_launches=_native.launch_count() - launches0,
                cuda_graphs=bool(args.cuda_graphs),
                h2d_bytes=ex.h2d_bytes, d2h_bytes=ex.d2h_bytes)


def run_reference(args):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "granite_switch")):
        return dict(impl="reference", unavailable="baseline/_ref is not installed")
    # vLLM inspects model classes in subprocesses: they must find the reference package too
    os.environ["PYTHONPATH"] = ref + os.pathsep + os.environ.get("PYTHONPATH", "")
    sys.path.insert(0, ref)
    import torch

    from ..composer.synthetic import write_random_checkpoint

    config, base = model_config(args.layers)
    ckpt = f"/tmp/gs_ref_ckpt_granite-3b_L{config.num_decoder_layers}_q"
    if not os.path.exists(os.path.join(ckpt, "config.json")):
        write_random_checkpoint(ckpt, config, device="cuda:0", seed=args.seed, lora_groups=("qkv_proj",))
        torch.cuda.empty_cache()
    import granite_switch  # noqa: F401  (the reference package)
    from granite_switch.vllm import register

    register()
    from vllm import LLM, SamplingParams

    prompts = make_prompts(args.requests, args.prompt_len, args.inv_len, base["vocab_size"],
                           config.adapter_token_ids, args.seed)
    llm = LLM(model=ckpt, skip_tokenizer_init=True, enable_prefix_caching=True, max_num_seqs=args.max_num_seqs,
              max_num_batched_tokens=args.max_num_batched_tokens, max_model_len=args.prompt_len + args.gen_len + 16,
              dtype="bfloat16", gpu_memory_utilization=0.88, seed=args.seed)
    sp = SamplingParams(max_tokens=args.gen_len, temperature=0.0, ignore_eos=True)
    llm.generate([{"prompt_token_ids": p} for p in prompts[:8]], SamplingParams(max_tokens=4, ignore_eos=True),
                 use_tqdm=False)
    llm.reset_prefix_cache()
    t0 = time.perf_counter()
    outs = llm.generate([{"prompt_token_ids": p} for p in prompts], sp, use_tqdm=False)
    wall = time.perf_counter() - t0
    gen = sum(len(o.outputs[0].token_ids) for o in outs)
    total = gen + sum(len(p) for p in prompts)
    return dict(impl="reference", value=round(gen / wall, 1), unit="generated tok/s", wall_s=round(wall, 3),
                total_tok_s=round(total / wall, 1), generated=gen, timing="host clock")


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--impl", choices=["native", "reference"], default="native")
    p.add_argument("--requests", type=int, default=256)
    p.add_argument("--prompt-len", type=int, default=2048)
    p.add_argument("--inv-len", type=int, default=4)
    p.add_argument("--gen-len", type=int, default=256)
    p.add_argument("--max-num-seqs", type=int, default=256)
    p.add_argument("--max-num-batched-tokens", type=int, default=8192)
    p.add_argument("--layers", type=int, default=None, help="override layer count (debug only)")
    p.add_argument("--cuda-graphs", action="store_true", help="replay decode-only steps from CUDA graphs")
    p.add_argument("--seed", type=int, default=0)
    args = p.parse_args()
    res = run_reference(args) if args.impl == "reference" else run_native(args)
    res.update(config=dict(model="granite-3b-shape", adapters="12 aLoRA r32 q/k/v", requests=args.requests,
                           prompt_len=args.prompt_len, gen_len=args.gen_len, dtype="bf16",
                           data="synthetic (random prompts, random-init weights)"))
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
