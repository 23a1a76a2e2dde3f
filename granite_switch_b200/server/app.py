"""OpenAI-compatible HTTP server over the serving engine.

Endpoints: ``POST /v1/completions`` (text or token-id prompts; token ids are
the form the multi-adapter prefix cache needs), ``POST /v1/chat/completions``
(rendered with the checkpoint's chat template; ``chat_template_kwargs`` such as
``adapter_name`` and ``documents`` select the adapter and its inputs),
``GET /v1/models``, ``GET /health`` and ``GET /metrics`` (Prometheus text with
the vLLM metric names: ``vllm:prefix_cache_queries_total``,
``vllm:prefix_cache_hits_total``, ``vllm:time_to_first_token_seconds``,
``vllm:e2e_request_latency_seconds``, ``vllm:num_requests_running/waiting``).

Run: ``python -m granite_switch_b200.server --model <composed dir> --port 8000``.
"""
from __future__ import annotations

import argparse
import json
import time
import uuid

from ..engine.llm_engine import DEFAULT_MAX_WAIT_STEPS
from ..engine.request import SamplingParams
from .async_engine import AsyncEngine


def _sampling(body: dict, default_max: int = 16) -> SamplingParams:
    stop_ids = tuple(body.get("stop_token_ids") or ())
    return SamplingParams(max_tokens=int(body.get("max_tokens") or default_max),
                          temperature=float(body.get("temperature", 0.0) or 0.0),
                          top_k=int(body.get("top_k", 0) or 0), top_p=float(body.get("top_p", 1.0) or 1.0),
                          seed=body.get("seed"), stop_token_ids=stop_ids,
                          ignore_eos=bool(body.get("ignore_eos", False)),
                          min_tokens=int(body.get("min_tokens", 0) or 0))


def build_app(async_engine: AsyncEngine, tokenizer=None, model_name: str = "granite-switch"):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="granite_switch_b200")

    def encode_prompt(prompt):
        if isinstance(prompt, list) and all(isinstance(t, int) for t in prompt):
            return [list(prompt)]
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], list):
            return [list(p) for p in prompt]
        if tokenizer is None:
            raise HTTPException(400, "this server has no tokenizer: send the prompt as token ids")
        texts = prompt if isinstance(prompt, list) else [prompt]
        return [tokenizer(t, add_special_tokens=False)["input_ids"] for t in texts]

    def decode(ids):
        if tokenizer is None:
            return ""
        return tokenizer.decode(ids, skip_special_tokens=True)

    def usage(reqs):
        p = sum(len(r.prompt_ids) for r in reqs)
        c = sum(len(r.output_ids) for r in reqs)
        cached = sum(r.num_cached_tokens for r in reqs)
        return {"prompt_tokens": p, "completion_tokens": c, "total_tokens": p + c,
                "prompt_tokens_details": {"cached_tokens": cached}}

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "granite_switch_b200"}]}

    @app.get("/metrics")
    async def metrics():
        return PlainTextResponse(async_engine.metrics_text())

    @app.post("/v1/completions")
    async def completions(body: dict):
        prompts = encode_prompt(body.get("prompt"))
        sp = _sampling(body)
        rid = f"cmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        if body.get("stream"):
            if len(prompts) != 1:
                raise HTTPException(400, "streaming supports one prompt")

            async def gen():
                async for item in async_engine.stream(prompts[0], sp):
                    if isinstance(item, list):
                        chunk = {"id": rid, "object": "text_completion", "created": created, "model": model_name,
                                 "choices": [{"index": 0, "text": decode(item), "token_ids": item,
                                              "finish_reason": None}]}
                    else:
                        chunk = {"id": rid, "object": "text_completion", "created": created, "model": model_name,
                                 "choices": [{"index": 0, "text": "", "token_ids": [],
                                              "finish_reason": item.finish_reason}], "usage": usage([item])}
                    yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        try:
            reqs = [await async_engine.generate(p, sp) for p in prompts]
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        choices = [{"index": i, "text": decode(r.output_ids), "token_ids": r.output_ids,
                    "finish_reason": r.finish_reason, "logprobs": None} for i, r in enumerate(reqs)]
        return JSONResponse({"id": rid, "object": "text_completion", "created": created, "model": model_name,
                             "choices": choices, "usage": usage(reqs)})

    @app.post("/v1/chat/completions")
    async def chat(body: dict):
        if tokenizer is None:
            raise HTTPException(400, "chat completions need the checkpoint's tokenizer")
        kwargs = dict(body.get("chat_template_kwargs") or {})
        kwargs.setdefault("add_generation_prompt", bool(body.get("add_generation_prompt", True)))
        text = tokenizer.apply_chat_template(body["messages"], tokenize=False, **kwargs)
        ids = tokenizer(text, add_special_tokens=False)["input_ids"]
        sp = _sampling(body)
        try:
            r = await async_engine.generate(ids, sp)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        out = {
            "id": f"chatcmpl-{uuid.uuid4().hex[:24]}", "object": "chat.completion", "created": int(time.time()),
            "model": model_name,
            "choices": [{"index": 0, "message": {"role": "assistant", "content": decode(r.output_ids)},
                         "finish_reason": r.finish_reason}],
            "usage": usage([r])}
        if body.get("return_token_ids"):
            out["prompt_token_ids"] = list(ids)
            out["choices"][0]["token_ids"] = r.output_ids
        return JSONResponse(out)

    return app


def main(argv=None):
    ap = argparse.ArgumentParser(description="granite_switch_b200 OpenAI-compatible server")
    ap.add_argument("--model", required=True, help="composed Granite Switch checkpoint directory")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--served-model-name", default=None)
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--max-num-batched-tokens", type=int, default=8192)
    ap.add_argument("--max-model-len", type=int, default=8192)
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.88)
    ap.add_argument("--no-prefix-caching", action="store_true")
    ap.add_argument("--device", default=None)
    ap.add_argument("--tensor-parallel-size", type=int, default=1)
    ap.add_argument("--pipeline-parallel-size", type=int, default=1)
    ap.add_argument("--no-fused-tp-comm", action="store_true", help="reduce with NCCL only")
    ap.add_argument("--kv-cache-dtype", choices=["auto", "bfloat16", "fp8", "fp8_e4m3"], default="auto",
                    help="KV cache storage: bf16 (auto) or e4m3 with a per-(token, KV head) scale")
    ap.add_argument("--no-async-scheduling", action="store_true",
                    help="read each step's sampled ids before scheduling the next")
    ap.add_argument("--scheduling-policy", choices=["cache_affinity", "fcfs"], default="cache_affinity",
                    help="admission order: requests whose context is cached first, or arrival order")
    ap.add_argument("--max-wait-steps", type=int, default=DEFAULT_MAX_WAIT_STEPS,
                    help="cache_affinity: engine steps after which a waiting cold request goes first "
                         "(bounds how long a new conversation waits under overload; negative: no bound)")
    args = ap.parse_args(argv)
    import uvicorn

    from ..engine import LLM, EngineConfig

    tp, pp = args.tensor_parallel_size, args.pipeline_parallel_size
    ecfg = EngineConfig(max_num_seqs=args.max_num_seqs, max_num_batched_tokens=args.max_num_batched_tokens,
                        max_model_len=args.max_model_len, gpu_memory_utilization=args.gpu_memory_utilization,
                        enable_prefix_caching=not args.no_prefix_caching, tensor_parallel_size=tp,
                        pipeline_parallel_size=pp, fused_tp_comm=not args.no_fused_tp_comm,
                        scheduling_policy=args.scheduling_policy,
                        max_wait_steps=args.max_wait_steps if args.max_wait_steps >= 0 else None,
                        kv_cache_dtype="fp8_e4m3" if args.kv_cache_dtype.startswith("fp8") else "bfloat16",
                        async_scheduling=not args.no_async_scheduling)
    sync = None
    if tp * pp > 1:
        # one process per GPU (torchrun); rank 0 serves HTTP and drives the others in lock step
        import datetime
        import os

        import torch
        import torch.distributed as dist

        from ..parallel.pipeline import init_parallel_groups
        from .async_engine import StepSync, follow

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        control = dist.new_group(backend="gloo")
        tp_rank, tp_group, pipe = init_parallel_groups(tp, pp)
        llm = LLM(args.model, device=f"cuda:{local}", engine_config=ecfg, tp_rank=tp_rank, tp_group=tp_group,
                  pipeline=pipe)
        if dist.get_rank() != 0:
            follow(llm.engine, control)
            dist.destroy_process_group()
            return
        sync = StepSync(control)
    else:
        llm = LLM(args.model, device=args.device, engine_config=ecfg)
    tok = None
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(args.model)
    except Exception:
        tok = None
    name = args.served_model_name or args.model.rstrip("/").split("/")[-1]
    ae = AsyncEngine(llm.engine, name, sync=sync)
    try:
        uvicorn.run(build_app(ae, tok, name), host=args.host, port=args.port, log_level="warning")
    finally:
        ae.shutdown()


if __name__ == "__main__":
    main()
