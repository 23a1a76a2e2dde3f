"""OpenAI-compatible server over the CPU reference executor (token-id prompts)."""
import json
import os

import pytest
import torch

from granite_switch_b200.composer.synthetic import compose_synthetic


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    from fastapi.testclient import TestClient

    from granite_switch_b200.engine import LLM, EngineConfig
    from granite_switch_b200.server.app import build_app
    from granite_switch_b200.server.async_engine import AsyncEngine

    d = str(tmp_path_factory.mktemp("srv"))
    compose_synthetic(d, "tiny", num_adapters=2, rank=8, seed=0, dtype=torch.float32, num_hidden_layers=2)
    llm = LLM(d, device="cpu", engine_config=EngineConfig(max_num_seqs=4, max_num_batched_tokens=256,
                                                          num_kv_blocks=64, max_model_len=512))
    ae = AsyncEngine(llm.engine, "tiny")
    with TestClient(build_app(ae, None, "tiny")) as c:
        c.model_dir = d
        yield c
    ae.shutdown()


def test_completions_token_ids_and_metrics(client):
    idx = json.load(open(os.path.join(client.model_dir, "adapter_index.json")))
    ctrl = idx["adapters"][0]["control_token"]["id"]
    ctx = list(range(5, 69))
    r1 = client.post("/v1/completions", json={"prompt": ctx + [ctrl, 7, 8], "max_tokens": 4})
    assert r1.status_code == 200, r1.text
    body = r1.json()
    assert len(body["choices"][0]["token_ids"]) == 4 and body["usage"]["completion_tokens"] == 4
    ctrl2 = idx["adapters"][1]["control_token"]["id"]
    r2 = client.post("/v1/completions", json={"prompt": ctx + [ctrl2, 9], "max_tokens": 2})
    assert r2.json()["usage"]["prompt_tokens_details"]["cached_tokens"] == 64
    m = client.get("/metrics").text
    assert "vllm:prefix_cache_hits_total" in m and "vllm:time_to_first_token_seconds_bucket" in m
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"


def test_text_prompt_without_tokenizer_is_rejected(client):
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 2})
    assert r.status_code == 400


def test_streaming(client):
    with client.stream("POST", "/v1/completions", json={"prompt": list(range(10, 30)), "max_tokens": 3,
                                                         "stream": True}) as r:
        lines = [l for l in r.iter_lines() if l]
    assert lines[-1] == "data: [DONE]"
    toks = []
    for l in lines[:-1]:
        toks += json.loads(l[6:])["choices"][0]["token_ids"]
    assert len(toks) == 3


def test_chat_completions_place_the_control_token(tmp_path):
    """Chat requests render the composed chat template: ``chat_template_kwargs.adapter_name``
    puts the adapter's control token in the prompt, and the prompt shares its prefix with the
    base render (aLoRA at the assistant boundary)."""
    from fastapi.testclient import TestClient

    from granite_switch_b200.composer.compose import compose_checkpoint
    from granite_switch_b200.composer.synthetic import base_config, random_base_state, synthetic_adapters
    from granite_switch_b200.composer.tokenizer_setup import configure_tokenizer, encode
    from granite_switch_b200.engine import LLM, EngineConfig
    from granite_switch_b200.server.app import build_app
    from granite_switch_b200.server.async_engine import AsyncEngine
    from tests.tokenizer_stub import granite_template, make_tokenizer

    tok = make_tokenizer(granite_template("4.1"))
    cfg = base_config("tiny", num_hidden_layers=2)
    ads = synthetic_adapters(cfg, 2, 8, ("q", "k", "v", "o"), seed=1)
    for a in ads:
        a.invocation_tokens = encode(tok, "<|start_of_role|>assistant<|end_of_role|>")
    ids, setup = configure_tokenizer(tok, ads)
    d = str(tmp_path / "chat")
    compose_checkpoint(cfg, random_base_state(cfg), ads, d, dtype=torch.float32, control_token_ids=ids,
                       default_substitute=setup.lora_substitute)
    llm = LLM(d, device="cpu", engine_config=EngineConfig(max_num_seqs=4, max_num_batched_tokens=256,
                                                          num_kv_blocks=64, max_model_len=512))
    ae = AsyncEngine(llm.engine, "tiny")
    msgs = [{"role": "user", "content": "Is the sky blue?"}]
    try:
        with TestClient(build_app(ae, tok, "tiny")) as c:
            plain = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2, "return_token_ids": True})
            assert plain.status_code == 200, plain.text
            r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2, "return_token_ids": True,
                                                     "chat_template_kwargs": {"adapter_name": "adapter_1"}})
            assert r.status_code == 200, r.text
            p0, p1 = plain.json()["prompt_token_ids"], r.json()["prompt_token_ids"]
            assert ids[1] in p1 and ids[1] not in p0
            cut = p1.index(ids[1])
            assert p1[:cut] == p0[:cut] and len(p1) == len(p0)
            assert r.json()["usage"]["prompt_tokens_details"]["cached_tokens"] >= 16 * (cut // 16) > 0
    finally:
        ae.shutdown()


def _lockstep_worker(rank, world, port, model_dir, prompts, q):
    import asyncio

    import torch.distributed as dist

    from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams
    from granite_switch_b200.server.async_engine import AsyncEngine, StepSync, follow

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    llm = LLM(model_dir, device="cpu", engine_config=EngineConfig(max_num_seqs=2, max_num_batched_tokens=64,
                                                                  num_kv_blocks=64, max_model_len=512))
    done = {}
    if rank == 0:
        ae = AsyncEngine(llm.engine, "tiny", sync=StepSync(dist.group.WORLD, heartbeat_s=0.05))

        async def run():
            reqs = await asyncio.gather(*[ae.generate(p, SamplingParams(max_tokens=5)) for p in prompts])
            return {r.request_id: r.output_ids for r in reqs}

        done = asyncio.run(run())
        ae.shutdown()
    else:
        llm.engine.on_finish = lambda r: done.__setitem__(r.request_id, list(r.output_ids))
        follow(llm.engine, dist.group.WORLD)
    out = [None] * world
    dist.all_gather_object(out, done)
    if rank == 0:
        q.put(out)
    dist.destroy_process_group()


def test_multi_rank_lockstep_serving(client):
    """Rank 0 serves and publishes each step's new requests; the follower rank replays them and
    takes the same scheduling decisions (gloo ranks on CPU)."""
    import socket

    import torch.multiprocessing as mp

    idx = json.load(open(os.path.join(client.model_dir, "adapter_index.json")))
    ctrl = idx["adapters"][1]["control_token"]["id"]
    prompts = [list(range(5, 40)), list(range(7, 30)) + [ctrl, 3], list(range(50, 90)), [9, 8, 7, ctrl, 6]]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_lockstep_worker, args=(r, 2, port, client.model_dir, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    lead, follower = out
    assert len(lead) == len(prompts) and lead == follower
