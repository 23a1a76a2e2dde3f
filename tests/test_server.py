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
