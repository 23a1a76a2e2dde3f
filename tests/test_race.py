"""Adapter-pipeline race against in-process servers (CPU engines): aLoRA adapters, which activate
at the generation prompt, reuse the conversation's cached context; LoRA adapters re-prefill it."""
import socket
import threading
import time

import pytest
import torch


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _serve(tmp_path, technology):
    import uvicorn

    from granite_switch_b200.composer.compose import compose_checkpoint
    from granite_switch_b200.composer.synthetic import base_config, random_base_state, synthetic_adapters
    from granite_switch_b200.composer.tokenizer_setup import configure_tokenizer, encode
    from granite_switch_b200.engine import LLM, EngineConfig
    from granite_switch_b200.server.app import build_app
    from granite_switch_b200.server.async_engine import AsyncEngine
    from tests.tokenizer_stub import granite_template, make_tokenizer

    tok = make_tokenizer(granite_template("4.1"))
    cfg = base_config("tiny", num_hidden_layers=2)
    ads = synthetic_adapters(cfg, 2, 8, ("q", "k", "v", "o"), seed=1, technology=technology)
    for a in ads:
        a.invocation_tokens = encode(tok, "<|start_of_role|>assistant<|end_of_role|>") if technology == "alora" \
            else None
    ids, setup = configure_tokenizer(tok, ads)
    d = str(tmp_path / technology)
    compose_checkpoint(cfg, random_base_state(cfg), ads, d, dtype=torch.float32, control_token_ids=ids,
                       default_substitute=setup.lora_substitute)
    llm = LLM(d, device="cpu", engine_config=EngineConfig(max_num_seqs=8, max_num_batched_tokens=1024,
                                                          num_kv_blocks=512, max_model_len=2048))
    ae = AsyncEngine(llm.engine, technology)
    port = _free_port()
    server = uvicorn.Server(uvicorn.Config(build_app(ae, tok, technology), host="127.0.0.1", port=port,
                                           log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    for _ in range(200):
        if server.started:
            break
        time.sleep(0.05)
    return server, th, ae, f"http://127.0.0.1:{port}"


@pytest.mark.slow
def test_alora_race_reuses_context(tmp_path):
    from granite_switch_b200.utils.race import main

    running = [_serve(tmp_path, "alora"), _serve(tmp_path, "lora")]
    try:
        out = main(["--server", f"ALORA={running[0][3]}", "--server", f"LORA={running[1][3]}",
                    "--step", "rewrite=adapter_0", "--step", "answerability=adapter_1",
                    "--conversations", "2", "--turns", "2", "--concurrency", "2", "--doc-words", "40",
                    "--step-tokens", "2", "--answer-tokens", "4", "--out", str(tmp_path / "race.json")])
    finally:
        for server, th, ae, _ in running:
            server.should_exit = True
            th.join(timeout=30)
            ae.shutdown()
    a, lo = out["servers"]["ALORA"], out["servers"]["LORA"]
    assert a["completions"] == lo["completions"] == 2 * 2 * 3
    assert set(a["step_times"]) == {"rewrite", "answerability", "generation"}
    assert a["server"]["prefix_hit_rate"] > lo["server"]["prefix_hit_rate"] >= 0
