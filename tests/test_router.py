"""Data-parallel router: conversation affinity, streaming pass-through, fleet metrics, fail-over.

The replicas here are small HTTP apps that report which replica served a call,
so the routing logic is tested without models (the replica server itself is
covered by test_server.py).
"""
import asyncio
import json
import socket
import threading
import time

import pytest

from granite_switch_b200.server.router import Router, affinity_key, build_router_app, rank_backends, sum_metrics


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _replica_app(name: str):
    from fastapi import FastAPI, Request
    from fastapi.responses import PlainTextResponse, StreamingResponse

    app = FastAPI()
    app.state.calls = 0

    async def serve(req: Request):
        body = await req.json()
        app.state.calls += 1
        if body.get("sleep_s"):
            await asyncio.sleep(body["sleep_s"])  # a slow generation
        if body.get("stream"):
            async def events():
                for i in range(3):
                    yield f"data: {json.dumps({'replica': name, 'i': i})}\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(events(), media_type="text/event-stream")
        return {"replica": name}

    app.post("/v1/completions")(serve)
    app.post("/v1/chat/completions")(serve)

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": "m"}]}

    @app.get("/metrics")
    async def metrics():
        return PlainTextResponse("# TYPE vllm:prefix_cache_hits_total counter\n"
                                 f"vllm:prefix_cache_hits_total {10 + app.state.calls}\n"
                                 'vllm:num_requests_running{model_name="m"} 2\n')

    return app


class _Replica:
    def __init__(self, name: str):
        import uvicorn

        self.app = _replica_app(name)
        self.port = _free_port()
        self.url = f"http://127.0.0.1:{self.port}"
        self.server = uvicorn.Server(uvicorn.Config(self.app, host="127.0.0.1", port=self.port, log_level="warning"))
        self.thread = threading.Thread(target=self.server.run, daemon=True)
        self.thread.start()
        deadline = time.time() + 20
        while not self.server.started and time.time() < deadline:
            time.sleep(0.05)
        assert self.server.started, "replica did not start"

    def stop(self):
        self.server.should_exit = True
        self.thread.join(10)


@pytest.fixture()
def replicas():
    rs = [_Replica("a"), _Replica("b"), _Replica("c")]
    yield rs
    for r in rs:
        r.stop()


def _conv(i: int, turn: int) -> dict:
    msgs = [{"role": "system", "content": f"document {i}"}, {"role": "user", "content": "first question"}]
    for t in range(turn):
        msgs += [{"role": "assistant", "content": f"answer {t}"}, {"role": "user", "content": f"question {t}"}]
    return {"messages": msgs, "max_tokens": 4, "chat_template_kwargs": {"adapter_name": f"adapter_{turn % 3}"}}


def test_affinity_key_and_rendezvous_ranking():
    # every turn (and every adapter call) of one conversation shares its key
    keys = {affinity_key("/v1/chat/completions", _conv(7, t)) for t in range(4)}
    assert len(keys) == 1
    assert affinity_key("/v1/chat/completions", _conv(8, 0)) not in keys
    assert affinity_key("/v1/completions", {"prompt": list(range(300)) + [1]}) == \
        affinity_key("/v1/completions", {"prompt": list(range(300)) + [2, 3]})
    assert affinity_key("/v1/completions", {"prompt": "x", "user": "u1"}) == "user:u1"
    assert affinity_key("/v1/completions", {"prompt": "x"}, {"x-session-id": "s"}) == "session:s"
    backends = ["http://r0", "http://r1", "http://r2", "http://r3"]
    owners = {k: rank_backends(str(k), backends)[0] for k in range(400)}
    assert len(set(owners.values())) == 4
    # dropping a replica moves only the keys it owned
    fewer = [b for b in backends if b != "http://r2"]
    for k, owner in owners.items():
        if owner != "http://r2":
            assert rank_backends(str(k), fewer)[0] == owner


def test_sum_metrics():
    a = "# TYPE x counter\nx 3\ny{l=\"1\"} 2\n"
    b = "# TYPE x counter\nx 4\ny{l=\"1\"} 1\ny{l=\"2\"} 5\n"
    out = sum_metrics([a, b])
    assert "x 7" in out and 'y{l="1"} 3' in out and 'y{l="2"} 5' in out and out.count("# TYPE x counter") == 1


def test_router_affinity_streaming_and_metrics(replicas):
    from fastapi.testclient import TestClient

    router = Router([r.url for r in replicas])
    with TestClient(build_router_app(router, health_interval_s=0)) as c:
        served = {}
        for i in range(12):
            for t in range(3):
                r = c.post("/v1/chat/completions", json=_conv(i, t))
                assert r.status_code == 200, r.text
                served.setdefault(i, set()).add(r.json()["replica"])
        assert all(len(s) == 1 for s in served.values())   # a conversation stays on one replica
        assert len(set().union(*served.values())) >= 2       # conversations spread over replicas
        with c.stream("POST", "/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 3, "stream": True}) as r:
            lines = [line for line in r.iter_lines() if line]
        assert lines[-1] == "data: [DONE]" and len(lines) == 4
        assert sum(router.inflight.values()) == 0
        m = c.get("/metrics").text
        # 36 chat calls + 1 stream, summed over the three replicas' counters (10 + calls each)
        assert "vllm:prefix_cache_hits_total 67" in m
        assert 'vllm:num_requests_running{model_name="m"} 6' in m
        assert "gsb_router_requests_total" in m and "gsb_router_failovers_total 0" in m
        assert c.get("/health").json()["status"] == "ok"
        assert c.get("/v1/models").json()["data"][0]["id"] == "m"


def test_router_failover(replicas):
    from fastapi.testclient import TestClient

    router = Router([r.url for r in replicas])
    down = replicas[1]
    with TestClient(build_router_app(router, health_interval_s=0)) as c:
        owned = [i for i in range(40) if router.choose(affinity_key("/v1/chat/completions", _conv(i, 0)))[0] == down.url]
        assert owned
        down.stop()
        for i in owned[:3]:
            r = c.post("/v1/chat/completions", json=_conv(i, 0))
            assert r.status_code == 200 and r.json()["replica"] != "b"
        assert router.failovers >= 1 and router.healthy[down.url] is False
        h = c.get("/health").json()
        assert h["status"] == "ok" and h["backends"][down.url] is False


def test_router_timeout_is_not_failover(replicas):
    """A replica that accepted the request but answers too slowly gets a 504: the request is
    not re-sent to another replica (it would run twice) and the replica stays in rotation."""
    from fastapi.testclient import TestClient

    router = Router([r.url for r in replicas], timeout_s=0.5)
    with TestClient(build_router_app(router, health_interval_s=0)) as c:
        body = {"prompt": [7, 8, 9], "max_tokens": 2, "sleep_s": 2.0}
        r = c.post("/v1/completions", json=body)
        assert r.status_code == 504, r.text
        assert sum(rep.app.state.calls for rep in replicas) == 1
        assert router.failovers == 0 and all(router.healthy.values())
        assert sum(router.inflight.values()) == 0


def test_router_stream_released_without_iteration(replicas):
    """The in-flight slot and the upstream response of a streaming call are released even when
    the relay generator never runs (the client went away before the body was read)."""
    from fastapi.testclient import TestClient

    router = Router([r.url for r in replicas])
    with TestClient(build_router_app(router, health_interval_s=0)) as c:
        with c.stream("POST", "/v1/completions", json={"prompt": [1, 2], "max_tokens": 3, "stream": True}):
            pass  # close without reading the body
        deadline = time.time() + 5
        while sum(router.inflight.values()) and time.time() < deadline:
            time.sleep(0.05)
        assert sum(router.inflight.values()) == 0
