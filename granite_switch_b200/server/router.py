"""Data-parallel front end: one OpenAI-compatible endpoint over several engine replicas.

Each replica is a ``python -m granite_switch_b200.server`` process (one GPU, or a
tensor / pipeline-parallel group under torchrun). The router keeps every request
of a conversation on one replica, so the conversation's KV stays in that
replica's prefix cache and each adapter call after the first re-reads it
instead of prefilling it again (the reference leaves data parallelism to
vLLM, which it never configures; this is the replica-per-GPU-group layout).

Affinity key, in order: the request's ``user`` field (OpenAI's end-user id), the
``X-Session-Id`` header, else the conversation's stable prefix: for chat
requests the first message (the system prompt or document) and the first user
turn; for completions the first 256 prompt token ids or 1024 prompt
characters. The replica is chosen by rendezvous hashing over the healthy
replicas (adding or removing a replica moves only the keys it wins or
owned). When the chosen replica has ``--max-inflight-skew`` more requests in
flight than the least loaded one, the request goes to the least loaded one.
A replica that refuses a connection is marked down and the request is retried
on the next replica in hash order; a background task re-probes ``/health``.
A request that reached a replica is never re-sent: a timeout answers 504 and a
connection broken mid-request 502, and neither marks the replica down (it may
still be generating, and one slow request says nothing about its health).

``python -m granite_switch_b200.server.router --backend http://127.0.0.1:8001
--backend http://127.0.0.1:8002 [--port 8000]``

Endpoints: ``POST /v1/completions``, ``POST /v1/chat/completions`` (streaming
passed through), ``GET /v1/models``, ``GET /health`` (503 when no replica is
up), ``GET /metrics`` (the router's own counters plus every series of the
replicas' ``/metrics`` summed over replicas, so fleet-wide prefix-cache hits
and token counts read like one server's).
"""
# (no postponed annotations: FastAPI resolves the endpoints' ``Request`` parameter
# from the annotation object, and ``Request`` is imported inside build_router_app)
import argparse
import asyncio
import contextlib
import hashlib
import json

STREAM_CHUNK = 1 << 14


def affinity_key(path: str, body: dict, headers: dict | None = None) -> str:
    """The string whose hash picks the replica (see the module docstring)."""
    if body.get("user"):
        return "user:" + str(body["user"])
    if headers:
        sid = headers.get("x-session-id") or headers.get("X-Session-Id")
        if sid:
            return "session:" + sid
    if path.endswith("/chat/completions"):
        msgs = body.get("messages") or []
        head = msgs[:1]
        first_user = next((m for m in msgs[1:] if m.get("role") == "user"), None)
        if first_user is not None:
            head = head + [first_user]
        return "chat:" + json.dumps(head, sort_keys=True, default=str)
    prompt = body.get("prompt", "")
    if isinstance(prompt, list) and prompt and isinstance(prompt[0], list):
        prompt = prompt[0]  # a batch: route by its first prompt
    if isinstance(prompt, list):
        return "ids:" + ",".join(str(int(t)) for t in prompt[:256])
    return "text:" + str(prompt)[:1024]


def _score(key: str, backend: str) -> int:
    return int.from_bytes(hashlib.blake2b(f"{key}\x00{backend}".encode(), digest_size=8).digest(), "big")


def rank_backends(key: str, backends: list[str]) -> list[str]:
    """Backends in rendezvous-hash order for ``key`` (the first one owns the key)."""
    return sorted(backends, key=lambda b: _score(key, b), reverse=True)


def sum_metrics(texts: list[str]) -> str:
    """Sum Prometheus text series with the same name and labels across replicas.

    Comment lines (``# HELP`` / ``# TYPE``) of the first replica that has a
    series are kept; sums of gauges are fleet totals too (requests running,
    waiting), which is what a fleet view wants.
    """
    order: list[str] = []
    values: dict[str, float] = {}
    comments: dict[str, list[str]] = {}
    pending: list[str] = []
    for text in texts:
        for line in text.splitlines():
            if not line:
                continue
            if line.startswith("#"):
                pending.append(line)
                continue
            series, _, val = line.rpartition(" ")
            try:
                v = float(val)
            except ValueError:
                pending = []
                continue
            if series not in values:
                order.append(series)
                values[series] = 0.0
                comments[series] = pending
            values[series] += v
            pending = []
    out = []
    for series in order:
        out.extend(comments[series])
        v = values[series]
        out.append(f"{series} {int(v) if v == int(v) else v}")
    return "\n".join(out) + ("\n" if out else "")


class Router:
    def __init__(self, backends: list[str], max_inflight_skew: int | None = 64, timeout_s: float = 3600.0):
        if not backends:
            raise ValueError("at least one backend is required")
        self.backends = [b.rstrip("/") for b in backends]
        self.healthy = {b: True for b in self.backends}
        self.inflight = {b: 0 for b in self.backends}
        self.requests = {b: 0 for b in self.backends}
        self.failovers = 0
        self.skew_moves = 0
        self.max_inflight_skew = max_inflight_skew
        self.timeout_s = timeout_s
        self.session = None

    async def start(self):
        import aiohttp

        self.session = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=self.timeout_s))

    async def close(self):
        if self.session is not None:
            await self.session.close()
            self.session = None

    def choose(self, key: str) -> list[str]:
        """Replicas to try, in order: the key's owner (or the least loaded one under skew), then the rest."""
        up = [b for b in self.backends if self.healthy[b]] or list(self.backends)
        order = rank_backends(key, up)
        if self.max_inflight_skew is not None and len(order) > 1:
            least = min(order, key=lambda b: self.inflight[b])
            if self.inflight[order[0]] - self.inflight[least] > self.max_inflight_skew:
                self.skew_moves += 1
                order.remove(least)
                order.insert(0, least)
        return order

    async def probe(self, backend: str) -> bool:
        try:
            async with self.session.get(backend + "/health", timeout=5) as r:
                ok = r.status == 200
        except Exception:
            ok = False
        self.healthy[backend] = ok
        return ok

    async def health_loop(self, interval_s: float):
        while True:
            await asyncio.gather(*(self.probe(b) for b in self.backends))
            await asyncio.sleep(interval_s)

    def metrics_text(self) -> str:
        lines = ["# TYPE gsb_router_requests_total counter"]
        lines += [f'gsb_router_requests_total{{backend="{b}"}} {n}' for b, n in self.requests.items()]
        lines.append("# TYPE gsb_router_inflight gauge")
        lines += [f'gsb_router_inflight{{backend="{b}"}} {n}' for b, n in self.inflight.items()]
        lines.append("# TYPE gsb_router_backend_up gauge")
        lines += [f'gsb_router_backend_up{{backend="{b}"}} {int(h)}' for b, h in self.healthy.items()]
        lines.append("# TYPE gsb_router_failovers_total counter")
        lines.append(f"gsb_router_failovers_total {self.failovers}")
        lines.append("# TYPE gsb_router_skew_moves_total counter")
        lines.append(f"gsb_router_skew_moves_total {self.skew_moves}")
        return "\n".join(lines) + "\n"


def build_router_app(router: Router, health_interval_s: float = 5.0):
    import aiohttp
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, PlainTextResponse, Response, StreamingResponse
    from starlette.background import BackgroundTask

    @contextlib.asynccontextmanager
    async def lifespan(app):
        await router.start()
        task = asyncio.create_task(router.health_loop(health_interval_s)) if health_interval_s > 0 else None
        try:
            yield
        finally:
            if task is not None:
                task.cancel()
                with contextlib.suppress(asyncio.CancelledError):
                    await task
            await router.close()

    app = FastAPI(lifespan=lifespan)

    async def forward(request: Request, path: str):
        raw = await request.body()
        try:
            body = json.loads(raw or b"{}")
        except json.JSONDecodeError:
            return JSONResponse({"error": {"message": "request body is not JSON"}}, status_code=400)
        key = affinity_key(path, body, dict(request.headers))
        headers = {"Content-Type": "application/json"}
        last_error = None
        for i, backend in enumerate(router.choose(key)):
            if i > 0:
                router.failovers += 1
            router.inflight[backend] += 1
            try:
                resp = await router.session.post(backend + path, data=raw, headers=headers)
            except aiohttp.ClientConnectorError as e:
                # the connection was never made, so the replica never saw the request: try the next one
                router.inflight[backend] -= 1
                router.healthy[backend] = False
                last_error = e
                continue
            except asyncio.TimeoutError:
                # the replica may have accepted the request and still be generating; sending it
                # elsewhere would run it twice, and one slow request says nothing about health
                router.inflight[backend] -= 1
                return JSONResponse({"error": {"message": f"replica {backend} timed out"}}, status_code=504)
            except aiohttp.ClientError as e:
                # the connection broke after the request went out: same reasoning as a timeout
                router.inflight[backend] -= 1
                return JSONResponse({"error": {"message": f"replica {backend} failed: {e}"}}, status_code=502)
            router.requests[backend] += 1
            done = False

            def release(resp=resp, backend=backend):
                # idempotent: reached from the relay's finally, the response's background task
                # (which runs when the client disconnects before the relay starts) or the
                # non-streaming path below
                nonlocal done
                if not done:
                    done = True
                    resp.release()
                    router.inflight[backend] -= 1

            if body.get("stream"):
                async def relay(resp=resp, release=release):
                    try:
                        async for chunk in resp.content.iter_chunked(STREAM_CHUNK):
                            yield chunk
                    finally:
                        release()

                try:
                    return StreamingResponse(relay(), status_code=resp.status,
                                             media_type=resp.headers.get("Content-Type", "text/event-stream"),
                                             background=BackgroundTask(release))
                except BaseException:
                    release()
                    raise
            try:
                data = await resp.read()
                return Response(content=data, status_code=resp.status,
                                media_type=resp.headers.get("Content-Type", "application/json"))
            finally:
                release()
        return JSONResponse({"error": {"message": f"no replica reachable: {last_error}"}}, status_code=503)

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await forward(request, "/v1/completions")

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        return await forward(request, "/v1/chat/completions")

    @app.get("/v1/models")
    async def models():
        for b in router.backends:
            if not router.healthy[b]:
                continue
            try:
                async with router.session.get(b + "/v1/models") as r:
                    return JSONResponse(await r.json(), status_code=r.status)
            except Exception:
                router.healthy[b] = False
        return JSONResponse({"error": {"message": "no replica reachable"}}, status_code=503)

    @app.get("/health")
    async def health():
        up = {b: router.healthy[b] for b in router.backends}
        return JSONResponse({"status": "ok" if any(up.values()) else "down", "backends": up},
                            status_code=200 if any(up.values()) else 503)

    @app.get("/metrics")
    async def metrics():
        texts = []
        for b in router.backends:
            if not router.healthy[b]:
                continue
            try:
                async with router.session.get(b + "/metrics") as r:
                    if r.status == 200:
                        texts.append(await r.text())
            except Exception:
                router.healthy[b] = False
        return PlainTextResponse(router.metrics_text() + sum_metrics(texts))

    return app


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--backend", action="append", required=True, help="replica base URL (repeatable)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-inflight-skew", type=int, default=64,
                    help="send to the least loaded replica when the owner has this many more requests in flight "
                         "(negative: never)")
    ap.add_argument("--health-interval", type=float, default=5.0, help="seconds between /health probes")
    args = ap.parse_args(argv)
    import uvicorn

    skew = args.max_inflight_skew if args.max_inflight_skew >= 0 else None
    app = build_router_app(Router(args.backend, skew), args.health_interval)
    uvicorn.run(app, host=args.host, port=args.port, log_level="warning")


if __name__ == "__main__":
    main()
