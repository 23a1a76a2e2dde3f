"""Multi-turn adapter-pipeline race against one or more OpenAI-compatible servers.

Each conversation is a document context followed by ``--turns`` user
questions. For every turn the client runs a pipeline of adapter calls over the
whole conversation (``--step NAME=ADAPTER``, each a short chat completion with
``chat_template_kwargs.adapter_name``), then a base-model answer that joins the
history. Serving aLoRA adapters, every call after the first re-reads the same
context from the prefix cache; serving LoRA adapters (active from the first
token), each adapter's call re-prefills it. Run one server per checkpoint and
compare (reference behaviour:
tutorials/scripts/comparison/alora_vs_lora_race/bench_pipeline_race.py, whose
RAG retrieval and intrinsic libraries are replaced here by synthetic documents
and plain chat calls, so it needs no extra packages).

``python -m granite_switch_b200.utils.race --server ALORA=http://127.0.0.1:8111
--server LORA=http://127.0.0.1:8112 --step rewrite=query_rewrite
--step answerability=answerability [--conversations 32 --turns 5 --concurrency 24]``

Writes ``--out`` (JSON): per server the wall time, the median latency of every
pipeline step, client-side completion counts, and the server's own prefix-cache
hit rate, mean TTFT and mean end-to-end latency over the run, from ``/metrics``.
"""
from __future__ import annotations

import argparse
import json
import random
import statistics
import threading
import time
import urllib.request
from concurrent.futures import ThreadPoolExecutor

_WORDS = ("the permit office form fee renewal resident license housing benefit tax county record "
          "application deadline service public health vehicle water energy school transit code").split()


def _post(url: str, body: dict, timeout: float) -> dict:
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read())


def _get(url: str, timeout: float = 10.0) -> str:
    with urllib.request.urlopen(url, timeout=timeout) as r:
        return r.read().decode()


def parse_metrics(text: str) -> dict[str, float]:
    """Prometheus text -> {name: value} for the unlabelled-by-bucket series (labels dropped, summed)."""
    out: dict[str, float] = {}
    for line in text.splitlines():
        if not line or line.startswith("#") or "_bucket" in line:
            continue
        name, _, val = line.rpartition(" ")
        name = name.split("{", 1)[0]
        try:
            out[name] = out.get(name, 0.0) + float(val)
        except ValueError:
            continue
    return out


def server_summary(before: dict[str, float], after: dict[str, float], prefix: str = "vllm:") -> dict:
    """Server-side figures over the run: prefix-cache hit rate, mean TTFT and mean request latency."""
    d = {k: after.get(k, 0.0) - before.get(k, 0.0) for k in after}
    q, h = d.get(prefix + "prefix_cache_queries_total", 0.0), d.get(prefix + "prefix_cache_hits_total", 0.0)

    def mean(name):
        n = d.get(prefix + name + "_count", 0.0)
        return d.get(prefix + name + "_sum", 0.0) / n if n else None

    return {"prefix_hit_rate": h / q if q else None, "prefix_cache_queries": q, "prefix_cache_hits": h,
            "mean_ttft_s": mean("time_to_first_token_seconds"),
            "mean_e2e_s": mean("e2e_request_latency_seconds"),
            "generation_tokens": d.get(prefix + "generation_tokens_total", 0.0)}


def make_conversations(n: int, turns: int, doc_words: int, seed: int = 0) -> list[dict]:
    rng = random.Random(seed)
    convs = []
    for i in range(n):
        doc = " ".join(rng.choice(_WORDS) for _ in range(doc_words))
        qs = [f"Question {t + 1}: what does the document say about {rng.choice(_WORDS)} and {rng.choice(_WORDS)}?"
              for t in range(turns)]
        convs.append({"id": i, "document": doc, "questions": qs})
    return convs


def run_conversation(base_url: str, conv: dict, steps: list[tuple[str, str]], step_tokens: int,
                     answer_tokens: int, timeout: float, times: dict[str, list[float]], lock) -> int:
    """One conversation's turns; returns the number of completions made."""
    url = base_url.rstrip("/") + "/v1/chat/completions"
    msgs = [{"role": "system", "content": "Answer from this document.\n" + conv["document"]}]
    calls = 0
    for q in conv["questions"]:
        msgs = msgs + [{"role": "user", "content": q}]
        for name, adapter in steps:
            t0 = time.perf_counter()
            _post(url, {"messages": msgs, "max_tokens": step_tokens, "temperature": 0.0,
                        "chat_template_kwargs": {"adapter_name": adapter}}, timeout)
            with lock:
                times.setdefault(name, []).append(time.perf_counter() - t0)
            calls += 1
        t0 = time.perf_counter()
        r = _post(url, {"messages": msgs, "max_tokens": answer_tokens, "temperature": 0.0}, timeout)
        with lock:
            times.setdefault("generation", []).append(time.perf_counter() - t0)
        calls += 1
        msgs = msgs + [{"role": "assistant", "content": r["choices"][0]["message"]["content"] or "ok"}]
    return calls


def race_server(label: str, base_url: str, convs: list[dict], steps, concurrency: int, step_tokens: int,
                answer_tokens: int, timeout: float = 600.0) -> dict:
    before = parse_metrics(_get(base_url.rstrip("/") + "/metrics"))
    times: dict[str, list[float]] = {}
    lock = threading.Lock()
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=concurrency) as pool:
        calls = sum(pool.map(lambda c: run_conversation(base_url, c, steps, step_tokens, answer_tokens, timeout,
                                                        times, lock), convs))
    wall = time.perf_counter() - t0
    after = parse_metrics(_get(base_url.rstrip("/") + "/metrics"))
    return {"label": label, "url": base_url, "wall_total": round(wall, 3), "completions": calls,
            "step_times": {k: {"median_s": round(statistics.median(v), 4), "n": len(v)} for k, v in times.items()},
            "server": server_summary(before, after)}


def main(argv=None) -> dict:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--server", action="append", required=True, help="LABEL=URL (repeatable)")
    p.add_argument("--step", action="append", default=None, help="NAME=ADAPTER pipeline step (repeatable)")
    p.add_argument("--conversations", type=int, default=32)
    p.add_argument("--turns", type=int, default=5)
    p.add_argument("--concurrency", type=int, default=24, help="conversations in flight per server")
    p.add_argument("--doc-words", type=int, default=1500)
    p.add_argument("--step-tokens", type=int, default=8)
    p.add_argument("--answer-tokens", type=int, default=64)
    p.add_argument("--mode", choices=["simultaneous", "sequential"], default="simultaneous")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--out", default="race_results.json")
    args = p.parse_args(argv)
    servers = [tuple(s.split("=", 1)) for s in args.server]
    steps = [tuple(s.split("=", 1)) for s in (args.step or ["step=adapter_0"])]
    convs = make_conversations(args.conversations, args.turns, args.doc_words, args.seed)
    run = lambda lu: race_server(lu[0], lu[1], convs, steps, args.concurrency, args.step_tokens,  # noqa: E731
                                 args.answer_tokens)
    t0 = time.perf_counter()
    if args.mode == "simultaneous" and len(servers) > 1:
        with ThreadPoolExecutor(max_workers=len(servers)) as pool:
            results = list(pool.map(run, servers))
    else:
        results = [run(s) for s in servers]
    out = {"created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), "wall": round(time.perf_counter() - t0, 3),
           "conversations": args.conversations, "turns": args.turns, "steps": [n for n, _ in steps],
           "servers": {r["label"]: r for r in results}}
    with open(args.out, "w") as f:
        json.dump(out, f, indent=2)
    for r in results:
        s = r["server"]
        hr = "n/a" if s["prefix_hit_rate"] is None else f"{100 * s['prefix_hit_rate']:.1f}%"
        print(f"{r['label']:>12}: wall {r['wall_total']:.1f} s, prefix-cache hit rate {hr}, "
              f"steps " + ", ".join(f"{k} {v['median_s']:.2f} s" for k, v in r["step_times"].items()))
    return out


if __name__ == "__main__":
    main()
