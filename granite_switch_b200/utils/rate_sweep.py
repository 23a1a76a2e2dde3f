"""Benchmark config 3 matrix: Poisson arrival rates x aLoRA / LoRA x admission policy.

``python -m granite_switch_b200.utils.rate_sweep [--rates 1 2.5 5 16] [--steps 120]
[--reference] [--out results.jsonl]``

Runs ``bench.py`` once per point in a child process (the 8B-shape multi-adapter
workload on one GPU: a shared 4096-token context and a chain of 8 adapter
calls per conversation), as aLoRA (the control token placed before each
call's invocation, so every call reuses the cached base context) and as
standard LoRA (the control token at the start of the prompt, so no call can
reuse another adapter's KV), under the engine's default cache-affinity
admission and under FCFS. With ``--reference`` the unmodified reference
(vLLM with the granite-switch plugin) runs the same points with its own
(FCFS) scheduler. Every bench line is written to ``--out`` as it arrives and a
markdown table (output tok/s, p50 / p90 TTFT over every arrival with queue
wait included, waiters at the end, prefix-hit rate) is printed at the end.

Rates below the server's capacity give stationary TTFTs; rates above it show
how each admission policy degrades under overload (the queue then grows for
the whole run, and TTFT depends on how long the run lasted).
(reference workload: tutorials/scripts/comparison/alora_vs_lora_race/bench_pipeline_race.py:480-557)
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run_point(impl: str, rate: float, mode: str, policy: str, steps: int, warmup: int, timeout: int) -> dict:
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", impl, "--rate", str(rate), "--mode", mode,
           "--steps", str(steps), "--warmup", str(warmup)]
    if impl == "native":
        cmd += ["--scheduling-policy", policy]
    try:
        r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired:
        return {"impl": impl, "rate": rate, "mode": mode, "policy": policy, "error": f"timed out after {timeout} s"}
    line = None
    for ln in r.stdout.splitlines():
        if ln.startswith("{") and '"impl"' in ln:
            line = json.loads(ln)
    if line is None:
        return {"impl": impl, "rate": rate, "mode": mode, "policy": policy, "error": f"rc={r.returncode}",
                "stderr": r.stderr[-800:]}
    line.update(rate=rate, mode=mode, policy=policy if impl == "native" else "fcfs (vLLM)")
    return line


def table(rows: list[dict]) -> str:
    out = ["| impl | rate conv/s | mode | admission | output tok/s | p50 TTFT s | p90 TTFT s | waiting at end | "
           "prefix-hit rate |", "|---|---|---|---|---|---|---|---|---|"]
    for r in rows:
        if "error" in r or "unavailable" in r:
            out.append(f"| {r.get('impl')} | {r.get('rate')} | {r.get('mode')} | {r.get('policy')} | "
                       f"{r.get('error') or r.get('unavailable')} | | | | |")
            continue
        out.append(f"| {r['impl']} | {r['rate']} | {r['mode']} | {r['policy']} | {r['value']:.0f} | "
                   f"{r.get('p50_ttft_s')} | {r.get('p90_ttft_s')} | {r.get('ttft_waiting_at_end')} | "
                   f"{r.get('prefix_hit_rate')} |")
    return "\n".join(out)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--rates", type=float, nargs="*", default=[1.0, 2.5, 5.0, 16.0])
    ap.add_argument("--modes", nargs="*", default=["alora", "lora"])
    ap.add_argument("--policies", nargs="*", default=["cache_affinity", "fcfs"])
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--reference", action="store_true", help="also run the reference arm at every rate and mode")
    ap.add_argument("--timeout", type=int, default=900, help="seconds per point")
    ap.add_argument("--out", default=None, help="append every bench line to this JSONL file")
    args = ap.parse_args(argv)
    rows = []
    points = [("native", rate, mode, pol) for rate in args.rates for mode in args.modes for pol in args.policies]
    if args.reference:
        points += [("reference", rate, mode, "fcfs") for rate in args.rates for mode in args.modes]
    for impl, rate, mode, pol in points:
        r = run_point(impl, rate, mode, pol, args.steps, args.warmup, args.timeout)
        rows.append(r)
        print(json.dumps(r), flush=True)
        if args.out:
            with open(args.out, "a") as f:
                f.write(json.dumps(r) + "\n")
    print(table(rows), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
