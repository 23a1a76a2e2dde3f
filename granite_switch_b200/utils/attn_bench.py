"""Attention kernel timing (CUDA events, after warm-up) on the benchmark model's head shape.

``python -m granite_switch_b200.utils.attn_bench [--iters 20]`` prints one JSON
line per case: tcgen05 prefill attention on a fresh causal 4k prompt and on 8
chunks of 512 new tokens over 3.5k cached tokens (TFLOP/s, causal FLOPs
counted once), and decode attention for 128 requests x 4.2k cached tokens
(GB/s of K/V read): over the bf16 cache with two or three ring stages, and over the
bf16 and fp8 caches with 1-3 key splits, L2 flushed (256 MB write) before each
launch (``decode_split``). 32 query / 8 KV heads, head_dim 128 (Granite-8B shape).
``--decode-only`` skips the prefill cases. ``--library`` also times FlashInfer's
Blackwell attention (the trtllm-gen paged decode and context kernels vLLM serves with on
B200) on the same caches, shapes and flush rule, and reports its largest difference from
this package's output.
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import _native
from ..ops import attention as A


def _setup(q_lens, kv_lens, hq=32, hkv=8, d=128, dev="cuda"):
    nblk = sum((l + 15) // 16 for l in kv_lens) + 4
    kc = torch.randn(nblk, hkv, 16, d, device=dev).bfloat16()
    vc = torch.randn_like(kc)
    maxb = max((l + 15) // 16 for l in kv_lens)
    bt = torch.zeros(len(kv_lens), maxb, dtype=torch.int32)
    p = 0
    for i, l in enumerate(kv_lens):
        for j in range((l + 15) // 16):
            bt[i, j] = p
            p += 1
    t = sum(q_lens)
    q = torch.randn(t, (hq + 2 * hkv) * d, device=dev).bfloat16()
    out = torch.empty(t, hq * d, device=dev).bfloat16()
    qs = [0]
    for l in q_lens:
        qs.append(qs[-1] + l)
    i32 = dict(dtype=torch.int32, device=dev)
    return kc, vc, bt.to(dev), q, out, torch.tensor(qs, **i32), torch.tensor(kv_lens, **i32)


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _time_flushed(fn, iters: int, flush: torch.Tensor) -> float:
    """Median event-timed launch with the L2 flushed before each."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2]


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--decode-only", action="store_true")
    p.add_argument("--library", action="store_true", help="also time FlashInfer's trtllm-gen kernels")
    args = p.parse_args()
    _native.native()
    hq, hkv, d = 32, 8, 128
    i32 = dict(dtype=torch.int32, device="cuda")
    prefill_cases = () if args.decode_only else (("prefill_causal_4k", [4096], [4096]),
                                                 ("prefill_8x512_over_3584", [512] * 8, [4096] * 8))
    for name, q_lens, kv_lens in prefill_cases:
        kc, vc, bt, q, out, qs, kvl = _setup(q_lens, kv_lens)
        # causal FLOPs: each query attends to (ctx + its index + 1) keys; 4 flop per (q, k, d)
        pairs = sum(ql * (kl - ql) + ql * (ql + 1) // 2 for ql, kl in zip(q_lens, kv_lens))
        flops = 4.0 * pairs * hq * d
        for rows in (128, 256):  # one / two query tiles per CTA
            ws, wr = A.build_work(q_lens, hq // hkv, rows, kv_lens)
            ws, wr = torch.tensor(ws, **i32), torch.tensor(wr, **i32)
            for packed in (0, 1):  # softmax on scalar / packed f32x2 arithmetic
                old = _native.native().attn_packed(packed)
                ms = _time(lambda: A.prefill_attention_tc(q, kc, vc, bt, qs, kvl, ws, wr, hq, 0.088, out, rows),
                           args.iters)
                _native.native().attn_packed(old)
                print(json.dumps({"case": name, "rows": rows, "packed": packed, "ms": round(ms, 4),
                                  "tflops": round(flops / ms / 1e9, 1)}), flush=True)
        if args.library:
            _library_prefill(name, q, kc, vc, bt, q_lens, kv_lens, hq, d, out, flops, args.iters)
    q_lens, kv_lens = [1] * 128, [4200] * 128
    kc, vc, bt, q, out, qs, kvl = _setup(q_lens, kv_lens)
    ws, wr = A.build_work(q_lens, hq // hkv, 16)
    ws, wr = torch.tensor(ws, **i32), torch.tensor(wr, **i32)
    kv_bytes = 2 * sum(kv_lens) * hkv * d * 2
    for stages in (3, 2):  # two CTAs per SM with 3 stages, or three with 2
        old = _native.native().attn_decode_stages(stages)
        ms = _time(lambda: A.paged_attention(q, kc, vc, bt, qs, kvl, ws, wr, 16, hq, 0.088, out, 1), args.iters)
        _native.native().attn_decode_stages(old)
        print(json.dumps({"case": "decode_128x4200", "stages": stages, "ms": round(ms, 4),
                          "gbs": round(kv_bytes / ms / 1e6, 1)}), flush=True)
    # bf16 and fp8 caches, key splits 1-3, L2 flushed before each launch
    dev = "cuda"
    nblk = kc.shape[0]
    k8 = torch.randint(0, 126, kc.shape, dtype=torch.uint8, device=dev)  # finite e4m3 bytes
    v8 = torch.randint(0, 126, (nblk, hkv, d, 16), dtype=torch.uint8, device=dev)
    ks = torch.full(kc.shape[:3], 0.01, device=dev)
    vs = torch.full_like(ks, 0.01)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    b = len(q_lens)
    for ns in (1, 2, 3):
        wso = torch.empty(ns, b, hq, d, device=dev)
        wsl = torch.empty(ns, b, hq, device=dev)
        for cache, kk, vv, sk, sv, per in (("bf16", kc, vc, None, None, 2), ("fp8", k8, v8, ks, vs, 1)):
            ms = _time_flushed(lambda: A.paged_attention(q, kk, vv, bt, qs, kvl, ws, wr, 16, hq, 0.088, out, ns,
                                                         wso, wsl, k_scale=sk, v_scale=sv), args.iters, flush)
            nbytes = 2 * sum(kv_lens) * hkv * d * per
            print(json.dumps({"case": "decode_split", "cache": cache, "nsplit": ns, "ms": round(ms, 4),
                              "kv_tbs": round(nbytes / ms / 1e9, 2)}), flush=True)
        # fp8 cache, 8-row tiles with the keys on the MMA's row side (3 stages, four CTAs per
        # SM, or 2 stages, five)
        ws8, wr8 = A.build_work(q_lens, hq // hkv, 8)
        ws8, wr8 = torch.tensor(ws8, **i32), torch.tensor(wr8, **i32)
        for st8 in (3, 2):
            old = _native.native().attn_fp8t_stages(st8)
            ms = _time_flushed(lambda: A.paged_attention(q, k8, v8, bt, qs, kvl, ws8, wr8, 8, hq, 0.088, out, ns,
                                                         wso, wsl, k_scale=ks, v_scale=vs), args.iters, flush)
            _native.native().attn_fp8t_stages(old)
            nbytes = 2 * sum(kv_lens) * hkv * d
            print(json.dumps({"case": "decode_split", "cache": "fp8", "rows": 8, "stages": st8, "nsplit": ns,
                              "ms": round(ms, 4), "kv_tbs": round(nbytes / ms / 1e9, 2)}), flush=True)
    if args.library:
        A.paged_attention(q, kc, vc, bt, qs, kvl, ws, wr, 16, hq, 0.088, out, 1)
        _library_decode(q, kc, vc, bt, kv_lens, hq, d, out, 2 * sum(kv_lens) * hkv * d * 2, args.iters, flush)
    _native.check_errors(torch.device("cuda", 0))


_WORKSPACE = None


def _workspace():
    global _WORKSPACE
    if _WORKSPACE is None:
        _WORKSPACE = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")
    return _WORKSPACE


def _library_decode(q, kc, vc, bt, kv_lens, hq, d, ours, kv_bytes, iters, flush):
    """FlashInfer trtllm-gen paged decode over the same bf16 pages ([pages, Hkv, 16, D], its
    HND layout), L2 flushed before each launch like ``decode_split``."""
    try:
        from flashinfer.decode import trtllm_batch_decode_with_kv_cache

        b = len(kv_lens)
        qq = q[:, :hq * d].reshape(b, hq, d).contiguous()
        seq = torch.tensor(kv_lens, dtype=torch.int32, device="cuda")
        out = torch.empty(b, hq, d, dtype=torch.bfloat16, device="cuda")

        def run():
            trtllm_batch_decode_with_kv_cache(qq, (kc, vc), _workspace(), bt, seq, max(kv_lens), bmm1_scale=0.088,
                                              bmm2_scale=1.0, out=out, kv_layout="HND")

        ms = _time_flushed(run, iters, flush)
        diff = (out.reshape(b, hq * d).float() - ours[:b].float()).abs().max().item()
        print(json.dumps({"case": "decode_split", "cache": "bf16", "impl": "flashinfer-trtllm-gen",
                          "ms": round(ms, 4), "kv_tbs": round(kv_bytes / ms / 1e9, 2),
                          "max_abs_diff_vs_native": round(diff, 4)}), flush=True)
    except Exception as e:  # the library is optional: report, do not fail the sweep
        print(json.dumps({"case": "decode_split", "impl": "flashinfer-trtllm-gen",
                          "unavailable": f"{type(e).__name__}: {e}"[:300]}), flush=True)


def _library_prefill(name, q, kc, vc, bt, q_lens, kv_lens, hq, d, ours, flops, iters):
    """FlashInfer trtllm-gen paged causal context attention on the same pages and queries."""
    try:
        from flashinfer.prefill import trtllm_batch_context_with_kv_cache

        t = sum(q_lens)
        qq = q[:, :hq * d].reshape(t, hq, d).contiguous()
        i32 = dict(dtype=torch.int32, device="cuda")
        cq, ck = [0], [0]
        for ql, kl in zip(q_lens, kv_lens):
            cq.append(cq[-1] + ql)
            ck.append(ck[-1] + kl)
        seq = torch.tensor(kv_lens, **i32)
        cq, ck = torch.tensor(cq, **i32), torch.tensor(ck, **i32)
        out = torch.empty(t, hq, d, dtype=torch.bfloat16, device="cuda")

        def run():
            trtllm_batch_context_with_kv_cache(qq, (kc, vc), _workspace(), bt, seq, max(q_lens), max(kv_lens), 0.088,
                                               1.0, len(q_lens), cq, ck, out=out, kv_layout="HND", causal=True)

        ms = _time(run, iters)
        # this package's output of the last timed configuration holds the same values
        diff = (out.reshape(t, hq * d).float() - ours[:t].float()).abs().max().item()
        print(json.dumps({"case": name, "impl": "flashinfer-trtllm-gen", "ms": round(ms, 4),
                          "tflops": round(flops / ms / 1e9, 1), "max_abs_diff_vs_native": round(diff, 4)}),
              flush=True)
    except Exception as e:
        print(json.dumps({"case": name, "impl": "flashinfer-trtllm-gen",
                          "unavailable": f"{type(e).__name__}: {e}"[:300]}), flush=True)


if __name__ == "__main__":
    main()
