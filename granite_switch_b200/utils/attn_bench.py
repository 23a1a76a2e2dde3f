"""Attention kernel timing (CUDA events, after warm-up) on the benchmark model's head shape.

``python -m granite_switch_b200.utils.attn_bench [--iters 20]`` prints one JSON
line per case: tcgen05 prefill attention on a fresh causal 4k prompt and on 8
chunks of 512 new tokens over 3.5k cached tokens (TFLOP/s, causal FLOPs
counted once), and decode attention for 128 requests x 4.2k cached tokens
(GB/s of K/V read). 32 query / 8 KV heads, head_dim 128 (Granite-8B shape).
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


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--iters", type=int, default=20)
    args = p.parse_args()
    _native.native()
    hq, hkv, d = 32, 8, 128
    i32 = dict(dtype=torch.int32, device="cuda")
    for name, q_lens, kv_lens in (("prefill_causal_4k", [4096], [4096]),
                                  ("prefill_8x512_over_3584", [512] * 8, [4096] * 8)):
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
    _native.check_errors(torch.device("cuda", 0))


if __name__ == "__main__":
    main()
