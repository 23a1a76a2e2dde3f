"""One launch of each native kernel on a representative shape, for profiler captures.

``python -m granite_switch_b200.utils.kernel_cases <case>`` with case in
gemm, gemm_pair, gemm_single, cublas, swiglu, attn_prefill64, moe, probe, decode_gemm, decode_shrink, lora_small, fp8_gemm,
fp8_quant, attn_prefill, attn_decode, attn_decode_fp8, attn_decode_fp8t, rmsnorm, rope, embed, routing, sample (or ``all``). Pair it with ``ncu --clock-control none -k regex:<kernel> -c 1`` (without
``--clock-control none`` ncu locks the GPU clocks).
"""
import sys

import torch

from granite_switch_b200.ops import gemm as G, elementwise as E, attention as A
from granite_switch_b200._native import native, err_buffer, check_errors
from granite_switch_b200.ops.routing import route_device
from granite_switch_b200.routing.scan import expert_table
from granite_switch_b200.engine.sampling import sample
from granite_switch_b200.engine.request import SamplingParams, Request
dev = "cuda"
torch.manual_seed(0)
err_buffer(torch.device(dev))
which = sys.argv[1] if len(sys.argv) > 1 else "all"
def want(n): return which in ("all", n)
H, I, T = 4096, 12800, 4096
if want("gemm"):  # qkv-shape prefill GEMM with fused LoRA expand (12 adapters r32, 3 slices)
    x = torch.randn(T, H, device=dev).bfloat16()
    w = (torch.randn(6144, H, device=dev) * 0.02).bfloat16()
    na, r = 12, 32
    ra = torch.randint(0, na + 1, (T,), device=dev, dtype=torch.int32)
    a_all = (torch.randn(3 * na * r, H, device=dev) * 0.02).bfloat16()
    lb = (torch.randn(6144, na * r, device=dev) * 0.02).bfloat16()
    tm = torch.full(((T + 127) // 128,), (1 << na) - 1, dtype=torch.int64, device=dev)
    s = G.lora_shrink(x, a_all, ra, r, na, tile_mask=tm)
    out = G.switched_gemm(x, w, s=s, lb=lb, tile_mask=tm, rank=r, num_adapters=na, slice_bounds=[0, 4096, 5120, 6144])
if want("gemm_pair"):  # base GEMM on CTA-pair tiles (M >= 512 selects them)
    x = torch.randn(T, H, device=dev).bfloat16()
    w = (torch.randn(I, H, device=dev) * 0.02).bfloat16()
    out = G.switched_gemm(x, w, bn=256)
if want("gemm_single"):  # the same GEMM on single-CTA 128x256 tiles
    native().gemm_pair_min_m(-1)
    x = torch.randn(T, H, device=dev).bfloat16()
    w = (torch.randn(I, H, device=dev) * 0.02).bfloat16()
    out = G.switched_gemm(x, w, bn=256)
if want("cublas"):  # library bar for the same shape (torch.matmul -> cuBLAS)
    x = torch.randn(T, H, device=dev).bfloat16()
    w = (torch.randn(I, H, device=dev) * 0.02).bfloat16()
    out = torch.matmul(x, w.t())
if want("swiglu"):
    x = torch.randn(T, H, device=dev).bfloat16()
    w = (torch.randn(2 * I, H, device=dev) * 0.02).bfloat16()
    out = G.switched_gemm(x, w, epi=G.EPI_SWIGLU, bn=256)
if want("decode_gemm"):  # down projection of the headline decode step (222 tokens): the decode kernel
    w = (torch.randn(H, I, device=dev) * 0.02).bfloat16()
    x2 = torch.randn(222, I, device=dev).bfloat16()
    h = torch.randn(222, H, device=dev).bfloat16()
    G.switched_gemm(x2, w, h, epi=G.EPI_RESADD, residual=h, scale=0.5)
if want("fp8_gemm") or want("fp8_quant"):  # block-scaled fp8 GEMM, 4096 x 12800 x 4096 (and its activation quantiser)
    from granite_switch_b200.ops import gemm_fp8 as F
    xq = torch.randn(T, H, device=dev).bfloat16()
    x8, sfa = F.quantize_rows_fp8(xq)
    if want("fp8_gemm"):
        w8, sfb = F.quantize_weight_fp8((torch.randn(I, H, device=dev) * 0.02).bfloat16())
        out8 = F.fp8_gemm(x8, sfa, w8, sfb)
if want("decode_shrink"):  # LoRA shrink of o_proj in the headline decode step (222 tokens, 12 adapters r32)
    xs = torch.randn(222, H, device=dev).bfloat16()
    a_all = (torch.randn(12 * 32, H, device=dev) * 0.02).bfloat16()
    ids = torch.randint(1, 13, (222,), device=dev, dtype=torch.int32)
    s_out = torch.empty(222, 12 * 32, device=dev, dtype=torch.bfloat16)
    G.lora_shrink(xs, a_all, ids, 32, 12, out=s_out)
if want("lora_small"):  # CUDA-core LoRA shrink of qkv at a 64-token decode step (3 slices, 12 adapters r32)
    xs = torch.randn(64, H, device=dev).bfloat16()
    a_all = (torch.randn(3 * 12 * 32, H, device=dev) * 0.02).bfloat16()
    ids = torch.randint(0, 13, (64,), device=dev, dtype=torch.int32)
    s_out = torch.empty(64, 3 * 12 * 32, device=dev, dtype=torch.bfloat16)
    G.lora_shrink(xs, a_all, ids, 32, 12, out=s_out)
if want("attn_prefill") or want("attn_decode") or want("attn_decode_fp8") or want("attn_decode_fp8t"):
    hq, hkv, d = 32, 8, 128
    def setup(q_lens, kv_lens):
        nblk = sum((l + 15)//16 for l in kv_lens) + 4
        kc = torch.randn(nblk, hkv, 16, d, device=dev).bfloat16(); vc = torch.randn_like(kc)
        maxb = max((l+15)//16 for l in kv_lens)
        bt = torch.arange(nblk, dtype=torch.int32)[: len(kv_lens) * maxb].view(len(kv_lens), maxb) if nblk >= len(kv_lens)*maxb else None
        bt = torch.zeros(len(kv_lens), maxb, dtype=torch.int32); p = 0
        for i, l in enumerate(kv_lens):
            for j in range((l+15)//16): bt[i, j] = p; p += 1
        Tq = sum(q_lens)
        q = torch.randn(Tq, (hq+2*hkv)*d, device=dev).bfloat16()
        out = torch.empty(Tq, hq*d, device=dev).bfloat16()
        qs = [0]
        for l in q_lens: qs.append(qs[-1]+l)
        return kc, vc, bt.to(dev), q, out, torch.tensor(qs, dtype=torch.int32, device=dev), torch.tensor(kv_lens, dtype=torch.int32, device=dev)
    if want("attn_prefill"):
        q_lens = [4096]; kc, vc, bt, q, out, qs, kvl = setup(q_lens, q_lens)
        ws, wr = [torch.tensor(v, dtype=torch.int32, device=dev) for v in A.build_work(q_lens, 4, 128)]
        A.prefill_attention_tc(q, kc, vc, bt, qs, kvl, ws, wr, hq, 0.088, out)
    if want("attn_decode"):
        q_lens = [1] * 128; kv = [4200] * 128; kc, vc, bt, q, out, qs, kvl = setup(q_lens, kv)
        ws, wr = [torch.tensor(v, dtype=torch.int32, device=dev) for v in A.build_work(q_lens, 4, 16)]
        A.paged_attention(q, kc, vc, bt, qs, kvl, ws, wr, 16, hq, 0.088, out, 1)
    if want("attn_decode_fp8"):  # the same decode step over the fp8 (e4m3) cache
        q_lens = [1] * 128; kv = [4200] * 128; kc, vc, bt, q, out, qs, kvl = setup(q_lens, kv)
        k8 = torch.randint(0, 126, kc.shape, dtype=torch.uint8, device=dev)  # finite e4m3 bytes
        v8 = torch.randint(0, 126, (kc.shape[0], hkv, d, 16), dtype=torch.uint8, device=dev)
        ks = torch.full(kc.shape[:3], 0.01, device=dev); vs = torch.full_like(ks, 0.01)
        ws, wr = [torch.tensor(v, dtype=torch.int32, device=dev) for v in A.build_work(q_lens, 4, 16)]
        A.paged_attention(q, k8, v8, bt, qs, kvl, ws, wr, 16, hq, 0.088, out, 1, k_scale=ks, v_scale=vs)
    if want("attn_decode_fp8t"):  # the same over the fp8 cache with 8-row tiles (keys on the MMA's row side)
        q_lens = [1] * 128; kv = [4200] * 128; kc, vc, bt, q, out, qs, kvl = setup(q_lens, kv)
        k8 = torch.randint(0, 126, kc.shape, dtype=torch.uint8, device=dev)
        v8 = torch.randint(0, 126, (kc.shape[0], hkv, d, 16), dtype=torch.uint8, device=dev)
        ks = torch.full(kc.shape[:3], 0.01, device=dev); vs = torch.full_like(ks, 0.01)
        ws, wr = [torch.tensor(v, dtype=torch.int32, device=dev) for v in A.build_work(q_lens, 4, 8)]
        A.paged_attention(q, k8, v8, bt, qs, kvl, ws, wr, 8, hq, 0.088, out, 1, k_scale=ks, v_scale=vs)
if want("attn_prefill64"):  # tcgen05 prefill attention, head_dim 64 (3B shape: 32 q / 8 kv heads)
    hq, hkv, d = 32, 8, 64
    q_lens = [2048, 2048]
    nblk = sum((l + 15) // 16 for l in q_lens) + 4
    kc = torch.randn(nblk, hkv, 16, d, device=dev).bfloat16(); vc = torch.randn_like(kc)
    bt = torch.arange(nblk - 4, dtype=torch.int32, device=dev).view(len(q_lens), -1)
    q = torch.randn(sum(q_lens), (hq + 2 * hkv) * d, device=dev).bfloat16()
    out = torch.empty(sum(q_lens), hq * d, device=dev).bfloat16()
    qs = torch.tensor([0, 2048, 4096], dtype=torch.int32, device=dev)
    ws, wr = [torch.tensor(v, dtype=torch.int32, device=dev) for v in A.build_work(q_lens, 4, 128, q_lens)]
    A.prefill_attention_tc(q, kc, vc, bt, qs, torch.tensor(q_lens, dtype=torch.int32, device=dev), ws, wr, hq,
                           0.125, out)
if want("moe"):  # expert bank: 8192 tokens, 40 experts top-8, H 1536, expert FFN 512
    Hm, Im, Em, Km, Tm = 1536, 512, 40, 8, 8192
    from granite_switch_b200.models.packing import pack_moe
    moe = pack_moe((torch.randn(Em, 2 * Im, Hm) * 0.02).bfloat16(), (torch.randn(Em, Hm, Im) * 0.02).bfloat16(),
                   torch.randn(Em, Hm).bfloat16(), Km, dev)
    x = torch.randn(Tm, Hm, device=dev).bfloat16()
    pmax = (Tm * Km + 127 * Em + 127) // 128 * 128
    logits = torch.empty(Tm, moe.router.shape[0], device=dev)
    ids = torch.empty(Tm * Km, dtype=torch.int32, device=dev); wts = torch.empty(Tm * Km, device=dev)
    cnt = torch.zeros(Em, dtype=torch.int32, device=dev); off = torch.empty_like(cnt); cur = torch.empty_like(cnt)
    tiles = torch.empty(pmax // 128, dtype=torch.int32, device=dev); slot = torch.empty_like(ids)
    xp = torch.zeros(pmax, Hm, device=dev).bfloat16(); ap = torch.zeros(pmax, Im, device=dev).bfloat16()
    yp = torch.zeros(pmax, Hm, device=dev).bfloat16(); h = torch.randn(Tm, Hm, device=dev).bfloat16()
    G.switched_gemm(x, moe.router, logits, epi=G.EPI_F32)
    native().moe_route(logits, Em, Km, ids, wts, cnt, off, cur, tiles)
    native().moe_scatter(x, ids, off, cur, slot, xp)
    G.switched_gemm(xp, moe.gate_up, ap, epi=G.EPI_SWIGLU, bn=moe.swiglu_tile, tile_expert=tiles)
    G.switched_gemm(ap, moe.down, yp, tile_expert=tiles)
    native().moe_combine(yp, slot, wts, Km, None, h, 1.0, h)
if want("probe"):
    hid = torch.randn(4096, H, device=dev).bfloat16()
    pw = torch.randn(4, 8, H, device=dev).bfloat16(); pb = torch.randn(4, 8, device=dev)
    rows = torch.arange(0, 4096, 32, dtype=torch.int32, device=dev); n = rows.numel()
    slots = (torch.arange(n, dtype=torch.int32, device=dev) % 4) + 1; outj = torch.arange(n, dtype=torch.int32, device=dev)
    verdict = torch.zeros(n, 8, device=dev); logits = torch.randn(n, 49152, device=dev)
    labels = torch.randint(0, 49152, (4, 8), dtype=torch.int32, device=dev)
    native().probe_verdict(hid, rows, slots, outj, pw, pb, verdict)
    native().probe_rewrite(logits, 0, outj, slots, labels, verdict)
if want("rmsnorm"):
    x = torch.randn(16384, H, device=dev).bfloat16(); w = torch.ones(H, device=dev).bfloat16()
    E.rmsnorm(x, w, 1e-5)
if want("rope"):
    cs = E.rope_cos_sin_table(8192, 128, 1e4, dev)
    qkv = torch.randn(8192, 48 * 128, device=dev).bfloat16(); pos = torch.arange(8192, device=dev)
    kc = torch.zeros(512, 8, 16, 128, device=dev).bfloat16(); vc = torch.zeros_like(kc)
    E.rope_kv(qkv, pos, cs, 32, 8, 128, kc, vc, torch.arange(8192, device=dev))
if want("embed"):
    tab = torch.randn(49164, H, device=dev).bfloat16(); ids = torch.randint(0, 49164, (8192,), device=dev)
    E.embed(ids, tab, None, 12.0)
if want("routing"):
    tbl = expert_table(list(range(49152, 49164)), 12, 49164).to(dev)
    T2 = 8192; ids = torch.randint(0, 49164, (T2,), device=dev)
    starts = torch.arange(0, T2 + 1, 64, dtype=torch.int32, device=dev); S = starts.numel() - 1
    remap = torch.arange(13, dtype=torch.int32, device=dev).view(1, 13)
    route_device(ids, starts, torch.zeros(S, dtype=torch.int32, device=dev), tbl, None, None, 12, remap,
                 torch.empty(T2, dtype=torch.int32, device=dev), torch.empty(T2, dtype=torch.int32, device=dev),
                 torch.empty(T2, dtype=torch.long, device=dev), torch.empty(S, dtype=torch.int32, device=dev),
                 torch.empty(1, T2, dtype=torch.int32, device=dev), torch.empty(1, (T2 + 127)//128, dtype=torch.int64, device=dev))
if want("sample"):
    logits = torch.randn(128, 49164, device=dev)
    reqs = [Request([1]) for _ in range(128)]
    sample(logits, [SamplingParams(temperature=0.8, top_k=50, top_p=0.9, seed=i) for i in range(128)], reqs)
    E.argmax(logits)
torch.cuda.synchronize()
check_errors(torch.device(dev))
print("ok", which)
