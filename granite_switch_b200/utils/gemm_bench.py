"""Switched-LoRA GEMM microbenchmark (the kernel sweep of the benchmark configs).

``python -m granite_switch_b200.utils.gemm_bench [--quick] [--pair-min-m M]``, or
``--decode M ...`` for the decode-sized 8B projections (:func:`decode_sweep`).

For every point (M tokens, N x K, rank r, number of adapters) the per-token
adapter ids are drawn uniformly over the adapters, then an activation mask
sends every token before a uniformly drawn invocation start to the base model
(id 0), as activated LoRA does. Timed per point, with CUDA events after
warm-up and an L2 flush (a 256 MB write) before every launch:

* ``native``  - LoRA shrink + tcgen05 switched GEMM with the expand fused in
  the mainloop (what a projection costs in the engine),
* ``base``    - the same tcgen05 GEMM with no adapters,
* ``cublas``  - ``torch.matmul`` of the base weight (the library bar).

With ``--fp8`` (block-scaled e4m3 base weight, 1x128 activation and 128x128
weight scales, LoRA in bf16; :mod:`ops.gemm_fp8`):

* ``fp8_native`` - activation quantiser + bf16 LoRA shrink + fp8 GEMM with the
  bf16 expand fused (what an fp8 projection costs),
* ``fp8_base``   - the fp8 GEMM alone on pre-quantised operands, no adapters.

With ``--reference`` the reference's own switched projection runs beside them
(``reference``): one cuBLAS GEMM of ``x`` against ``[W; A_1..A_n]`` and the
reference's Triton expand kernel (``switch_lora_expand`` from the installed
reference package, reference: src/granite_switch/vllm/core/lora.py:540-566 and
src/granite_switch/kernels/switch_lora_kernel.py:414-458), with its kernel
metadata (kernel-local ids, 32-row tile bitmasks, per-slice shrink columns, rank
tiers 16..512, rank 8 promoted to 16) built here as its layer builds it.

TFLOP/s count the base product only (2 M N K), so the columns compare
directly. One JSON line per point on stdout.
"""
from __future__ import annotations

import argparse
import json

import torch

from .._native import check_errors, err_buffer, native
from ..ops import gemm as G

SHAPES = [(4096, 4096), (12800, 4096), (4096, 12800)]  # N x K
MS = [16, 256, 4096]
RANKS = [8, 32, 64]
ADAPTERS = [1, 4, 12, 32]


def _flush_buffer(dev):
    return torch.empty(256 << 20, dtype=torch.uint8, device=dev)


def time_launches(fn, flush, iters=20, warmup=3) -> float:
    """Median device time (ms) of ``fn`` over ``iters`` launches, L2 flushed before each."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def make_case(m, n, k, rank, na, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = (torch.randn(m, k, device=dev, generator=g)).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
    rp = (rank + 31) // 32 * 32  # the kernel pads ranks to multiples of 32
    ids = torch.randint(1, na + 1, (m,), device=dev, generator=g, dtype=torch.int32)
    start = int(torch.randint(0, m, (1,), generator=torch.Generator().manual_seed(seed)).item())
    ids[:start] = 0  # activated LoRA: tokens before the invocation run the base weights
    a_rows = (na * rp + 63) // 64 * 64
    a_all = torch.zeros(a_rows, k, device=dev, dtype=torch.bfloat16)
    a_all[: na * rp] = (torch.randn(na * rp, k, device=dev, generator=g) * 0.02).bfloat16()
    lb = (torch.randn(n, na * rp, device=dev, generator=g) * 0.02).bfloat16()
    tiles = (m + 127) // 128
    mask = torch.zeros(tiles, dtype=torch.int64)
    ids_h = ids.cpu()
    for t in range(tiles):
        bits = 0
        for a in ids_h[t * 128:(t + 1) * 128].unique().tolist():
            if a > 0:
                bits |= 1 << (a - 1)
        mask[t] = bits if bits < (1 << 63) else bits - (1 << 64)
    return dict(x=x, w=w, ids=ids, a_all=a_all, lb=lb, mask=mask.to(dev), rank=rp, na=na)


def _reference_kernels():
    """The reference's Triton switched-LoRA module from ``baseline/_ref`` (None if absent)."""
    import importlib
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    for base in (os.path.join(root, "baseline", "_ref"), os.path.join(root, "baseline", "_ref", "src")):
        if os.path.isfile(os.path.join(base, "granite_switch", "kernels", "switch_lora_kernel.py")):
            if base not in sys.path:
                sys.path.insert(0, base)
            return importlib.import_module("granite_switch.kernels.switch_lora_kernel")
    return None


def reference_case(c, n, k, rank, ref):
    """The reference layer's operands for one point: W_ext (base rows, then every adapter's
    A rows), the packed B of the rank tier, kernel-local ids, the 32-row tile bitmask and
    the per-slice shrink column table (one slice)."""
    r = ref.promote_rank(rank)
    na, dev = c["na"], c["x"].device
    g = torch.Generator(device=dev).manual_seed(1)
    a = (torch.randn(na, 1, r, k, device=dev, generator=g) * 0.02).bfloat16()
    w_ext = ref.build_w_ext(c["w"], {r: a})
    lb = (torch.randn(na, n, r, device=dev, generator=g) * 0.02).bfloat16().contiguous()
    ids = c["ids"].long()
    bm = ref.get_switch_lora_expand_config()["block_m"]
    tiles = (ids.shape[0] + bm - 1) // bm
    bits = torch.zeros(tiles, dtype=torch.int64)
    ids_h = ids.cpu()
    for t in range(tiles):
        v = 0
        for x in ids_h[t * bm:(t + 1) * bm].unique().tolist():
            if x > 0:
                v |= 1 << (x - 1)
        bits[t] = v if v < (1 << 63) else v - (1 << 64)
    tiers = list(ref.SUPPORTED_RANKS)
    na_t = tuple(na if t == r else 0 for t in tiers)
    col_r = torch.tensor([[n for _ in tiers]], dtype=torch.int32, device=dev)  # tier r's block starts at N
    block_n = ref.get_switch_lora_expand_config()["block_n"]
    tile_slice = torch.zeros((n + block_n - 1) // block_n, dtype=torch.int32, device=dev)
    return dict(w_ext=w_ext, lb=lb, ids=ids, bits=bits.to(dev), na=na_t, col_r=col_r, tile_slice=tile_slice,
                block_n=block_n)


def run_point(m, n, k, rank, na, flush, dev, iters=20, compare_pair=False, fp8=False, ref=None):
    c = make_case(m, n, k, rank, na, dev)
    x, w = c["x"], c["w"]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    s = torch.empty(m, max(64, c["a_all"].shape[0]), dtype=torch.bfloat16, device=dev)[:, : c["a_all"].shape[0]]

    def native_fn():
        G.lora_shrink(x, c["a_all"], c["ids"], c["rank"], c["na"], out=s, tile_mask=c["mask"])
        G.switched_gemm(x, w, out, s=s, lb=c["lb"], tile_mask=c["mask"], rank=c["rank"], num_adapters=c["na"],
                        slice_bounds=[0, n])

    def base_fn():
        G.switched_gemm(x, w, out)

    def cublas_fn():
        torch.matmul(x, w.t(), out=out)

    res = {}
    fns = [("native", native_fn, None), ("base", base_fn, None), ("cublas", cublas_fn, None)]
    if compare_pair:  # same point on the CTA-pair and the single-CTA kernel, interleaved
        fns = [("native_pair", native_fn, 1), ("native_single", native_fn, -1), ("base_pair", base_fn, 1),
               ("base_single", base_fn, -1), ("cublas", cublas_fn, None)]
    if fp8:
        from ..ops import gemm_fp8 as F

        x8, sfa = F.quantize_rows_fp8(x)
        w8, sfb = F.quantize_weight_fp8(w)

        def fp8_native_fn():
            F.quantize_rows_fp8(x, x8, sfa)
            G.lora_shrink(x, c["a_all"], c["ids"], c["rank"], c["na"], out=s, tile_mask=c["mask"])
            F.fp8_gemm(x8, sfa, w8, sfb, out, s=s, lb=c["lb"], tile_mask=c["mask"], rank=c["rank"],
                       num_adapters=c["na"])

        def fp8_base_fn():
            F.fp8_gemm(x8, sfa, w8, sfb, out)

        fns += [("fp8_native", fp8_native_fn, None), ("fp8_base", fp8_base_fn, None)]
    if ref is not None:
        rc = reference_case(c, n, k, rank, ref)
        x_ext = torch.empty(m, rc["w_ext"].shape[0], dtype=torch.bfloat16, device=dev)

        def reference_fn():
            torch.mm(x, rc["w_ext"].t(), out=x_ext)
            ref.switch_lora_expand(x_ext, rc["ids"], rc["bits"], rc["lb"], rc["tile_slice"], rc["col_r"], rc["na"],
                                   1, rc["block_n"], n)

        fns.append(("reference", reference_fn, None))
    nat = native()
    for name, fn, pair in fns:
        old = nat.gemm_pair_min_m(pair) if pair is not None else None
        ms = time_launches(fn, flush, iters)
        if old is not None:
            nat.gemm_pair_min_m(old)
        res[name] = dict(ms=round(ms, 4), tflops=round(2 * m * n * k / ms / 1e9, 1))
    check_errors(x.device)
    return res


DECODE_SHAPES = {  # 8B-shape projections: name -> (N, K, epilogue, LoRA on)
    "qkv": (6144, 4096, "store", True),
    "o": (4096, 4096, "resadd", True),
    "gate_up": (25600, 4096, "swiglu", False),
    "down": (4096, 12800, "resadd", False),
}


def _hbm_gbs() -> float:
    import os

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0  # earlier measurement on this pool, when the file is absent


def decode_sweep(ms, iters: int = 50, rotate_bytes: int = 400 << 20) -> None:
    """Decode-sized projections (the 8B shapes at M tokens, 12 adapters r32 where LoRA is on):
    device time per call from CUDA-graph replays of ``iters`` calls with enough weight copies rotated (``rotate_bytes`` in all, over three
    times the 126 MB L2) that every call streams its weights from HBM, the operand-swapped decode kernel against the general kernel. Prints
    microseconds and the weight bytes' fraction of the measured HBM copy bandwidth."""
    dev = torch.device("cuda", 0)
    nat = native()
    hbm = _hbm_gbs()
    na, rank = 12, 32
    for m in ms:
        for name, (n, k, epi, lora) in DECODE_SHAPES.items():
            g = torch.Generator(device=dev).manual_seed(m)
            copies = max(3, -(-rotate_bytes // (n * k * 2)))
            ws = [(torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16() for _ in range(copies)]
            x = torch.randn(m, k, device=dev, generator=g).bfloat16()
            out = torch.empty(m, n // 2 if epi == "swiglu" else n, device=dev, dtype=torch.bfloat16)
            kind = {"store": G.EPI_STORE, "resadd": G.EPI_RESADD, "swiglu": G.EPI_SWIGLU}[epi]
            extra = {}
            shrink = None
            if lora:
                slices = 3 if name == "qkv" else 1
                ids = torch.randint(1, na + 1, (m,), device=dev, dtype=torch.int32, generator=g)
                mask = torch.zeros((m + 127) // 128, dtype=torch.int64, device=dev)
                for t in range(mask.numel()):
                    bits = 0
                    for a in ids[t * 128:(t + 1) * 128].unique().tolist():
                        bits |= 1 << (a - 1)
                    mask[t] = bits
                a_all = (torch.randn(slices * na * rank, k, device=dev, generator=g) * 0.02).bfloat16()
                s = torch.empty(m, a_all.shape[0], device=dev, dtype=torch.bfloat16)
                lb = (torch.randn(n, na * rank, device=dev, generator=g) * 0.02).bfloat16()
                bounds = [0, 4096, 5120, 6144] if name == "qkv" else [0, n]
                extra = dict(s=s, lb=lb, tile_mask=mask, rank=rank, num_adapters=na, slice_bounds=bounds)

                def shrink():
                    G.lora_shrink(x, a_all, ids, rank, na, out=s, tile_mask=mask)
            res = {}
            parts = ["full", "base"] + (["shrink"] if lora else [])
            for tag, dm in (("decode", 256), ("general", 0)):
                old = nat.gemm_decode_max_m(dm)
                for what in parts:
                    i = [0]

                    def call(what=what):
                        w = ws[i[0] % copies]
                        i[0] += 1
                        if what == "shrink":
                            shrink()
                            return
                        if what == "full" and shrink is not None:
                            shrink()
                        G.switched_gemm(x, w, out, epi=kind, residual=out if epi == "resadd" else None,
                                        bn=128 if epi == "swiglu" else None, **(extra if what == "full" else {}))

                    for _ in range(5):
                        call()
                    torch.cuda.synchronize()
                    # device time only: the calls are replayed from a CUDA graph, so host
                    # launch cost (which the engine overlaps with earlier kernels) is excluded
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph):
                        for _ in range(iters):
                            call()
                    graph.replay()
                    torch.cuda.synchronize()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    graph.replay()
                    b.record()
                    torch.cuda.synchronize()
                    del graph
                    us = a.elapsed_time(b) / iters * 1e3
                    gbs = n * k * 2 / (us * 1e-6) / 1e9
                    res[f"{tag}_{what}"] = dict(us=round(us, 2), hbm_frac=round(gbs / hbm, 3))
                nat.gemm_decode_max_m(old)
            check_errors(dev)
            print(json.dumps(dict(m=m, proj=name, n=n, k=k, lora=lora, **res)), flush=True)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--decode", type=int, nargs="*", default=None,
                   help="time the decode-sized 8B projections at these M instead of the sweep")
    p.add_argument("--quick", action="store_true", help="r=32, 12 adapters only")
    p.add_argument("--ms", type=int, nargs="*", default=None)
    p.add_argument("--pair-min-m", type=int, default=None, help="smallest M of the CTA-pair kernel (<0: off)")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--compare-pair", action="store_true", help="time CTA-pair and single-CTA tiles side by side")
    p.add_argument("--fp8", action="store_true", help="also time the block-scaled fp8 GEMM")
    p.add_argument("--reference", action="store_true",
                   help="also time the reference's switched projection (cuBLAS + its Triton expand)")
    p.add_argument("--shapes", nargs="*", default=None, help="N x K pairs as NxK (default: the three 8B shapes)")
    p.add_argument("--small-shrink-max-m", type=int, default=None,
                   help="largest M whose LoRA shrink runs on CUDA cores (A/B of the crossover)")
    args = p.parse_args()
    if args.small_shrink_max_m is not None:
        G.SMALL_SHRINK_MAX_M = args.small_shrink_max_m
    dev = torch.device("cuda", 0)
    err_buffer(dev)
    if args.decode is not None:
        decode_sweep(args.decode or [222])
        return
    nat = native()
    if args.pair_min_m is not None:
        nat.gemm_pair_min_m(args.pair_min_m)
    flush = _flush_buffer(dev)
    ranks = [32] if args.quick else RANKS
    adapters = [12] if args.quick else ADAPTERS
    shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.shapes] if args.shapes else SHAPES
    ref = _reference_kernels() if args.reference else None
    if args.reference and ref is None:
        print(json.dumps({"reference": "unavailable: the reference package is not installed under baseline/_ref"}))
    for m in args.ms or MS:
        for n, k in shapes:
            for r in ranks:
                for na in adapters:
                    res = run_point(m, n, k, r, na, flush, dev, args.iters, args.compare_pair, args.fp8, ref)
                    print(json.dumps(dict(m=m, n=n, k=k, rank=r, adapters=na, **res)), flush=True)


if __name__ == "__main__":
    main()
