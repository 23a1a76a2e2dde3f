"""Fused tensor-parallel collective-GEMM sweep (run under torchrun, one process per GPU).

``torchrun --nproc-per-node N --master-addr 127.0.0.1 -m granite_switch_b200.parallel.tp_sweep``

For d_model 4096 and FFN 12800 sharded over N ranks, and tokens M in
{8, 64, 512, 8192}, two row-parallel projections are timed:

* ``o``    M x 4096 <- M x (4096/N) . (4096/N) x 4096, reduced over ranks
* ``down`` M x 4096 <- M x (12800/N) . (12800/N) x 4096, reduced over ranks

each as

* ``fused``    the tcgen05 switched GEMM whose epilogue adds every output
  tile into a symmetric buffer through its NVLink multicast address
  (``multimem.red``; the NVSwitch sums the partials and every rank's copy
  receives the total), then the bounded peer barrier;
* ``fused_ar`` the GEMM stores its partial to the local symmetric buffer,
  then (between two barriers) every rank sums a 1/N slice of rows through
  the switch (``multimem.ld_reduce``) and multicasts it (``multimem.st``);
* ``baseline`` cuBLAS (``torch.matmul``) followed by an NCCL all-reduce, the
  path the reference serves with.

``+col`` variants append the next column-parallel GEMM (M x 4096 ->
M x 6144/N, the qkv shape): the fused path reads the replicated reduced
output from local memory (the all-gather happened inside the switch), the
baseline runs cuBLAS after its all-reduce.

Timing: CUDA events around ``--iters`` back-to-back launches after warm-up,
max over ranks. Roofline per point: max(FLOPs / measured bf16 peak, bytes
that must cross NVLink per GPU / 770 GB/s), with bytes = 2 (N-1)/N x M x 4096
x 2 B (a reduce-scatter plus an all-gather, per direction); the reported
``frac`` is roofline / achieved. Rank 0 prints one JSON line per point.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU on this pool
H, FFN, QKV = 4096, 12800, 6144


def _peak_tflops() -> float:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0  # earlier measurement on this pool


def _time(fn, iters, group) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier(group=group)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="*", default=[8, 64, 512, 8192])
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    from .._native import check_errors, err_buffer, native
    from ..ops import gemm as G
    from .fused import FusedTPComm

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    group = dist.group.WORLD
    err_buffer(dev)
    max_m = max(args.tokens)
    comm = FusedTPComm(group, dev, max_m, H)
    peak = _peak_tflops()
    g = torch.Generator(device=dev).manual_seed(rank)
    wq = (torch.randn(QKV // world, H, device=dev, generator=g) * 0.02).bfloat16()
    for name, k_full in (("o", H), ("down", FFN)):
        k = k_full // world
        w = (torch.randn(H, k, device=dev, generator=g) * 0.02).bfloat16()
        for m in args.tokens:
            x = torch.randn(m, k, device=dev, generator=g).bfloat16()
            h = torch.zeros(m, H, device=dev, dtype=torch.bfloat16)
            ybase = torch.empty(m, H, device=dev, dtype=torch.bfloat16)
            qkv = torch.empty(m, QKV // world, device=dev, dtype=torch.bfloat16)

            def fused(col=False):
                b = comm.turn
                comm.turn ^= 1
                y = comm.y[b, :m]
                mc = comm.mc + b * comm.max_tokens * comm.hidden * 2
                G.switched_gemm(x, w, y, epi=G.EPI_MULTIMEM_RED, scale=1.0, mc_out=mc)
                comm.barrier()
                if col:
                    G.switched_gemm(y, wq, qkv)
                y.zero_()  # the consumer clears the buffer before its next use

            def baseline(col=False):
                torch.matmul(x, w.t(), out=ybase)
                dist.all_reduce(ybase, group=group)
                if col:
                    torch.matmul(ybase, wq.t(), out=qkv)

            flops = 2.0 * m * k * H
            bytes_link = 2.0 * (world - 1) / world * m * H * 2
            res = {}
            for tag, fn in (("fused", lambda: fused()), ("baseline", lambda: baseline()),
                            ("fused+col", lambda: fused(True)), ("baseline+col", lambda: baseline(True))):
                ms = _time(fn, args.iters, group)
                fl = flops + (2.0 * m * H * (QKV // world) if tag.endswith("+col") else 0.0)
                roof_ms = max(fl / (peak * 1e9), bytes_link / (LINK_GBS * 1e6))
                res[tag] = dict(ms=round(ms, 4), frac=round(roof_ms / ms, 3))
            check_errors(dev)
            if rank == 0:
                print(json.dumps(dict(op=name, tp=world, tokens=m, k_per_rank=k, roofline_bound=(
                    "compute" if flops / (peak * 1e9) > bytes_link / (LINK_GBS * 1e6) else "nvlink"), **res)),
                    flush=True)
    dist.barrier(group=group)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
