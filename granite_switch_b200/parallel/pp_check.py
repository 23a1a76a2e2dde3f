"""Pipeline-parallel self-check: PP (x TP) logits against one GPU on the same random model.

Run under torchrun, one process per GPU::

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m granite_switch_b200.parallel.pp_check [--tp 1]

World = tp * pp. Every rank builds the same seeded random model and keeps its
stage's layers (and its TP shard); three engine steps (a prefill step and two
decode steps, greedy, each split into two micro-batches) run through the
native executor, the last stage's TP
rank 0 gathers the logits and compares them with the unsharded model run
alone on its GPU. Prints one JSON line and exits non-zero on a mismatch.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def _run(config, device, steps_out, tp_rank=0, tp=1, tp_group=None, pipeline=None):
    from ..engine.executor import NativeExecutor
    from ..engine.kv_cache import BlockManager
    from ..engine.llm_engine import HostRouter
    from ..engine.request import Request, SamplingParams
    from ..engine.scheduler import Scheduler
    from ..models.native import NativeGraniteSwitch

    m = NativeGraniteSwitch.from_random(config, device, max_tokens=512, num_kv_blocks=256,
                                        lora_modules=("qkv", "o"), rank=16, seed=7, tp_rank=tp_rank, tp_size=tp,
                                        tp_group=tp_group, max_seqs=16, pipeline=pipeline)
    ex = NativeExecutor(m, 1024, tp_group, tp)
    ex.PP_SPLIT_MIN_TOKENS = 0  # the check's steps are small: split them all into micro-batches
    bm = BlockManager(256)
    router = HostRouter(config)
    sch = Scheduler(bm, 8, 512, True, route_fn=router)
    g = torch.Generator().manual_seed(3)
    ctrl = config.adapter_token_ids
    for i in range(3):
        ids = torch.randint(5, 2000, (40 + 17 * i,), generator=g).tolist() + [ctrl[i], 9, 10]
        sch.add(Request(ids, SamplingParams(max_tokens=3)))
    logits_seen = []
    for _ in range(3):
        out = sch.schedule()
        hb, logits = ex.compute_logits(out)
        if logits is not None:
            logits_seen.append(logits.float().cpu())
        toks = ex.d_tokens[0, : len(hb.rows)]
        if logits is not None:
            toks.copy_(logits.argmax(dim=-1))
        if pipeline is not None:
            pipeline.broadcast_tokens(toks)
        toks = toks.tolist()
        j = 0
        for c in out.chunks:
            r = c.req
            r.carry = router(r.all_ids[c.start:c.start + c.num_tokens], r.carry)
            r.num_computed = c.start + c.num_tokens
            if c.needs_sample:
                r.output_ids.append(toks[j])
                j += 1
    steps_out.extend(logits_seen)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    args = ap.parse_args()
    from .._native import read_errors
    from .pipeline import init_parallel_groups
    from .tp_check import _config

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    tp = args.tp
    pp = world // tp
    tp_rank, tp_group, pipe = init_parallel_groups(tp, pp)
    config = _config()
    got = []
    _run(config, device, got, tp_rank, tp, tp_group, pipe)
    errs = read_errors(device)
    dist.barrier()
    ok = True
    if pipe.rank == pipe.size - 1 and tp_rank == 0:
        ref = []
        _run(config, device, ref)
        worst = max(((a - b).abs().max() / b.abs().max()).item() for a, b in zip(got, ref))
        agree = sum(int((a.argmax(-1) == b.argmax(-1)).sum()) for a, b in zip(got, ref))
        total = sum(b.shape[0] for b in ref)
        ok = worst < 0.05 and agree >= total - 1 and errs == 0 and len(got) == len(ref) == 3
        print(json.dumps({"pp": pp, "tp": tp, "max_rel_err": round(worst, 5), "argmax_agree": agree,
                          "rows": total, "device_errors": errs, "ok": ok}), flush=True)
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(flag.item()) else 1


if __name__ == "__main__":
    sys.exit(main())
