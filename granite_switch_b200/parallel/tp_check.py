"""Tensor-parallel self-check: TP=N logits (NCCL and fused) against TP=1 on the same random model.

Run under torchrun, one process per GPU::

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m granite_switch_b200.parallel.tp_check

Every rank builds the same seeded random model, keeps its shard, runs one
prefill step and two decode steps through the native executor, and gathers
the logits: over NCCL, with the fused reductions, and with every fused
reduction on the large-step path. Rank 0 also builds the unsharded model alone and compares. With
``--engine`` every rank also serves prompts through the engine with pipelined and with blocking
steps (NCCL and fused reductions) and requires identical greedy tokens. Prints one JSON line per
checked mode on rank 0 and exits non-zero on a mismatch.
"""
from __future__ import annotations

import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def _config():
    from ..composer.synthetic import base_config
    from ..config import GraniteSwitchConfig

    base = base_config(dict(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                            num_attention_heads=8, num_key_value_heads=4, head_dim=128, rope_theta=10000.0))
    na = 4
    v = base["vocab_size"]
    cfg = dict(base)
    cfg.update(num_adapters=na, adapter_token_ids=list(range(v, v + na)), adapter_substitute_token_ids=[1] * na,
               adapter_ranks=[16] * na, max_lora_rank=16, lora_target_modules=["qkv_proj", "o_proj"],
               num_hidden_layers=base["num_hidden_layers"] + 2, vocab_size=v + na)
    return GraniteSwitchConfig(**cfg)


def _run(config, device, tp, rank, group, fused, red_max_tokens=None, lora=("qkv", "o")):
    from ..engine import EngineConfig
    from ..engine.executor import NativeExecutor
    from ..engine.kv_cache import BlockManager
    from ..engine.llm_engine import HostRouter
    from ..engine.request import Request, SamplingParams
    from ..engine.scheduler import Scheduler
    from ..models.native import NativeGraniteSwitch

    m = NativeGraniteSwitch.from_random(config, device, max_tokens=512, num_kv_blocks=256,
                                        lora_modules=lora, rank=16, seed=7, tp_rank=rank, tp_size=tp,
                                        tp_group=group, max_seqs=16)
    if fused:
        from .fused import attach_fused_comm

        if not attach_fused_comm(m, group):
            return None
        if red_max_tokens is not None:
            m.comm.red_max_tokens = red_max_tokens
    ex = NativeExecutor(m, 1024, group, tp)
    bm = BlockManager(256)
    router = HostRouter(config)
    sch = Scheduler(bm, 8, 512, True, route_fn=router)
    g = torch.Generator().manual_seed(3)
    ctrl = config.adapter_token_ids
    for i in range(3):
        ids = torch.randint(5, 2000, (40 + 17 * i,), generator=g).tolist() + [ctrl[i], 9, 10]
        sch.add(Request(ids, SamplingParams(max_tokens=3)))
    outs = []
    for _ in range(3):
        out = sch.schedule()
        _, logits = ex.compute_logits(out)
        outs.append(logits.float().cpu())
        toks = logits.argmax(dim=-1).tolist()
        j = 0
        for c in out.chunks:
            r = c.req
            r.carry = router(r.all_ids[c.start:c.start + c.num_tokens], r.carry)
            r.num_computed = c.start + c.num_tokens
            if c.needs_sample:
                r.output_ids.append(toks[j])
                j += 1
    from .._native import read_errors

    errs = read_errors(device)
    return outs, errs


def _check_primitives(device, group, rank, world) -> dict:
    """Each fused-collective primitive against an NCCL all-reduce of the same data."""
    from .._native import native
    from ..ops import gemm as G
    from .fused import FusedTPComm

    m, h, k = 200, 512, 256
    comm = FusedTPComm(group, device, m, h)
    out = {}
    g = torch.Generator(device=device).manual_seed(11 + rank)
    x = torch.randn(m, k, device=device, generator=g).bfloat16()
    w = (torch.randn(h, k, device=device, generator=g) * 0.05).bfloat16()
    part = G.switched_gemm(x, w)
    want = part.clone()
    dist.all_reduce(want, group=group)
    mc0 = comm.mc
    y = comm.y[0, :m]
    y.zero_()
    torch.cuda.synchronize()
    dist.barrier(group=group)
    G.switched_gemm(x, w, y, epi=G.EPI_MULTIMEM_RED, mc_out=mc0)
    comm.barrier()
    torch.cuda.synchronize()
    out["gemm_multimem_red"] = round(((y.float() - want.float()).abs().max() / want.float().abs().max()).item(), 5)
    # the model's sequence: three projections back to back through row_parallel + finish
    # (alternating buffers, rank 0 folds in the residual), no host synchronisation
    class _M:
        def _proj(self, pl, xx, yy, epi=G.EPI_STORE, residual=None, scale=1.0, mc_out=0):
            return G.switched_gemm(xx, pl, yy, epi=epi, residual=residual, scale=scale, mc_out=mc_out)

    for red in (10 ** 6, 0):
        comm.red_max_tokens = red
        hres = torch.randn(m, h, device=device, generator=torch.Generator(device=device).manual_seed(5)).bfloat16()
        nw = torch.ones(h, device=device, dtype=torch.bfloat16)
        xs = [torch.randn(m, k, device=device, generator=g).bfloat16() for _ in range(3)]
        hh, xx = hres.clone(), torch.empty(m, h, device=device, dtype=torch.bfloat16)
        ref = hres.clone()
        for xi in xs:
            y = comm.row_parallel(_M(), w, xi, hh, 0.5)
            comm.finish(y, hh, nw, xx, 1e-5)
        for xi in xs:
            p = G.switched_gemm(xi, w, scale=0.5)
            dist.all_reduce(p, group=group)
            ref = (ref.float() + p.float()).bfloat16()
        torch.cuda.synchronize()
        err = ((hh.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
        out["row_parallel_" + ("red" if red else "allreduce")] = round(err, 5)
    return out


def _engine_tokens(config, device, world, rank, group, async_on: bool, fused: bool, lora,
                   graphs: bool = False) -> tuple[list[list[int]], int]:
    """Greedy tokens of the serving engine (``LLM``) on this rank's shard: chunked prefill,
    decode rows and, with ``async_on``, pipelined steps whose decode inputs are fed back on
    the device; with ``graphs``, decode-only steps replayed from CUDA graphs where the
    engine captures them (fused reductions). Returns the tokens and the graph replays (-1
    when the fused reductions could not be attached)."""
    from ..engine import LLM, EngineConfig, SamplingParams

    ecfg = EngineConfig(max_num_seqs=8, max_num_batched_tokens=96, num_kv_blocks=256, max_model_len=512,
                        tensor_parallel_size=world, fused_tp_comm=fused, async_scheduling=async_on,
                        use_cuda_graphs=graphs)
    llm = LLM(config, device=str(device), engine_config=ecfg,
              random_init=dict(lora_modules=lora, rank=16, seed=7), tp_rank=rank, tp_group=group)
    assert llm.engine.async_steps == async_on
    g = torch.Generator().manual_seed(5)
    v = config.vocab_size - config.num_adapters
    prompts = []
    for i in range(8):
        n = int(torch.randint(20, 120, (1,), generator=g))
        ids = torch.randint(5, v, (n,), generator=g).tolist()
        ids.insert(n // 2, config.adapter_token_ids[i % config.num_adapters])
        prompts.append(ids)
    outs = llm.generate(prompts, SamplingParams(max_tokens=10))
    replays = int(getattr(llm.engine.executor, "graph_replays", 0))
    fused_on = getattr(llm.model, "comm", None) is not None
    return [o.output_ids for o in outs], (replays if fused_on else -1)


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--lora", default="qkv,o", help="comma-separated LoRA modules of the check model")
    ap.add_argument("--engine", action="store_true",
                    help="also compare the serving engine's pipelined steps with blocking steps (greedy tokens)")
    args = ap.parse_args(argv)
    lora = tuple(x for x in args.lora.split(",") if x)
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    group = dist.group.WORLD
    config = _config()
    prim = _check_primitives(device, group, rank, world)
    if rank == 0:
        print(json.dumps({"primitives": prim}), flush=True)
    dist.barrier()
    results = {}
    nccl = _run(config, device, world, rank, group, fused=False, lora=lora)
    results["nccl"] = nccl
    dist.barrier()
    fused = _run(config, device, world, rank, group, fused=True, lora=lora)
    results["fused"] = fused
    dist.barrier()
    # every reduction on the large-step path (partial stored, NCCL all-reduce)
    results["fused_allreduce"] = _run(config, device, world, rank, group, fused=True, red_max_tokens=0, lora=lora)
    dist.barrier()
    ok = True
    if rank == 0:
        ref, _ = _run(config, device, 1, 0, None, fused=False, lora=lora)
        for mode, res in results.items():
            if res is None:
                print(json.dumps({"mode": mode, "skipped": "no NVLS multicast support"}), flush=True)
                continue
            outs, errs = res
            worst = max(((a - b).abs().max() / b.abs().max()).item() for a, b in zip(outs, ref))
            agree = sum(int((a.argmax(-1) == b.argmax(-1)).sum()) for a, b in zip(outs, ref))
            total = sum(b.shape[0] for b in ref)
            good = worst < 0.05 and agree >= total - 1 and errs == 0
            ok &= good
            print(json.dumps({"mode": mode, "tp": world, "max_rel_err": round(worst, 5), "argmax_agree": agree,
                              "rows": total, "device_errors": errs, "ok": good}), flush=True)
    if args.engine:
        for fused in (False, True):
            # blocking, eager steps vs pipelined steps with decode graphs (captured only
            # when every reduction is fused: with NCCL reductions the second run is eager too)
            sync_t, _ = _engine_tokens(config, device, world, rank, group, False, fused, lora, graphs=False)
            dist.barrier()
            async_t, replays = _engine_tokens(config, device, world, rank, group, True, fused, lora, graphs=True)
            dist.barrier()
            same = sync_t == async_t and all(len(t) == 10 for t in async_t)
            if fused and replays >= 0:
                same &= replays > 0  # with the fused reductions on, decode graphs were replayed
            ok &= same
            if rank == 0:
                print(json.dumps({"mode": "engine_async_vs_sync", "tp": world, "fused": fused, "ok": same,
                                  "graph_replays": replays}),
                      flush=True)
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(flag.item()) else 1


if __name__ == "__main__":
    sys.exit(main())
