"""Native engine step (sm_100a kernels) vs the PyTorch reference executor, same schedule."""
import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200.composer.synthetic import compose_synthetic

    d = str(tmp_path_factory.mktemp("eng_gpu"))
    compose_synthetic(d, "tiny", num_adapters=3, rank=8, targets=("q", "k", "v", "o", "gate", "up", "down"),
                      seed=0, dtype=torch.float32, invocation_len=4, alpha=16.0, num_hidden_layers=2)
    return d


def _prompts(d, n, seed=0):
    idx = json.load(open(os.path.join(d, "adapter_index.json")))
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        L = int(torch.randint(20, 200, (1,), generator=g))
        ids = torch.randint(0, 1000, (L,), generator=g).tolist()
        a = i % 3
        inv = idx["adapters"][a]["invocation_token_ids"]
        ids += [idx["adapters"][a]["control_token"]["id"]] + inv[1:]
        out.append(ids)
    return out


@pytest.mark.parametrize("budget", [48, 2048])
def test_native_step_logits_match_reference(tiny_dir, budget):
    from granite_switch_b200.checkpoint import load_state_dict
    from granite_switch_b200.config import GraniteSwitchConfig
    from granite_switch_b200.engine.executor import NativeExecutor, ReferenceExecutor
    from granite_switch_b200.engine.kv_cache import BlockManager
    from granite_switch_b200.engine.llm_engine import HostRouter
    from granite_switch_b200.engine.request import Request, SamplingParams
    from granite_switch_b200.engine.scheduler import Scheduler
    from granite_switch_b200.models import GraniteSwitchForCausalLM
    from granite_switch_b200.models.native import NativeGraniteSwitch
    from granite_switch_b200._native import check_errors

    cfg = GraniteSwitchConfig.from_pretrained(tiny_dir)
    dev = torch.device("cuda")
    nb = 128
    nm = NativeGraniteSwitch.from_state_dict(cfg, load_state_dict(tiny_dir), dev, max_tokens=2048,
                                             num_kv_blocks=nb, max_seqs=16)
    nat = NativeExecutor(nm, 1024)
    ref = ReferenceExecutor(GraniteSwitchForCausalLM.from_pretrained(tiny_dir).eval(), nb)
    bm = BlockManager(nb)
    router = HostRouter(cfg)
    sch = Scheduler(bm, 8, budget, True, route_fn=router)
    reqs = [Request(p, SamplingParams(max_tokens=5)) for p in _prompts(tiny_dir, 5)]
    for r in reqs:
        sch.add(r)
    steps = 0
    worst = 0.0
    agree = total = 0
    while sch.has_work() and steps < 200:
        out = sch.schedule()
        _, ln = nat.compute_logits(out)
        _, lr = ref.compute_logits(out)
        torch.cuda.synchronize()
        j = 0
        for c in out.chunks:
            r = c.req
            r.carry = router(r.all_ids[c.start:c.start + c.num_tokens], r.carry)
            r.num_computed = c.start + c.num_tokens
            bm.register_full_blocks(r)
            if c.needs_sample:
                a, b = ln[j].float().cpu(), lr[j].float()
                worst = max(worst, ((a - b).abs().max() / b.abs().max()).item())
                tok = int(b.argmax())
                agree += int(int(a.argmax()) == tok)
                total += 1
                r.output_ids.append(tok)
                j += 1
                if len(r.output_ids) >= r.sampling.max_tokens:
                    sch.finish(r, "length")
        steps += 1
    check_errors(dev)
    assert total == 25
    assert worst < 0.05, worst
    assert agree >= total - 2


@pytest.fixture(scope="module")
def sr_dir(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200.composer.synthetic import compose_synthetic

    d = str(tmp_path_factory.mktemp("eng_gpu_sr"))
    compose_synthetic(d, "tiny", num_adapters=3, rank=8, targets=("q", "k", "v", "o", "gate", "up", "down"),
                      seed=1, dtype=torch.float32, invocation_len=4, alpha=16.0, num_hidden_layers=2,
                      cross_rank=16, std_b=0.03)
    return d


@pytest.fixture(scope="module")
def probe_dir(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200.composer.synthetic import compose_synthetic

    d = str(tmp_path_factory.mktemp("eng_gpu_probe"))
    compose_synthetic(d, "tiny", num_adapters=3, rank=8, targets=("q", "k", "v", "o"), seed=2,
                      dtype=torch.float32, invocation_len=4, alpha=16.0, num_hidden_layers=2,
                      num_probes=2, probe_read_layers=[0, None])
    return d


def _compare_engine(d, prompts, budget, max_tokens=4):
    """Native executor vs the CPU oracle on the same schedule; returns (worst rel err, agree, total, rows)."""
    from granite_switch_b200.checkpoint import load_state_dict
    from granite_switch_b200.config import GraniteSwitchConfig
    from granite_switch_b200.engine.executor import NativeExecutor, ReferenceExecutor
    from granite_switch_b200.engine.kv_cache import BlockManager
    from granite_switch_b200.engine.llm_engine import HostRouter
    from granite_switch_b200.engine.request import Request, SamplingParams
    from granite_switch_b200.engine.scheduler import Scheduler
    from granite_switch_b200.models import GraniteSwitchForCausalLM
    from granite_switch_b200.models.native import NativeGraniteSwitch
    from granite_switch_b200._native import check_errors

    cfg = GraniteSwitchConfig.from_pretrained(d)
    dev = torch.device("cuda")
    nb = 128
    nm = NativeGraniteSwitch.from_state_dict(cfg, load_state_dict(d), dev, max_tokens=2048, num_kv_blocks=nb,
                                             max_seqs=16)
    nat = NativeExecutor(nm, 1024)
    ref = ReferenceExecutor(GraniteSwitchForCausalLM.from_pretrained(d).eval(), nb)
    bm = BlockManager(nb)
    router = HostRouter(cfg)
    sch = Scheduler(bm, 8, budget, True, route_fn=router)
    for p in prompts:
        sch.add(Request(p, SamplingParams(max_tokens=max_tokens)))
    worst, agree, total, rows = 0.0, 0, 0, []
    steps = 0
    while sch.has_work() and steps < 200:
        out = sch.schedule()
        _, ln = nat.compute_logits(out)
        _, lr = ref.compute_logits(out)
        torch.cuda.synchronize()
        j = 0
        for c in out.chunks:
            r = c.req
            r.carry = router(r.all_ids[c.start:c.start + c.num_tokens], r.carry)
            r.num_computed = c.start + c.num_tokens
            bm.register_full_blocks(r)
            if c.needs_sample:
                a, b = ln[j].float().cpu(), lr[j].float()
                fin = torch.isfinite(b)
                assert torch.equal(fin, torch.isfinite(a)), "-inf pattern differs"
                worst = max(worst, ((a[fin] - b[fin]).abs().max() / b[fin].abs().max()).item())
                tok = int(b.argmax())
                agree += int(int(a.argmax()) == tok)
                total += 1
                rows.append((a, b))
                r.output_ids.append(tok)
                j += 1
                if len(r.output_ids) >= r.sampling.max_tokens:
                    sch.finish(r, "length")
        steps += 1
    check_errors(dev)
    return worst, agree, total, rows


@pytest.mark.parametrize("budget", [40, 2048])
def test_native_shadow_residual_matches_reference(sr_dir, budget):
    worst, agree, total, _ = _compare_engine(sr_dir, _prompts(sr_dir, 4, seed=3), budget)
    assert total == 16
    assert worst < 0.05, worst
    assert agree >= total - 1


def test_native_probe_verdict_matches_reference(probe_dir):
    from granite_switch_b200.config import GraniteSwitchConfig

    cfg = GraniteSwitchConfig.from_pretrained(probe_dir)
    g = torch.Generator().manual_seed(4)
    prompts = _prompts(probe_dir, 2, seed=5)
    for slot in (0, 1, 1):
        ids = torch.randint(0, 1000, (int(torch.randint(20, 90, (1,), generator=g)),), generator=g).tolist()
        prompts.append(ids + [cfg.probe_control_token_ids[slot]])
    worst, agree, total, rows = _compare_engine(probe_dir, prompts, 256, max_tokens=1)
    assert total == 5
    assert worst < 0.05, worst
    assert agree == total
    n_probe_rows = sum(1 for a, b in rows if torch.isinf(b).any())
    assert n_probe_rows == 3


def test_cuda_graph_decode_matches_eager(tiny_dir):
    """Decode steps replayed from CUDA graphs (padded batch buckets) give the eager engine's tokens."""
    from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams

    prompts = _prompts(tiny_dir, 11, seed=9)
    outs, routes = {}, {}
    for graphs in (False, True):
        ecfg = EngineConfig(max_num_seqs=16, max_num_batched_tokens=512, num_kv_blocks=256, max_model_len=512,
                            use_cuda_graphs=graphs)
        llm = LLM(tiny_dir, device="cuda:0", engine_config=ecfg)
        trace = llm.enable_routing_trace()
        res = llm.generate(prompts, SamplingParams(max_tokens=12))
        outs[graphs] = [o.output_ids for o in res]
        # the routing trace reads the static buffers, so graph replays are traced too
        routes[graphs] = [trace.of_request(o.request_id, "adapter") for o in res]
        if graphs:
            ex = llm.engine.executor
            assert ex.graph_replays > 0 and set(ex.graphs) <= {8, 16}
    assert outs[True] == outs[False]
    assert routes[True] == routes[False] and all(len(r) == len(p) + 11 for r, p in zip(routes[True], prompts))


@pytest.fixture(scope="module", params=["moe", "moe_shared", "moe_sr"])
def moe_dir(request, tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200.composer.synthetic import compose_synthetic

    d = str(tmp_path_factory.mktemp("eng_gpu_" + request.param))
    extra = dict(shared_intermediate_size=512) if request.param != "moe" else {}
    if request.param == "moe_sr":  # Shadow Residual: the adapter stream shares the base stream's routing
        extra.update(cross_rank=16, std_b=0.03)
    targets = ("q", "k", "v", "o", "gate", "up", "down") if extra else ("q", "k", "v", "o")
    compose_synthetic(d, "tiny", num_adapters=3, rank=8, targets=targets, seed=6, dtype=torch.float32,
                      invocation_len=4, alpha=16.0, num_hidden_layers=2, num_local_experts=8,
                      num_experts_per_tok=2, intermediate_size=256, **extra)
    return d


@pytest.mark.parametrize("budget", [48, 2048])
def test_native_moe_matches_reference(moe_dir, budget):
    """Frozen expert bank (grouped tcgen05 GEMMs, per-expert 128-row segments) vs the CPU oracle."""
    worst, agree, total, _ = _compare_engine(moe_dir, _prompts(moe_dir, 5, seed=7), budget)
    assert total == 20
    assert worst < 0.05, worst
    assert agree >= total - 1


def test_fp8_kv_cache_engine_close_to_bf16():
    """The engine with an fp8 (e4m3, per-row scale) KV cache: over a prefill step and two decode
    steps of a tiny random model (prefill chunks, a prefix-cache hit, decode rows), the logits
    stay within a few percent of the bf16 cache's and most greedy tokens agree (both runs are fed
    the bf16 run's tokens)."""
    import torch

    from granite_switch_b200.composer.synthetic import base_config
    from granite_switch_b200.config import GraniteSwitchConfig
    from granite_switch_b200.engine import EngineConfig
    from granite_switch_b200.engine.executor import NativeExecutor
    from granite_switch_b200.engine.kv_cache import BlockManager
    from granite_switch_b200.engine.llm_engine import HostRouter
    from granite_switch_b200.engine.request import Request, SamplingParams
    from granite_switch_b200.engine.scheduler import Scheduler
    from granite_switch_b200.models.native import NativeGraniteSwitch

    base = base_config("tiny")
    na, v = 3, base["vocab_size"]
    cfg = dict(base)
    cfg.update(num_adapters=na, adapter_token_ids=list(range(v, v + na)), adapter_substitute_token_ids=[1] * na,
               adapter_ranks=[8] * na, max_lora_rank=8, lora_target_modules=["qkv_proj", "o_proj"],
               num_hidden_layers=base["num_hidden_layers"] + 2, vocab_size=v + na)
    config = GraniteSwitchConfig(**cfg)
    dev = torch.device("cuda", 0)
    ctx = [int(t) for t in torch.randint(5, 900, (300,), generator=torch.Generator().manual_seed(0))]
    results, forced = {}, []
    for fp8 in (False, True):
        m = NativeGraniteSwitch.from_random(config, dev, max_tokens=1024, num_kv_blocks=128, lora_modules=("qkv", "o"),
                                            rank=8, seed=3, max_seqs=8)
        m.kv_fp8 = fp8
        m._alloc_buffers()
        ex = NativeExecutor(m, 1024)
        bm = BlockManager(128)
        router = HostRouter(config)
        sch = Scheduler(bm, 8, 1024, True, route_fn=router)
        for ids in (ctx + [v, 9, 10], ctx + [v + 1, 11], [3, 4, 5, v + 2] * 20):
            sch.add(Request(ids, SamplingParams(max_tokens=3)))
        outs = []
        for step in range(3):
            out = sch.schedule()
            _, logits = ex.compute_logits(out)
            outs.append(logits.float().cpu())
            # both runs feed the bf16 run's greedy tokens: the random model's logits are
            # nearly flat, and one flipped argmax would change every later step's input
            if not fp8:
                forced.append(logits.argmax(-1).tolist())
            toks = forced[step]
            j = 0
            for c in out.chunks:
                r = c.req
                r.carry = router(r.all_ids[c.start:c.start + c.num_tokens], r.carry)
                r.num_computed = c.start + c.num_tokens
                bm.register_full_blocks(r)
                if c.needs_sample:
                    r.output_ids.append(toks[j])
                    j += 1
        results[fp8] = outs
    for a, b in zip(results[False], results[True]):
        assert a.shape == b.shape
        assert (a - b).abs().max() <= 0.05 * a.abs().max(), float((a - b).abs().max())
        assert (a.argmax(-1) == b.argmax(-1)).float().mean() >= 0.66
    from granite_switch_b200._native import check_errors

    check_errors(dev)


def test_overlapped_attention_plans_match_serial(tiny_dir):
    """Steps with decode rows and prefill chunks give bit-identical logits whether the
    prefill attention runs on a side stream beside the decode attention or after it."""
    from granite_switch_b200.checkpoint import load_state_dict
    from granite_switch_b200.config import GraniteSwitchConfig
    from granite_switch_b200.engine.executor import NativeExecutor
    from granite_switch_b200.engine.kv_cache import BlockManager
    from granite_switch_b200.engine.llm_engine import HostRouter
    from granite_switch_b200.engine.request import Request, SamplingParams
    from granite_switch_b200.engine.scheduler import Scheduler
    from granite_switch_b200.models.native import NativeGraniteSwitch
    from granite_switch_b200._native import check_errors

    cfg = GraniteSwitchConfig.from_pretrained(tiny_dir)
    dev = torch.device("cuda")
    nb = 128
    nm = NativeGraniteSwitch.from_state_dict(cfg, load_state_dict(tiny_dir), dev, max_tokens=2048,
                                             num_kv_blocks=nb, max_seqs=16)
    nat = NativeExecutor(nm, 1024)
    bm = BlockManager(nb)
    router = HostRouter(cfg)
    sch = Scheduler(bm, 8, 64, True, route_fn=router)
    for p in _prompts(tiny_dir, 6, seed=3):
        sch.add(Request(p, SamplingParams(max_tokens=6)))
    mixed = steps = 0
    while sch.has_work() and steps < 200:
        out = sch.schedule()
        nm.overlap_attention = False
        _, serial = nat.compute_logits(out)
        serial = serial.clone() if serial is not None else None  # None: no row samples this step
        nm.overlap_attention = True
        _, overlapped = nat.compute_logits(out)
        torch.cuda.synchronize()
        assert (serial is None) == (overlapped is None)
        if serial is not None:
            assert torch.equal(serial, overlapped)
        q_lens = [c.num_tokens for c in out.chunks]
        g = cfg.num_attention_heads // cfg.num_key_value_heads
        mixed += int(any(q * g <= 16 for q in q_lens) and any(q * g > 16 for q in q_lens))
        j = 0
        for c in out.chunks:
            r = c.req
            r.carry = router(r.all_ids[c.start:c.start + c.num_tokens], r.carry)
            r.num_computed = c.start + c.num_tokens
            bm.register_full_blocks(r)
            if c.needs_sample:
                r.output_ids.append(int(serial[j].argmax()))
                j += 1
                if len(r.output_ids) >= r.sampling.max_tokens:
                    sch.finish(r, "length")
        steps += 1
    check_errors(dev)
    assert mixed > 0  # some steps had both plans
