"""Engine (scheduler, paged KV, prefix cache, chunked prefill) vs plain generate, on CPU."""
import json
import os

import pytest
import torch

from granite_switch_b200.composer.synthetic import compose_synthetic
from granite_switch_b200.engine import LLM, EngineConfig, SamplingParams
from granite_switch_b200.engine.kv_cache import BlockManager, chain_hashes
from granite_switch_b200.engine.request import Request
from granite_switch_b200.engine.scheduler import Scheduler, SchedulerOutput
from granite_switch_b200.models import GraniteSwitchForCausalLM


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("eng"))
    compose_synthetic(d, "tiny", num_adapters=3, rank=8, targets=("q", "k", "v", "o"), seed=0,
                      dtype=torch.float32, invocation_len=4, alpha=16.0, num_hidden_layers=2)
    return d


def _prompts(d, n, seed=0, lo=20, hi=60):
    idx = json.load(open(os.path.join(d, "adapter_index.json")))
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        L = int(torch.randint(lo, hi, (1,), generator=g))
        ids = torch.randint(0, 1000, (L,), generator=g).tolist()
        a = i % 3
        inv = idx["adapters"][a]["invocation_token_ids"]
        ids += [idx["adapters"][a]["control_token"]["id"]] + inv[1:]
        out.append(ids)
    return out


def _ref_generate(d, prompts, n):
    m = GraniteSwitchForCausalLM.from_pretrained(d).eval()
    outs = []
    for p in prompts:
        o = m.generate(torch.tensor([p]), max_new_tokens=n)
        outs.append(o[0, len(p):].tolist())
    return outs


@pytest.mark.parametrize("budget", [16, 1024])
def test_engine_matches_generate(tiny_dir, budget):
    prompts = _prompts(tiny_dir, 5)
    ecfg = EngineConfig(max_num_seqs=3, max_num_batched_tokens=budget, num_kv_blocks=64, max_model_len=256)
    llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
    outs = llm.generate(prompts, SamplingParams(max_tokens=6))
    ref = _ref_generate(tiny_dir, prompts, 6)
    for o, r in zip(outs, ref):
        assert o.output_ids == r


def test_prefix_cache_shared_across_adapters(tiny_dir):
    """aLoRA: the base context is cached once and reused by calls to other adapters."""
    idx = json.load(open(os.path.join(tiny_dir, "adapter_index.json")))
    g = torch.Generator().manual_seed(5)
    ctx = torch.randint(0, 1000, (100,), generator=g).tolist()
    calls = []
    for a in range(3):
        inv = idx["adapters"][a]["invocation_token_ids"]
        calls.append(ctx + [idx["adapters"][a]["control_token"]["id"]] + inv[1:])
    ecfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=512, num_kv_blocks=64, max_model_len=256)
    llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
    first = llm.generate([calls[0]], SamplingParams(max_tokens=4))[0]
    assert first.num_cached_tokens == 0
    rest = llm.generate(calls[1:], SamplingParams(max_tokens=4))
    assert all(r.num_cached_tokens == 96 for r in rest)  # 6 full context blocks
    ref = _ref_generate(tiny_dir, calls, 4)
    assert [first.output_ids] + [r.output_ids for r in rest] == ref


@pytest.mark.parametrize("policy", ["fcfs", "cache_affinity"])
def test_preemption_keeps_outputs(tiny_dir, policy):
    prompts = _prompts(tiny_dir, 6, seed=2, lo=40, hi=70)
    ecfg = EngineConfig(max_num_seqs=6, max_num_batched_tokens=64, num_kv_blocks=14, max_model_len=256,
                        scheduling_policy=policy)
    llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
    outs = llm.generate(prompts, SamplingParams(max_tokens=8))
    assert llm.engine.scheduler.num_preemptions > 0
    ref = _ref_generate(tiny_dir, prompts, 8)
    for o, r in zip(outs, ref):
        assert o.output_ids == r


def test_block_manager_lru_and_hashes():
    bm = BlockManager(4)
    r1 = Request(list(range(40)))
    assert bm.match_prefix(r1) == 0
    assert bm.allocate(r1, 40)
    r1.num_computed = 40
    bm.register_full_blocks(r1)
    bm.free_request(r1)
    assert bm.num_free == 4 and len(bm.evictable) == 2
    r2 = Request(list(range(40)) + [7])
    assert bm.match_prefix(r2) == 32
    assert chain_hashes(list(range(40)), 2) == r1.block_hashes[:2]
    r3 = Request([9] * 70)
    bm.match_prefix(r3)
    assert not bm.allocate(r3, 70)  # 5 blocks > 4


def _cache_context(bm, ctx):
    """Run one request over ``ctx`` through the block manager so its full blocks end up cached."""
    r = Request(ctx + [1])
    bm.match_prefix(r)
    assert bm.allocate(r, len(r.prompt_ids))
    r.num_computed = len(r.prompt_ids)
    bm.register_full_blocks(r)
    bm.free_request(r)


@pytest.mark.parametrize("policy", ["fcfs", "cache_affinity"])
def test_scheduling_policy_admission_order(policy):
    """cache_affinity admits a request whose context is cached ahead of an older cold one;
    fcfs keeps arrival order."""
    bm = BlockManager(64)
    ctx = list(range(100, 164))  # four full blocks
    _cache_context(bm, ctx)
    assert bm.first_block_cached(ctx + [2]) and not bm.first_block_cached(list(range(500, 540)))
    sch = Scheduler(bm, max_num_seqs=1, max_num_batched_tokens=512, policy=policy)
    cold, warm = Request(list(range(500, 540))), Request(ctx + [2, 3])
    sch.add(cold)
    sch.add(warm)
    assert sch.num_waiting == 2
    first = sch.schedule().chunks[0].req
    assert first is (warm if policy == "cache_affinity" else cold)
    assert first.num_cached_tokens == (64 if policy == "cache_affinity" else 0)
    # the other request waits for a free sequence slot, then runs
    sch.finish(first, "length")
    assert sch.schedule().chunks[0].req is (cold if policy == "cache_affinity" else warm)
    assert sch.num_waiting == 0


def test_cache_affinity_max_wait_steps():
    """A cold request passed over for max_wait_steps engine steps is admitted ahead of warm ones."""
    bm = BlockManager(64)
    ctx = list(range(100, 164))
    _cache_context(bm, ctx)
    sch = Scheduler(bm, max_num_seqs=1, max_num_batched_tokens=512, policy="cache_affinity", max_wait_steps=2)
    cold = Request(list(range(500, 540)))
    sch.add(cold)
    order = []
    for i in range(3):
        sch.add(Request(ctx + [2, i]))  # a warm arrival every step
        r = sch.schedule().chunks[0].req
        order.append(r is cold)
        sch.finish(r, "length")
    assert order == [False, True, False]


def _starve(max_wait_steps, steps):
    """Step a one-slot cache-affinity scheduler with a warm arrival every step; return the
    step at which the single cold request was admitted (None if never)."""
    bm = BlockManager(64)
    ctx = list(range(100, 164))
    _cache_context(bm, ctx)
    sch = Scheduler(bm, max_num_seqs=1, max_num_batched_tokens=512, policy="cache_affinity",
                    max_wait_steps=max_wait_steps)
    cold = Request(list(range(500, 540)))
    sch.add(cold)
    for i in range(steps):
        sch.add(Request(ctx + [2, i % 50]))  # the next call of a resident conversation
        r = sch.schedule().chunks[0].req
        sch.finish(r, "length")
        if r is cold:
            return i + 1
    return None


def test_cache_affinity_default_bound_prevents_starvation():
    """A steady stream of warm calls starves a cold request forever without a bound; the
    engine's default bound admits it after DEFAULT_MAX_WAIT_STEPS steps."""
    from granite_switch_b200.engine import DEFAULT_MAX_WAIT_STEPS, EngineConfig

    assert EngineConfig().max_wait_steps == DEFAULT_MAX_WAIT_STEPS
    assert _starve(None, DEFAULT_MAX_WAIT_STEPS + 50) is None
    assert _starve(EngineConfig().max_wait_steps, DEFAULT_MAX_WAIT_STEPS + 50) == DEFAULT_MAX_WAIT_STEPS


def test_cache_affinity_preempted_and_abort():
    bm = BlockManager(64)
    sch = Scheduler(bm, max_num_seqs=2, max_num_batched_tokens=512, policy="cache_affinity")
    a = Request(list(range(10, 50)))
    sch.add(a)
    assert sch.schedule().chunks[0].req is a
    b = Request(list(range(60, 100)))
    sch.add(b)  # cold, arrives while a runs
    sch._preempt(a, SchedulerOutput())
    assert sch.warm[0] is a  # a preempted request resumes before cold arrivals
    assert [c.req for c in sch.schedule().chunks] == [a, b]
    c = Request(list(range(10, 50)) + [5])
    a.num_computed = 40  # a's prefill ran: its two full blocks are published
    bm.register_full_blocks(a)
    sch.add(c)
    assert c in sch.warm and sch.abort(c.request_id) and c not in sch.warm
    with pytest.raises(ValueError):
        Scheduler(bm, policy="lifo")


def test_routing_trace(tiny_dir, tmp_path):
    """Per-step routing records: positions run 0..n-1 per request and the adapter index switches
    on at the control token (aLoRA), across chunked-prefill and decode steps."""
    idx = json.load(open(os.path.join(tiny_dir, "adapter_index.json")))
    prompts = _prompts(tiny_dir, 3)
    ecfg = EngineConfig(max_num_seqs=3, max_num_batched_tokens=16, num_kv_blocks=64, max_model_len=256)
    llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
    path = str(tmp_path / "trace.jsonl")
    trace = llm.enable_routing_trace(path)
    outs = llm.generate(prompts, SamplingParams(max_tokens=3))
    for i, (p, o) in enumerate(zip(prompts, outs)):
        pos = trace.of_request(o.request_id, "positions")
        ids = trace.of_request(o.request_id, "ids")
        assert pos == list(range(len(pos))) and ids == (p + o.output_ids)[:len(ids)]
        ctrl = p.index(idx["adapters"][i % 3]["control_token"]["id"])
        adapter = trace.of_request(o.request_id, "adapter")
        assert adapter == [0] * ctrl + [i % 3 + 1] * (len(adapter) - ctrl)
    trace.flush()
    lines = open(path).read().splitlines()
    assert len(lines) == trace.step and json.loads(lines[0])["spans"]


def test_prefill_layout_choice():
    """Two query tiles per CTA only when long, mostly fresh chunks carry most prefill tokens."""
    from granite_switch_b200.ops import attention as A

    assert A.tc_rows_for([4096, 3968], [4096, 3968]) == 256
    assert A.tc_rows_for([512] * 8, [4096] * 8) == 128
    assert A.tc_rows_for([40, 60], [40, 60]) == 128
    assert A.tc_rows_for([2048, 64], [2048, 9000]) == 256


def test_short_chunks_over_long_prefix_split_kv():
    """Short prefill chunks after long cached prefixes split each tcgen05 tile's key range;
    fresh or many chunks keep one CTA per tile."""
    import types

    from granite_switch_b200.models.native import NativeGraniteSwitch
    from granite_switch_b200.ops import attention as A

    assert A.split_prefill([48, 48], [4548, 4548], 4, 8) == 5    # 32 CTAs of 128 rows -> 5 splits
    assert A.split_prefill([4096], [4096], 4, 8) == 0            # 1024 CTAs
    assert A.split_prefill([48, 48], [300, 500], 4, 8) == 0      # short contexts
    assert A.split_prefill([48, 48, 300], [4548, 4548, 300], 4, 8) == 2  # 112 CTAs
    assert A.split_prefill([300] * 3, [4548] * 3, 4, 8) == 0     # 240 CTAs
    assert A.split_prefill([48, 48], [4548, 4548], 4, 8, rows=64) == 4  # 48 CTAs of 64 rows (fp8 cache)
    assert A.choose_splits(1024, 4200) == 2    # decode: 128 requests x 8 KV heads
    assert A.choose_splits(2048, 4200) == 1    # enough CTAs without a split
    assert A.choose_splits(64, 8192) == 16     # a small batch: capped at 512 keys per split
    assert A.choose_splits(64, 300) == 1       # short contexts never split
    m = types.SimpleNamespace(num_q=32, num_kv=8, head_dim=128, use_tc_attention=True, ws_tokens=512, kv_fp8=False)
    q = [48, 48] + [1] * 126
    kv = [4548, 4548] + [4500] * 126
    plans = NativeGraniteSwitch.attention_plans(m, q, kv)
    # decode rows: 126 x 8 KV heads = 1,008 CTAs, under the 1,536 a split grid aims at -> 2 splits
    assert [(p[2], p[3]) for p in plans] == [(16, 2), (128, 5)]
    assert sorted(plans[1][0]) == [0, 0, 1, 1]  # two 128-row tiles per chunk
    plans = NativeGraniteSwitch.attention_plans(m, [4096] + [1] * 127, [4096] + [4500] * 127)
    assert plans[1][2] == 256 and plans[1][3] == 1
    m.ws_tokens = 128  # the split workspace cannot hold the step: no split
    assert NativeGraniteSwitch.attention_plans(m, q, kv)[1][2:] == (128, 1)
    # fp8 cache: decode rows in 8-row tiles (keys on the MMA's row side), prefill chunks on
    # the 64-row mma.sync layout with its own key split
    m.ws_tokens, m.kv_fp8 = 512, True
    plans = NativeGraniteSwitch.attention_plans(m, q, kv)
    assert [(p[2], p[3]) for p in plans] == [(8, 2), (64, 4)]
    assert len(plans[0][0]) == 126  # one 8-row tile per decode request (4 query heads each)


def test_pick_bn_policy():
    """GEMM N-tile choice: widest filling tile for large M, 128 for two row tiles, narrowest
    filling tile for one row tile and for the LoRA shrink."""
    from granite_switch_b200.ops.gemm import pick_bn

    assert pick_bn(8192, 6144) == 256
    assert pick_bn(222, 6144) == 128 and pick_bn(222, 4096) == 128
    assert pick_bn(100, 6144) == 64 and pick_bn(300, 4096) == 64
    assert pick_bn(222, 384, (128, 64), two_tile_bn=None) == 64
    assert pick_bn(222, 768) == 64  # a tensor-parallel shard: too few 128-wide tiles


def test_cache_affinity_raises_hit_rate_under_overload():
    """Chained calls under overload with a small KV cache: cache-affinity admission keeps the
    running conversations' contexts resident, FCFS admission evicts them for new contexts.
    The model is replaced by an executor that returns fixed tokens (scheduling only)."""
    import types

    from granite_switch_b200.engine.llm_engine import LLMEngine
    from granite_switch_b200.engine.request import SamplingParams
    from granite_switch_b200.utils.workload import WorkloadConfig, advance, call_prompt, make_workload

    cfg = types.SimpleNamespace(num_adapters=0, adapter_token_ids=[], eos_token_id=None)

    class _Exec:
        def execute(self, out):
            return [7 for c in out.chunks if c.needs_sample]

    def run(policy):
        eng = LLMEngine(cfg, _Exec(), 96, EngineConfig(max_num_seqs=4, max_num_batched_tokens=256,
                                                       max_model_len=1024, scheduling_policy=policy))
        convs = make_workload(WorkloadConfig(num_conversations=24, rate=float("inf"), context_len=160, calls=4,
                                             inv_min=4, inv_max=8, gen_min=4, gen_max=8, vocab=1000, num_adapters=1,
                                             seed=1))
        by_req = {}

        def submit(conv):
            r = eng.add_request(call_prompt(conv, [999]), SamplingParams(max_tokens=conv.calls[conv.next_call].gen_len,
                                                                        ignore_eos=True))
            by_req[r.request_id] = conv

        def on_finish(req):
            conv = by_req.pop(req.request_id)
            if advance(conv, req.prompt_ids, req.output_ids):
                submit(conv)

        eng.on_finish = on_finish
        for c in convs:
            submit(c)
        steps = 0
        while eng.has_unfinished() and steps < 5000:
            eng.step()
            steps += 1
        assert not eng.has_unfinished()
        assert all(c.next_call == 4 for c in convs)  # every call of every conversation ran
        return eng.prefix_cache_hit_rate()

    fcfs, affinity = run("fcfs"), run("cache_affinity")
    assert affinity > fcfs + 0.2, (fcfs, affinity)


def test_device_error_aborts_the_step(tiny_dir):
    """A kernel error reported in a step (here: the executor's error word, faked) aborts the
    requests that step carried, drops the prefix cache and re-raises; the engine then keeps
    serving the other requests, whose outputs still match plain generate."""
    from granite_switch_b200._native import ERR_ATTN_WAIT, DeviceError

    prompts = _prompts(tiny_dir, 4, seed=3)
    ecfg = EngineConfig(max_num_seqs=2, max_num_batched_tokens=1024, num_kv_blocks=64, max_model_len=256)
    llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
    eng = llm.engine
    real = eng.executor.execute
    calls = {"n": 0}

    def flaky(out):
        calls["n"] += 1
        if calls["n"] == 3:  # third step: the kernels report an attention wait that ran out
            raise DeviceError(ERR_ATTN_WAIT, "attention page id", 7)
        return real(out)

    eng.executor.execute = flaky
    reqs = [eng.add_request(p, SamplingParams(max_tokens=6)) for p in prompts]
    errors = []
    while eng.has_unfinished():
        try:
            eng.step()
        except DeviceError as e:
            errors.append(e)
    assert len(errors) == 1 and "attention-wait-timeout" in str(errors[0]) and "attention page id = 7" in str(errors[0])
    assert eng.stats.device_errors == 1
    failed = [r for r in reqs if r.finish_reason == "error"]
    ok = [r for r in reqs if r.finish_reason == "length"]
    assert failed and ok and len(failed) + len(ok) == len(reqs)
    ref = _ref_generate(tiny_dir, [r.prompt_ids for r in ok], 6)
    assert [r.output_ids for r in ok] == ref


def test_executor_error_word_check():
    """The executor turns a nonzero error word into DeviceError with the site decoded."""
    from granite_switch_b200._native import ERR_BAD_SHAPE, DeviceError, describe_error, site_name

    assert site_name(0) is None and site_name(3) == "KV slot"
    e = DeviceError(ERR_BAD_SHAPE, site_name(3), 99)
    assert "bad-shape" in str(e) and "KV slot = 99" in str(e) and e.word == ERR_BAD_SHAPE
    assert describe_error(0x3).count("timeout") == 2


@pytest.mark.parametrize("budget,blocks", [(64, 14), (1024, 64)])
def test_async_steps_match_sync(tiny_dir, budget, blocks):
    """Pipelined steps (step i+1 launched before step i's ids are read, decode rows fed on the
    device) give the same outputs as blocking steps: chunked prefill, preemption under a small
    KV cache, per-request max_tokens, stop tokens taken from the sync run, and seeded
    temperature sampling."""
    prompts = _prompts(tiny_dir, 6, seed=4, lo=30, hi=70)

    def run(async_on, params):
        ecfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=budget, num_kv_blocks=blocks, max_model_len=256,
                            async_scheduling=async_on)
        llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
        assert llm.engine.async_steps == async_on
        outs = llm.generate(prompts, params)
        return [o.output_ids for o in outs], [o.finish_reason for o in outs], llm.engine

    greedy = [SamplingParams(max_tokens=3 + i) for i in range(len(prompts))]
    ref_ids, _, _ = run(False, greedy)
    # stop on a token the sync run produced mid-sequence
    stop = [SamplingParams(max_tokens=8, stop_token_ids=(ids[2],)) for ids in ref_ids]
    sampled = [SamplingParams(max_tokens=6, temperature=0.8, seed=11 + i) for i in range(len(prompts))]
    for params in (greedy, stop, sampled):
        a_ids, a_reason, eng = run(True, params)
        s_ids, s_reason, _ = run(False, params)
        assert a_ids == s_ids and a_reason == s_reason
        assert not eng.has_unfinished() and eng._inflight is None
        assert all(t >= 0 for ids in a_ids for t in ids)


def test_async_abort_while_running(tiny_dir):
    """A request aborted while a step that carries it is in flight gets no token from that
    step; the others match blocking steps."""
    prompts = _prompts(tiny_dir, 3, seed=5)
    ecfg = EngineConfig(max_num_seqs=3, max_num_batched_tokens=1024, num_kv_blocks=64, max_model_len=256)
    llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
    eng = llm.engine
    reqs = [eng.add_request(p, SamplingParams(max_tokens=6)) for p in prompts]
    eng.step()
    eng.step()
    assert eng._inflight is not None and any(c.req is reqs[0] for c in eng._inflight.out.chunks)
    n = len(reqs[0].output_ids)
    assert eng.abort_request(reqs[0].request_id)
    while eng.has_unfinished():
        eng.step()
    ref = _ref_generate(tiny_dir, prompts[1:], 6)
    assert [r.output_ids for r in reqs[1:]] == ref
    assert reqs[0].finish_reason == "abort" and len(reqs[0].output_ids) == n
    assert all(t >= 0 for t in reqs[0].output_ids)


def test_pp_microbatch_split():
    """A pipelined step splits into two micro-batches of whole sequences holding about half
    the tokens each; no split with one sequence, probes or a routing trace."""
    import types

    from granite_switch_b200.engine.executor import NativeExecutor
    from granite_switch_b200.engine.request import Request
    from granite_switch_b200.engine.scheduler import ScheduledChunk, SchedulerOutput

    ex = types.SimpleNamespace(pp_microbatches=True, routing_trace=None, model=types.SimpleNamespace(probe_w=None),
                               PP_SPLIT_MIN_TOKENS=2)

    def out(sizes):
        return SchedulerOutput(chunks=[ScheduledChunk(Request(list(range(n + 1))), 0, n) for n in sizes])

    for sizes, k in (([1, 1], 1), ([100, 1, 1, 1], 1), ([1, 1, 1, 100], 3), ([10, 10, 10, 10], 2), ([5, 50, 5], 2)):
        parts = NativeExecutor._pp_parts(ex, out(sizes))
        assert [len(p.chunks) for p in parts] == [k, len(sizes) - k], (sizes, [len(p.chunks) for p in parts])
    assert NativeExecutor._pp_parts(ex, out([64])) is None
    ex.PP_SPLIT_MIN_TOKENS = 1024
    assert NativeExecutor._pp_parts(ex, out([500, 500])) is None  # weight-bound: run whole
    assert NativeExecutor._pp_parts(ex, out([600, 600])) is not None
    ex.model.probe_w = object()
    assert NativeExecutor._pp_parts(ex, out([8, 8])) is None


def test_async_launch_failure_loses_no_step(tiny_dir):
    """A launch that raises (not a device error) leaves the engine consistent: the running
    step's ids are still resolved, the step that failed to launch runs again on the next
    call, and every output matches plain generate."""
    prompts = _prompts(tiny_dir, 3, seed=6)
    ecfg = EngineConfig(max_num_seqs=3, max_num_batched_tokens=1024, num_kv_blocks=64, max_model_len=256)
    llm = LLM(tiny_dir, device="cpu", engine_config=ecfg)
    eng = llm.engine
    real = eng.executor.launch
    calls = {"n": 0}

    def flaky(out):
        calls["n"] += 1
        if calls["n"] == 3:
            raise RuntimeError("launch failed")
        return real(out)

    eng.executor.launch = flaky
    reqs = [eng.add_request(p, SamplingParams(max_tokens=6)) for p in prompts]
    failures = 0
    while eng.has_unfinished():
        try:
            eng.step()
        except RuntimeError:
            failures += 1
    assert failures == 1
    assert [r.output_ids for r in reqs] == _ref_generate(tiny_dir, prompts, 6)


def test_graph_bucket_gating_under_tp():
    """Decode-only steps take the smallest padded bucket; under tensor parallelism only
    buckets whose reductions all ride in the fused epilogue (no NCCL inside a graph)."""
    import types

    from granite_switch_b200.engine.executor import NativeExecutor

    def ex(tp, comm, max_seqs=256, dual=False, moe=False):
        e = NativeExecutor.__new__(NativeExecutor)
        e.use_cuda_graphs, e.tp_size = True, tp
        e.model = types.SimpleNamespace(max_seqs=max_seqs, max_tokens=8192, comm=comm, dual=dual, has_moe=moe)
        return e

    def step(n, decode_only=True):
        return types.SimpleNamespace(is_decode_only=decode_only, chunks=[None] * n)

    fused = types.SimpleNamespace(red_max_tokens=256)
    assert ex(1, None)._graph_bucket(step(100)) == 128
    assert ex(1, None)._graph_bucket(step(100, decode_only=False)) is None
    assert ex(1, None, max_seqs=64)._graph_bucket(step(100)) is None  # beyond the largest bucket that fits
    assert ex(2, None)._graph_bucket(step(100)) is None                # NCCL reductions: eager
    assert ex(8, fused)._graph_bucket(step(100)) == 128                # fused up to 256 rows
    assert ex(8, fused)._graph_bucket(step(300)) is None               # bucket 512 would all-reduce over NCCL
    assert ex(8, fused, dual=True)._graph_bucket(step(10)) is None     # Shadow-Residual reduces over NCCL
    assert ex(8, fused, moe=True)._graph_bucket(step(10)) is None      # so do expert banks
