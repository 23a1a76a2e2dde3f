"""Native norm / embedding / RoPE+KV / argmax / routing / attention vs PyTorch fp32 oracles (GPU)."""
import random

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200 import _native

    _native.native()


def _check(dev="cuda"):
    from granite_switch_b200._native import check_errors

    check_errors(torch.device(dev))


@pytest.mark.parametrize("h", [64, 2048, 4096])
def test_rmsnorm(h):
    from granite_switch_b200.ops import elementwise as E

    x = torch.randn(37, h, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(h, device="cuda")).bfloat16()
    out = E.rmsnorm(x, w, 1e-5)
    ref = E.rmsnorm_reference(x, w, 1e-5)
    assert (out.float() - ref.float()).abs().max() <= 0.02 * ref.float().abs().max()
    rows = torch.tensor([3, 0, 36], device="cuda")
    out2 = E.rmsnorm(x, w, 1e-5, rows=rows)
    assert torch.equal(out2, out[rows])


def test_embed_exchange():
    from granite_switch_b200.ops import elementwise as E

    table = torch.randn(300, 64, device="cuda").bfloat16()
    lut = torch.full((302,), -1, dtype=torch.long, device="cuda")
    lut[300], lut[301] = 5, 7
    ids = torch.tensor([1, 300, 2, 301, 299], device="cuda")
    table2 = torch.cat([table, torch.zeros(2, 64, device="cuda").bfloat16()])
    out = E.embed(ids, table2, lut, 12.0)
    ref = E.embed_reference(ids, table2, lut, 12.0)
    assert torch.equal(out, ref)
    _check()


@pytest.mark.parametrize("d", [64, 128])
def test_rope_kv_write(d):
    from granite_switch_b200.ops import elementwise as E

    hq, hkv, t = 8, 2, 20
    cs = E.rope_cos_sin_table(4096, d, 10000.0, "cuda")
    qkv = torch.randn(t, (hq + 2 * hkv) * d, device="cuda").bfloat16()
    pos = torch.randint(0, 4000, (t,), device="cuda")
    kc = torch.zeros(8, hkv, 16, d, device="cuda").bfloat16()
    vc = torch.zeros_like(kc)
    slots = torch.randperm(8 * 16, device="cuda")[:t]
    orig = qkv.clone()
    E.rope_kv(qkv, pos, cs, hq, hkv, d, kc, vc, slots)
    q_ref = E.rope_reference(orig[:, : hq * d].view(t, hq, d), pos, cs)
    k_ref = E.rope_reference(orig[:, hq * d:(hq + hkv) * d].view(t, hkv, d), pos, cs)
    v_ref = orig[:, (hq + hkv) * d:].view(t, hkv, d)
    assert (qkv[:, : hq * d].view(t, hq, d).float() - q_ref.float()).abs().max() < 2e-2
    for i in range(t):
        b, o = int(slots[i]) // 16, int(slots[i]) % 16
        assert (kc[b, :, o].float() - k_ref[i].float()).abs().max() < 2e-2
        assert torch.equal(vc[b, :, o], v_ref[i])
    _check()


def test_argmax():
    from granite_switch_b200.ops import elementwise as E

    x = torch.randn(9, 49155, device="cuda")
    x[3, 17] = 100.0
    assert torch.equal(E.argmax(x), x.argmax(dim=1))


def test_routing_kernel_matches_scan():
    from granite_switch_b200.ops.routing import route_device, tile_masks_reference
    from granite_switch_b200.routing.scan import expert_table, route_flat

    rng = random.Random(0)
    na = 5
    ctrl = [1000 + i for i in range(na)]
    tbl = expert_table(ctrl, na, 1100)
    lens = [rng.randrange(1, 700) for _ in range(7)] + [1, 1, 1]
    ids = []
    for n in lens:
        ids += [rng.choice(ctrl) if rng.random() < 0.02 else rng.randrange(0, 1000) for _ in range(n)]
    starts = [0]
    for n in lens:
        starts.append(starts[-1] + n)
    carries = [rng.randrange(0, na + 1) for _ in lens]
    ref, ref_c = route_flat(torch.tensor(ids), starts, carries, tbl)
    T = len(ids)
    dev = "cuda"
    lut = torch.full((1100,), -1, dtype=torch.long)
    for i, c in enumerate(ctrl):
        lut[c] = i
    kind = torch.zeros(na + 1, dtype=torch.bool)
    kind[3] = True  # slot 3 is a probe
    remap = torch.tensor([[0, 1, 2, 3, 4, 5], [0, 0, 1, 0, 0, 2]], dtype=torch.int32)
    out_a = torch.empty(T, dtype=torch.int32, device=dev)
    out_l = torch.empty(T, dtype=torch.int32, device=dev)
    out_ids = torch.empty(T, dtype=torch.long, device=dev)
    out_c = torch.empty(len(lens), dtype=torch.int32, device=dev)
    ra = torch.empty(2, T, dtype=torch.int32, device=dev)
    tm = torch.empty(2, (T + 127) // 128, dtype=torch.int64, device=dev)
    route_device(torch.tensor(ids, device=dev), torch.tensor(starts, dtype=torch.int32, device=dev),
                 torch.tensor(carries, dtype=torch.int32, device=dev), tbl.to(dev), lut.to(dev), kind.to(dev),
                 na, remap.to(dev), out_a, out_l, out_ids, out_c, ra, tm)
    assert out_a.cpu().tolist() == ref.tolist()
    assert out_c.cpu().tolist() == ref_c
    lora = torch.where(ref == 3, torch.zeros_like(ref), ref)
    assert out_l.cpu().tolist() == lora.tolist()
    ex = torch.tensor(ids)
    ex = torch.where(lut[ex] >= 0, lut[ex], ex)
    assert out_ids.cpu().tolist() == ex.tolist()
    for m in range(2):
        want = remap[m][lora].int()
        assert ra[m].cpu().tolist() == want.tolist()
        assert tm[m].cpu().tolist() == tile_masks_reference(want).tolist()


def _make_cache(lens, hkv, d, seed=0):
    torch.manual_seed(seed)
    nblk = sum((l + 15) // 16 for l in lens) + 3
    kc = torch.randn(nblk, hkv, 16, d, device="cuda").bfloat16()
    vc = torch.randn(nblk, hkv, 16, d, device="cuda").bfloat16()
    perm = torch.randperm(nblk).tolist()
    maxb = max((l + 15) // 16 for l in lens)
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32)
    p = 0
    for i, l in enumerate(lens):
        for j in range((l + 15) // 16):
            bt[i, j] = perm[p]
            p += 1
    return kc, vc, bt.cuda()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("mode", ["prefill", "prefill128", "decode", "decode2", "short_after_long"])
@pytest.mark.parametrize("nsplit", [1, 3])
def test_paged_attention(d, mode, nsplit):
    from granite_switch_b200._native import native
    from granite_switch_b200.ops import attention as A

    old_stages = native().attn_decode_stages(2 if mode == "decode2" else 3)
    mode = "decode" if mode == "decode2" else mode

    hq, hkv = 8, 2
    g = hq // hkv
    if mode == "decode":
        q_lens = [1, 1, 2, 1, 4]
        kv_lens = [1, 37, 300, 1025, 64]
        rows = 16
    elif mode == "short_after_long":  # a conversation's next call: split-KV prefill layout
        q_lens = [48, 40, 17]
        kv_lens = [4548, 2100, 1040]
        rows = 64
        nsplit = 4 if nsplit > 1 else 1
    else:
        q_lens = [5, 64, 130, 1, 40]
        kv_lens = [5, 200, 130, 77, 1000]
        rows = 128 if mode == "prefill128" else 64
    kc, vc, bt = _make_cache(kv_lens, hkv, d)
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()  # qkv buffer, q at the front
    out = torch.zeros(T, hq * d, device="cuda").bfloat16()
    qs = [0]
    for l in q_lens:
        qs.append(qs[-1] + l)
    ws, wr = A.build_work(q_lens, g, rows)
    dev = "cuda"
    ws_o = torch.empty(nsplit * T * hq * d, device=dev)
    ws_l = torch.empty(nsplit * T * hq, device=dev)
    A.paged_attention(q, kc, vc, bt, torch.tensor(qs, dtype=torch.int32, device=dev),
                      torch.tensor(kv_lens, dtype=torch.int32, device=dev),
                      torch.tensor(ws, dtype=torch.int32, device=dev), torch.tensor(wr, dtype=torch.int32, device=dev),
                      rows, hq, 0.125, out, nsplit, ws_o, ws_l)
    native().attn_decode_stages(old_stages)
    ref = A.paged_attention_reference(q, kc, vc, bt, q_lens, kv_lens, hq, 0.125)
    err = (out.float() - ref).abs().max().item()
    assert err < 3e-2, err
    _check()


@pytest.mark.parametrize("pre_rows", [64, 128])
@pytest.mark.parametrize("dec_split", [1, 3])
def test_step_plans_share_output_and_workspace(dec_split, pre_rows):
    """The two attention plans of one engine step (decode rows, then short prefill chunks over
    long cached prefixes with split keys) write disjoint rows of one output and share the split
    workspaces: each split merge must touch only its own plan's rows."""
    from granite_switch_b200.ops import attention as A

    hq, hkv, d = 8, 2, 128
    g = hq // hkv
    q_lens = [1, 1, 48, 2, 40]
    kv_lens = [300, 2100, 4548, 700, 1500]
    kc, vc, bt = _make_cache(kv_lens, hkv, d, seed=5)
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()
    out = torch.zeros(T, hq * d, device="cuda").bfloat16()
    qs = [0]
    for n in q_lens:
        qs.append(qs[-1] + n)
    dev = "cuda"
    # unwritten workspace entries read as NaN
    ws_o = torch.full((4 * T * hq * d,), float("nan"), device=dev)
    ws_l = torch.full((4 * T * hq,), float("nan"), device=dev)
    dec = [i for i, n in enumerate(q_lens) if n * g <= 16]
    pre = [i for i, n in enumerate(q_lens) if n * g > 16]
    for idx, rows, ns in ((dec, 16, dec_split), (pre, pre_rows, 4)):
        sw, wr = A.build_work([q_lens[i] for i in idx], g, rows)
        args = (q, kc, vc, bt, torch.tensor(qs, dtype=torch.int32, device=dev),
                torch.tensor(kv_lens, dtype=torch.int32, device=dev),
                torch.tensor([idx[t] for t in sw], dtype=torch.int32, device=dev),
                torch.tensor(wr, dtype=torch.int32, device=dev))
        if rows == 128:  # tcgen05 prefill with split keys
            A.prefill_attention_tc(*args, hq, 0.125, out, rows, ns, ws_o, ws_l)
        else:
            A.paged_attention(*args, rows, hq, 0.125, out, ns, ws_o, ws_l)
    ref = A.paged_attention_reference(q, kc, vc, bt, q_lens, kv_lens, hq, 0.125)
    err = (out.float() - ref).abs().max().item()
    assert err < 3e-2, err
    _check()


@pytest.mark.parametrize("rows,nsplit", [(128, 1), (128, 3), (256, 1)])
@pytest.mark.parametrize("packed", [0, 1])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("case", ["fresh", "cached_prefix", "mixed"])
def test_prefill_attention_tcgen05(case, d, packed, rows, nsplit):
    from granite_switch_b200._native import native
    from granite_switch_b200.ops import attention as A

    old = native().attn_packed(packed)  # softmax on scalar or packed f32x2 arithmetic

    hq, hkv = 8, 2
    g = hq // hkv
    if case == "fresh":
        q_lens, kv_lens = [130, 64, 5], [130, 64, 5]
    elif case == "cached_prefix":
        q_lens, kv_lens = [40, 100], [300, 1100]
    else:
        q_lens, kv_lens = [1, 257, 33], [77, 257, 700]
    kc, vc, bt = _make_cache(kv_lens, hkv, d, seed=3)
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()
    out = torch.zeros(T, hq * d, device="cuda").bfloat16()
    qs = [0]
    for l in q_lens:
        qs.append(qs[-1] + l)
    ws, wr = A.build_work(q_lens, g, rows)
    dev = "cuda"
    # key-split partials; unwritten workspace entries read as NaN
    ws_o = torch.full((nsplit * T * hq * d,), float("nan"), device=dev)
    ws_l = torch.full((nsplit * T * hq,), float("nan"), device=dev)
    A.prefill_attention_tc(q, kc, vc, bt, torch.tensor(qs, dtype=torch.int32, device=dev),
                           torch.tensor(kv_lens, dtype=torch.int32, device=dev),
                           torch.tensor(ws, dtype=torch.int32, device=dev),
                           torch.tensor(wr, dtype=torch.int32, device=dev), hq, 0.088, out, rows, nsplit, ws_o, ws_l)
    native().attn_packed(old)
    ref = A.paged_attention_reference(q, kc, vc, bt, q_lens, kv_lens, hq, 0.088)
    err = (out.float() - ref).abs().max().item()
    assert err < 3e-2, err
    _check()


def test_bad_indices_reported_not_faulted():
    """A token id or page id outside its tensor is replaced by entry 0 and reported with its
    site and value. The tensors given to the kernels are prefix views of larger allocations,
    so even an unchecked access would stay inside allocated memory."""
    from granite_switch_b200._native import read_error_detail
    from granite_switch_b200.ops import attention as A
    from granite_switch_b200.ops import elementwise as E

    dev = torch.device("cuda", 0)
    read_error_detail(dev)  # start clean
    table = torch.randn(300, 64, device="cuda").bfloat16()
    view = table[:290]
    out = E.embed(torch.tensor([1, 295, 2], device="cuda"), view, None, 1.0)
    w, site, idx = read_error_detail(dev)
    assert w & 8 and site == "embedding token id" and idx == 295
    assert torch.equal(out[1], view[0]) and torch.equal(out[0], view[1])

    hq, hkv, d = 8, 2, 128
    kv_lens = [300, 500]
    kc, vc, bt = _make_cache(kv_lens, hkv, d)
    n_ok = kc.shape[0] - 3
    assert int(bt.max()) >= n_ok  # some pages fall outside the view
    q_lens = [1, 1]
    q = torch.randn(2, (hq + 2 * hkv) * d, device="cuda").bfloat16()
    out = torch.zeros(2, hq * d, device="cuda").bfloat16()
    ws, wr = A.build_work(q_lens, hq // hkv, 16)
    i32 = dict(dtype=torch.int32, device="cuda")
    args = (torch.tensor([0, 1, 2], **i32), torch.tensor(kv_lens, **i32), torch.tensor(ws, **i32),
            torch.tensor(wr, **i32))
    A.paged_attention(q, kc[:n_ok], vc[:n_ok], bt, *args, 16, hq, 0.1, out)
    w, site, idx = read_error_detail(dev)
    assert w & 8 and site == "attention page id" and idx >= n_ok
    ws, wr = A.build_work(q_lens, hq // hkv, 128)
    args = args[:2] + (torch.tensor(ws, **i32), torch.tensor(wr, **i32))
    A.prefill_attention_tc(q, kc[:n_ok], vc[:n_ok], bt, *args, hq, 0.1, out)
    w, site, idx = read_error_detail(dev)
    assert w & 8 and site == "tcgen05 attention page id" and idx >= n_ok
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("d", [64, 128])
def test_kv_write_fp8_roundtrip(d):
    """fp8 cache write: every (token, KV head) row is stored as e4m3 with scale max|x| / 448;
    dequantised it is within e4m3's rounding of the bf16 row (half an ulp of a 3-bit mantissa,
    plus the subnormal step)."""
    from granite_switch_b200.ops import attention as A

    hq, hkv, t, nb = 8, 2, 50, 16
    qkv = (torch.randn(t, (hq + 2 * hkv) * d, device="cuda") * torch.rand(t, 1, device="cuda") * 8).bfloat16()
    slots = torch.randperm(nb * 16, device="cuda")[:t]
    k8 = torch.zeros(nb, hkv, 16, d, dtype=torch.uint8, device="cuda")
    v8 = torch.zeros(nb, hkv, d, 16, dtype=torch.uint8, device="cuda")
    ks = torch.ones(nb, hkv, 16, device="cuda")
    vs = torch.ones(nb, hkv, 16, device="cuda")
    A.kv_write_fp8(qkv, slots, k8, v8, ks, vs, hq, hkv, d)
    kf, vf = A.dequantize_fp8_cache(k8, v8, ks, vs)
    blk, off = slots // 16, slots % 16
    k = qkv[:, hq * d:(hq + hkv) * d].float().view(t, hkv, d)
    v = qkv[:, (hq + hkv) * d:].float().view(t, hkv, d)
    for x, deq, sc in ((k, kf, ks), (v, vf, vs)):
        got = deq[blk, :, off]  # [t, hkv, d]
        scale = sc[blk, :, off].unsqueeze(-1)
        amax = x.abs().amax(-1, keepdim=True)
        torch.testing.assert_close(scale, torch.where(amax > 0, amax / 448, torch.ones_like(amax)))
        bound = 0.0625 * x.abs() + scale * 2.0 ** -9 + 1e-7
        assert ((got - x).abs() <= bound).all()
    _check()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("hq,hkv", [(8, 2), (32, 8), (4, 1)])
def test_rope_kv_fp8_fused_matches_separate(d, hq, hkv):
    """The fused RoPE + fp8 K/V write leaves qkv, the fp8 pages and the scales bit for bit as
    RoPE followed by the separate quantised write does."""
    from granite_switch_b200.ops import attention as A
    from granite_switch_b200.ops import elementwise as E

    t, nb, max_pos = 37, 12, 512
    gen = torch.Generator(device="cuda").manual_seed(d + hq)
    qkv = (torch.randn(t, (hq + 2 * hkv) * d, device="cuda", generator=gen) * 3).bfloat16()
    pos = torch.randint(0, max_pos, (t,), device="cuda", generator=gen)
    cos_sin = E.rope_cos_sin_table(max_pos, d, 10000.0, "cuda")
    slots = torch.randperm(nb * 16, device="cuda", generator=gen)[:t]
    outs = []
    for fused in (False, True):
        q = qkv.clone()
        k8 = torch.zeros(nb, hkv, 16, d, dtype=torch.uint8, device="cuda")
        v8 = torch.zeros(nb, hkv, d, 16, dtype=torch.uint8, device="cuda")
        ks = torch.zeros(nb, hkv, 16, device="cuda")
        vs = torch.zeros(nb, hkv, 16, device="cuda")
        if fused:
            A.rope_kv_fp8(q, pos, cos_sin, slots, k8, v8, ks, vs, hq, hkv, d)
        else:
            E.rope_kv(q, pos, cos_sin, hq, hkv, d)
            A.kv_write_fp8(q, slots, k8, v8, ks, vs, hq, hkv, d)
        outs.append((q, k8, v8, ks, vs))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    _check()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("mode", ["decode", "decode8", "prefill", "prefill128", "short_after_long"])
@pytest.mark.parametrize("nsplit", [1, 3])
@pytest.mark.parametrize("hq", [8, 4])
def test_paged_attention_fp8(d, mode, nsplit, hq):
    """Paged attention over the fp8 cache (every mma.sync layout, including the 8-row decode
    tiles with the keys on the MMA's row side; split keys, GQA groups of 4 and 2) against the
    fp32 oracle on the dequantised cache: the kernel's only extra error is bf16 rounding."""
    from granite_switch_b200.ops import attention as A

    hkv = 2
    g = hq // hkv
    if mode in ("decode", "decode8"):
        # decode8: a 4-token request at 4 heads per KV head spans two 8-row tiles
        q_lens, kv_lens, rows = [1, 1, 2, 1, 4], [1, 37, 300, 1025, 64], (16 if mode == "decode" else 8)
    elif mode == "short_after_long":
        q_lens, kv_lens, rows = [48, 40, 17], [4548, 2100, 1040], 64
        nsplit = 4 if nsplit > 1 else 1
    else:
        q_lens, kv_lens = [5, 64, 130, 1, 40], [5, 200, 130, 77, 1000]
        rows = 128 if mode == "prefill128" else 64
    nb = sum((n + 15) // 16 for n in kv_lens) + 4
    gen = torch.Generator(device="cuda").manual_seed(3)
    # fill every page through the write kernel: random K/V rows at every slot
    slots_all = torch.arange(nb * 16, device="cuda")
    src = torch.randn(nb * 16, (hq + 2 * hkv) * d, device="cuda", generator=gen).bfloat16()
    k8 = torch.zeros(nb, hkv, 16, d, dtype=torch.uint8, device="cuda")
    v8 = torch.zeros(nb, hkv, d, 16, dtype=torch.uint8, device="cuda")
    ks = torch.ones(nb, hkv, 16, device="cuda")
    vs = torch.ones(nb, hkv, 16, device="cuda")
    A.kv_write_fp8(src, slots_all, k8, v8, ks, vs, hq, hkv, d)
    kf, vf = A.dequantize_fp8_cache(k8, v8, ks, vs)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(1))
    maxb = max((n + 15) // 16 for n in kv_lens)
    bt = torch.zeros(len(kv_lens), maxb, dtype=torch.int32)
    p = 0
    for i, n in enumerate(kv_lens):
        for j in range((n + 15) // 16):
            bt[i, j] = perm[p]
            p += 1
    bt = bt.cuda()
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * d, device="cuda", generator=gen).bfloat16()
    out = torch.zeros(T, hq * d, device="cuda").bfloat16()
    qs = [0]
    for n in q_lens:
        qs.append(qs[-1] + n)
    ws, wr = A.build_work(q_lens, g, rows)
    ws_o = torch.empty(nsplit * T * hq * d, device="cuda")
    ws_l = torch.empty(nsplit * T * hq, device="cuda")
    A.paged_attention(q, k8, v8, bt, torch.tensor(qs, dtype=torch.int32, device="cuda"),
                      torch.tensor(kv_lens, dtype=torch.int32, device="cuda"),
                      torch.tensor(ws, dtype=torch.int32, device="cuda"),
                      torch.tensor(wr, dtype=torch.int32, device="cuda"), rows, hq, 0.125, out, nsplit, ws_o, ws_l,
                      ks, vs)
    ref = A.paged_attention_reference(q, kf, vf, bt, q_lens, kv_lens, hq, 0.125)
    err = (out.float() - ref).abs().max().item()
    assert err < 3e-2, err
    _check()
