"""tcgen05 switched GEMM vs the fp32 PyTorch oracle (GPU)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(*shape, scale=1.0, dev="cuda"):
    return (torch.randn(*shape, device=dev) * scale).to(torch.bfloat16)


def _close(a, b, tol=2e-2):
    a = a.float()
    b = b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= tol * ref + 1e-2, f"max err {err} vs max |ref| {ref}"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200 import _native

    _native.native()  # fail loudly if the extension is missing


@pytest.mark.parametrize("m", [1, 77, 128, 300])
@pytest.mark.parametrize("bn", [64, 128, 256])
def test_plain_store(m, bn):
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(0)
    n, k = 512, 320
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    out = G.switched_gemm(x, w, bn=bn)
    torch.cuda.synchronize()
    _close(out, G.switched_gemm_reference(x, w))
    from granite_switch_b200._native import check_errors

    check_errors(x.device)


@pytest.mark.parametrize("bn", [64, 256])
def test_f32_and_resadd(bn):
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(1)
    m, n, k = 200, 256, 256
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    out = G.switched_gemm(x, w, epi=G.EPI_F32, scale=0.5, bn=bn)
    _close(out, G.switched_gemm_reference(x, w, epi=G.EPI_F32, scale=0.5))
    res = _rand(m, n)
    res_copy = res.clone()
    G.switched_gemm(x, w, res, epi=G.EPI_RESADD, residual=res, scale=0.22, bn=bn)
    _close(res, G.switched_gemm_reference(x, w, epi=G.EPI_RESADD, residual=res_copy, scale=0.22))


@pytest.mark.parametrize("m", [5, 130])
def test_lora_expand_fused(m):
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(2)
    k, na, rank = 256, 3, 32
    bounds = [0, 256, 384, 512]  # q | k | v slices
    n = bounds[-1]
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    row_adapter = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    a_all = torch.zeros(320, k, device="cuda", dtype=torch.bfloat16)  # 288 rows padded to 64
    a_all[:3 * na * rank] = _rand(3 * na * rank, k, scale=0.05)
    s = G.lora_shrink(x, a_all, row_adapter, rank, na)
    s_ref = G.switched_gemm_reference(x, a_all, epi=G.EPI_MASK_ADAPTER, row_adapter=row_adapter,
                                      mask_rank=rank, mask_num_adapters=na)
    _close(s[:, :288], s_ref[:, :288])
    lb = _rand(n, na * rank, scale=0.05)
    tiles = (m + 127) // 128
    mask = torch.zeros(tiles, dtype=torch.int64, device="cuda")
    for t in range(tiles):
        ids = row_adapter[t * 128:(t + 1) * 128]
        bits = 0
        for a in ids.unique().tolist():
            if a > 0:
                bits |= 1 << (a - 1)
        mask[t] = bits
    out = G.switched_gemm(x, w, s=s, lb=lb, tile_mask=mask, rank=rank, num_adapters=na,
                          slice_bounds=bounds, bn=128)
    ref = G.switched_gemm_reference(x, w, s=s, lb=lb, rank=rank, num_adapters=na,
                                    slice_bounds=bounds)
    _close(out, ref)
    # shrink restricted to the adapters present per tile gives the same projection
    s2 = torch.full_like(s, float("nan"))
    G.lora_shrink(x, a_all, row_adapter, rank, na, out=s2, tile_mask=mask)
    out2 = G.switched_gemm(x, w, s=s2, lb=lb, tile_mask=mask, rank=rank, num_adapters=na,
                           slice_bounds=bounds, bn=128)
    _close(out2, ref)


def test_swiglu_split_lora():
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(3)
    m, k, na, rank, bn = 150, 128, 2, 32, 128
    n = 512
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    row_adapter = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    s = _rand(m, 2 * na * rank, scale=0.5)
    # zero columns not owned by the row's adapter, as the shrink would
    cols = torch.arange(2 * na * rank, device="cuda")
    keep = ((cols // rank) % na + 1).unsqueeze(0) == row_adapter.long().unsqueeze(1)
    s = (s.float() * keep).to(torch.bfloat16)
    lb = _rand(n, na * rank, scale=0.05)
    out = G.switched_gemm(x, w, epi=G.EPI_SWIGLU, s=s, lb=lb, rank=rank, num_adapters=na,
                          slice_bounds=[0, n], bn=bn)
    ref = G.switched_gemm_reference(x, w, epi=G.EPI_SWIGLU, s=s, lb=lb, rank=rank,
                                    num_adapters=na, swiglu_tile=bn)
    _close(out, ref)


def _tile_mask(row_adapter, m):
    tiles = (m + 127) // 128
    mask = torch.zeros(tiles, dtype=torch.int64, device="cuda")
    for t in range(tiles):
        bits = 0
        for a in row_adapter[t * 128:(t + 1) * 128].unique().tolist():
            if a > 0:
                bits |= 1 << (a - 1)
        mask[t] = bits
    return mask


class _PairMinM:
    """Temporarily route GEMMs with M >= m to the CTA-pair kernel (m < 0: never)."""

    def __init__(self, m):
        self.m = m

    def __enter__(self):
        from granite_switch_b200._native import native

        self.old = native().gemm_pair_min_m(self.m)

    def __exit__(self, *a):
        from granite_switch_b200._native import native

        native().gemm_pair_min_m(self.old)


@pytest.mark.parametrize("m", [256, 300, 513, 1000])
def test_pair_store_and_resadd(m):
    """CTA-pair (cta_group::2) tiles, including a pair whose second CTA is past M."""
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(4)
    n, k = 768, 512
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    with _PairMinM(1):
        out = G.switched_gemm(x, w, bn=256)
        res = _rand(m, n)
        res_copy = res.clone()
        G.switched_gemm(x, w, res, epi=G.EPI_RESADD, residual=res, scale=0.22, bn=256)
    torch.cuda.synchronize()
    check_errors(x.device)
    _close(out, G.switched_gemm_reference(x, w))
    _close(res, G.switched_gemm_reference(x, w, epi=G.EPI_RESADD, residual=res_copy, scale=0.22))
    with _PairMinM(-1), _SplitK(0):  # same accumulation order: no split of K on the single-CTA side
        single = G.switched_gemm(x, w, bn=256)
    assert torch.equal(out, single), "pair and single-CTA tiles must agree bit for bit"


@pytest.mark.parametrize("m", [384, 700])
def test_pair_lora_expand(m):
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(5)
    k, na, rank = 256, 5, 32
    bounds = [0, 512, 768, 1024]
    n = bounds[-1]
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    row_adapter = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    row_adapter[:128] = 0  # one all-base tile next to mixed tiles
    cols = 3 * na * rank
    s = _rand(m, cols, scale=0.5)
    keep = ((torch.arange(cols, device="cuda") // rank) % na + 1).unsqueeze(0) == row_adapter.long().unsqueeze(1)
    s = (s.float() * keep).to(torch.bfloat16)
    lb = _rand(n, na * rank, scale=0.05)
    mask = _tile_mask(row_adapter, m)
    with _PairMinM(1):
        out = G.switched_gemm(x, w, s=s, lb=lb, tile_mask=mask, rank=rank, num_adapters=na,
                              slice_bounds=bounds, bn=256)
    torch.cuda.synchronize()
    check_errors(x.device)
    ref = G.switched_gemm_reference(x, w, s=s, lb=lb, rank=rank, num_adapters=na, slice_bounds=bounds)
    _close(out, ref)


@pytest.mark.parametrize("m", [256, 650])
def test_pair_swiglu_split_lora(m):
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(6)
    k, na, rank, bn = 256, 3, 64, 256
    n = 1024
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    row_adapter = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    s = _rand(m, 2 * na * rank, scale=0.5)
    cols = torch.arange(2 * na * rank, device="cuda")
    keep = ((cols // rank) % na + 1).unsqueeze(0) == row_adapter.long().unsqueeze(1)
    s = (s.float() * keep).to(torch.bfloat16)
    lb = _rand(n, na * rank, scale=0.05)
    mask = _tile_mask(row_adapter, m)
    with _PairMinM(1):
        out = G.switched_gemm(x, w, epi=G.EPI_SWIGLU, s=s, lb=lb, tile_mask=mask, rank=rank,
                              num_adapters=na, slice_bounds=[0, n], bn=bn)
    torch.cuda.synchronize()
    check_errors(x.device)
    ref = G.switched_gemm_reference(x, w, epi=G.EPI_SWIGLU, s=s, lb=lb, rank=rank, num_adapters=na,
                                    swiglu_tile=bn)
    _close(out, ref)
    with _PairMinM(-1):
        single = G.switched_gemm(x, w, epi=G.EPI_SWIGLU, s=s, lb=lb, tile_mask=mask, rank=rank,
                                 num_adapters=na, slice_bounds=[0, n], bn=bn)
    _close(out, single, tol=1e-2)


@pytest.mark.parametrize("pair", [1, -1])
def test_many_tiles_per_cta(pair):
    """Enough tiles that every CTA drains several accumulators through its staging buffers."""
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(7)
    m, n, k = 2304, 2048, 256
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    with _PairMinM(pair):
        out = G.switched_gemm(x, w, bn=256)
        res = _rand(m, n)
        res_copy = res.clone()
        G.switched_gemm(x, w, res, epi=G.EPI_RESADD, residual=res, scale=0.5, bn=256)
        wg = _rand(2 * n, k, scale=0.05)
        act = G.switched_gemm(x, wg, epi=G.EPI_SWIGLU, bn=256)
    torch.cuda.synchronize()
    check_errors(x.device)
    _close(out, G.switched_gemm_reference(x, w))
    _close(res, G.switched_gemm_reference(x, w, epi=G.EPI_RESADD, residual=res_copy, scale=0.5))
    _close(act, G.switched_gemm_reference(x, wg, epi=G.EPI_SWIGLU, swiglu_tile=256))


@pytest.mark.parametrize("pair", [1, -1])
@pytest.mark.parametrize("m", [600, 1100])
def test_swiglu_lora_engine_layout(pair, m):
    """gate/up as the engine runs it: rank 32 (one LoRA K block), S a strided view of a wider
    buffer, base-only tiles before the adapter rows."""
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(8)
    k, na, rank, bn, n = 256, 3, 32, 256, 1024
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    row_adapter = torch.zeros(m, device="cuda", dtype=torch.int32)
    row_adapter[m // 2:] = torch.randint(0, na + 1, (m - m // 2,), device="cuda", dtype=torch.int32)
    cols = 2 * na * rank
    s_buf = torch.zeros(m, 320, device="cuda", dtype=torch.bfloat16)
    s = s_buf[:, :cols]
    sv = _rand(m, cols, scale=0.5)
    keep = ((torch.arange(cols, device="cuda") // rank) % na + 1).unsqueeze(0) == row_adapter.long().unsqueeze(1)
    s.copy_((sv.float() * keep).to(torch.bfloat16))
    lb = _rand(n, na * rank, scale=0.05)
    mask = _tile_mask(row_adapter, m)
    with _PairMinM(pair):
        out = G.switched_gemm(x, w, epi=G.EPI_SWIGLU, s=s, lb=lb, tile_mask=mask, rank=rank,
                              num_adapters=na, slice_bounds=[0, n], bn=bn)
    torch.cuda.synchronize()
    check_errors(x.device)
    ref = G.switched_gemm_reference(x, w, epi=G.EPI_SWIGLU, s=s.contiguous(), lb=lb, rank=rank,
                                    num_adapters=na, swiglu_tile=bn)
    _close(out, ref)


@pytest.mark.parametrize("epi", ["store", "swiglu"])
def test_pair_expand_with_tile_restricted_shrink(epi):
    """The tile-restricted shrink leaves S columns of absent adapters unwritten (NaN here);
    a pair whose two 128-row tiles hold different adapters must not read them."""
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(9)
    m, k, na, rank = 700, 256, 3, 32
    n = 1024
    x = _rand(m, k)
    w = _rand(n, k, scale=0.05)
    row_adapter = torch.zeros(m, device="cuda", dtype=torch.int32)
    row_adapter[128:256] = 1          # tile 1: adapter 1 only (its pair partner, tile 0, is base)
    row_adapter[256:384] = 2          # tiles 2 / 3 hold different adapters
    row_adapter[400:500] = 3
    row_adapter[640:] = 2             # a partial last tile
    mask = _tile_mask(row_adapter, m)
    slices = 2 if epi == "swiglu" else 1
    a_rows = (slices * na * rank + 63) // 64 * 64
    a_all = torch.zeros(a_rows, k, device="cuda", dtype=torch.bfloat16)
    a_all[: slices * na * rank] = _rand(slices * na * rank, k, scale=0.05)
    s = torch.full((m, a_rows), float("nan"), device="cuda", dtype=torch.bfloat16)
    G.lora_shrink(x, a_all, row_adapter, rank, na, out=s, tile_mask=mask)
    s_full = G.lora_shrink(x, a_all, row_adapter, rank, na)
    lb = _rand(n, na * rank, scale=0.05)
    kw = dict(s=s, lb=lb, tile_mask=mask, rank=rank, num_adapters=na, bn=256)
    with _PairMinM(1):
        if epi == "swiglu":
            out = G.switched_gemm(x, w, epi=G.EPI_SWIGLU, slice_bounds=[0, n], **kw)
        else:
            out = G.switched_gemm(x, w, slice_bounds=[0, n], **kw)
    torch.cuda.synchronize()
    check_errors(x.device)
    if epi == "swiglu":
        ref = G.switched_gemm_reference(x, w, epi=G.EPI_SWIGLU, s=s_full, lb=lb, rank=rank, num_adapters=na,
                                        swiglu_tile=256)
    else:
        ref = G.switched_gemm_reference(x, w, s=s_full, lb=lb, rank=rank, num_adapters=na, slice_bounds=[0, n])
    assert not torch.isnan(out.float()).any()
    _close(out, ref)


@pytest.mark.parametrize("epi", ["store", "swiglu"])
def test_grouped_gemm(epi):
    """Grouped mode: each 128-row tile multiplies its expert's weights; -1 tiles are left untouched."""
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(10)
    e, n, k = 5, 512, 256
    tiles = torch.tensor([3, 0, 0, 4, -1, 2, -1], dtype=torch.int32, device="cuda")
    m = 128 * tiles.numel()
    x = _rand(m, k)
    w = _rand(e, n, k, scale=0.05)
    out = torch.full((m, n // 2 if epi == "swiglu" else n), 7.0, device="cuda", dtype=torch.bfloat16)
    if epi == "swiglu":
        G.switched_gemm(x, w, out, epi=G.EPI_SWIGLU, bn=256, tile_expert=tiles)
    else:
        G.switched_gemm(x, w, out, tile_expert=tiles)
    torch.cuda.synchronize()
    check_errors(x.device)
    for t, ex in enumerate(tiles.tolist()):
        rows = slice(128 * t, 128 * (t + 1))
        if ex < 0:
            assert bool((out[rows].float() == 7.0).all())
            continue
        if epi == "swiglu":
            ref = G.switched_gemm_reference(x[rows], w[ex], epi=G.EPI_SWIGLU, swiglu_tile=256)
        else:
            ref = G.switched_gemm_reference(x[rows], w[ex])
        _close(out[rows], ref)


class _DecodeMaxM:
    """Temporarily set the largest M of the operand-swapped decode kernel (0: off)."""

    def __init__(self, v):
        self.v = v

    def __enter__(self):
        from granite_switch_b200._native import native

        self.old = native().gemm_decode_max_m(self.v)
        return self

    def __exit__(self, *a):
        from granite_switch_b200._native import native

        native().gemm_decode_max_m(self.old)


class _SplitK:
    """Temporarily set the output-tile count below which single-CTA GEMMs split K (0: never)."""

    def __init__(self, v):
        self.v = v

    def __enter__(self):
        from granite_switch_b200._native import native

        self.old = native().gemm_splitk_max_tiles(self.v)

    def __exit__(self, *a):
        from granite_switch_b200._native import native

        native().gemm_splitk_max_tiles(self.old)


@pytest.mark.parametrize("epi", ["store", "resadd", "swiglu", "f32"])
@pytest.mark.parametrize("m,k", [(1, 4096), (77, 12800), (200, 4096)])
def test_split_k_decode_shapes(epi, m, k):
    """Decode-sized GEMMs split K across CTAs (fp32 parts + reduce epilogue): equal to the
    unsplit kernel and to the fp32 oracle, with the LoRA expand in the last part."""
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(7)
    n, na, rank = 4096, 3, 32
    x = _rand(m, k)
    w = _rand(n, k, scale=0.02)
    row_adapter = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    lb = _rand(n, na * rank, scale=0.05)
    width = (2 if epi == "swiglu" else 1) * na * rank  # SwiGLU: gate and up shrink slices
    cols = torch.arange(width, device="cuda")
    keep = ((cols // rank) % na + 1).unsqueeze(0) == row_adapter.long().unsqueeze(1)
    s = (_rand(m, width, scale=0.5).float() * keep).to(torch.bfloat16)
    mask = _tile_mask(row_adapter, m)
    res = _rand(m, n)
    kind = {"store": G.EPI_STORE, "resadd": G.EPI_RESADD, "swiglu": G.EPI_SWIGLU, "f32": G.EPI_F32}[epi]
    bn = 64 if epi != "swiglu" else 128
    kw = dict(epi=kind, residual=res if epi == "resadd" else None, scale=0.5, s=s, lb=lb, tile_mask=mask,
              rank=rank, num_adapters=na, slice_bounds=[0, n], bn=bn)
    with _DecodeMaxM(0), _SplitK(74):  # the general kernel's split-K (decode kernel off)
        split = G.switched_gemm(x, w, **kw)
    with _DecodeMaxM(0), _SplitK(0):
        whole = G.switched_gemm(x, w, **kw)
    ref = G.switched_gemm_reference(x, w, epi=kind, residual=kw["residual"], scale=0.5, s=s, lb=lb, rank=rank,
                                    num_adapters=na, slice_bounds=[0, n], swiglu_tile=bn)
    _close(split, ref)
    _close(split, whole)
    from granite_switch_b200._native import check_errors

    check_errors(torch.device("cuda", 0))


def _masked_s(m, width, rank, na, row_adapter):
    cols = torch.arange(width, device="cuda")
    keep = ((cols // rank) % na + 1).unsqueeze(0) == row_adapter.long().unsqueeze(1)
    return (_rand(m, width, scale=0.5).float() * keep).to(torch.bfloat16)


@pytest.mark.parametrize("epi", ["store", "resadd", "swiglu"])
@pytest.mark.parametrize("m", [1, 5, 77, 130, 222, 256])
@pytest.mark.parametrize("n,k", [(512, 320), (4096, 4096), (1024, 12800)])
def test_decode_gemm_epilogues(epi, m, n, k):
    """Operand-swapped decode kernel (M <= 256; one CTA per 128 weight rows, K split over a
    cluster and reduced through distributed shared memory): equal to the fp32 oracle and to
    the general kernel, and bitwise deterministic."""
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(11)
    x = _rand(m, k)
    w = _rand(n, k, scale=0.02)
    res = _rand(m, n)
    kind = {"store": G.EPI_STORE, "resadd": G.EPI_RESADD, "swiglu": G.EPI_SWIGLU}[epi]
    bn = 128 if epi == "swiglu" else None
    out_cols = n // 2 if epi == "swiglu" else n

    def run():
        o = torch.empty(m, out_cols, device="cuda", dtype=torch.bfloat16)
        if epi == "resadd":
            o.copy_(res)
        G.switched_gemm(x, w, o, epi=kind, residual=o if epi == "resadd" else None, scale=0.5, bn=bn)
        return o

    with _DecodeMaxM(256):
        a = run()
        b = run()
    with _DecodeMaxM(0):
        general = run()
    ref = G.switched_gemm_reference(x, w, epi=kind, residual=res if epi == "resadd" else None, scale=0.5,
                                    swiglu_tile=128)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    _close(a, ref)
    _close(a, general)
    from granite_switch_b200._native import check_errors

    check_errors(torch.device("cuda", 0))


@pytest.mark.parametrize("m", [3, 100, 222])
@pytest.mark.parametrize("k", [512, 4096])
def test_decode_gemm_lora_slices(m, k):
    """qkv-shaped switched GEMM on the decode kernel: the shrink (adapter-mask epilogue, tiles of
    absent adapters skipped) and the expand over three slices, LoRA blocks spread over the
    cluster's K parts; against the oracle and the general kernel."""
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(12)
    na, rank = 5, 32
    bounds = [0, 1024, 1280, 1536]
    n = bounds[-1]
    x = _rand(m, k)
    w = _rand(n, k, scale=0.02)
    row_adapter = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    row_adapter[row_adapter == 2] = 3  # one adapter absent: its shrink tiles are skipped
    width = 3 * na * rank
    a_all = torch.zeros((width + 63) // 64 * 64, k, device="cuda", dtype=torch.bfloat16)
    a_all[:width] = _rand(width, k, scale=0.02)
    lb = _rand(n, na * rank, scale=0.05)
    mask = _tile_mask(row_adapter, m)
    s_ref = G.switched_gemm_reference(x, a_all, epi=G.EPI_MASK_ADAPTER, row_adapter=row_adapter,
                                      mask_rank=rank, mask_num_adapters=na)
    with _DecodeMaxM(256):
        s = torch.full((m, a_all.shape[0]), float("nan"), device="cuda", dtype=torch.bfloat16)
        G.lora_shrink(x, a_all, row_adapter, rank, na, out=s, tile_mask=mask)
        out = G.switched_gemm(x, w, s=s, lb=lb, tile_mask=mask, rank=rank, num_adapters=na, slice_bounds=bounds)
        out2 = G.switched_gemm(x, w, s=s, lb=lb, tile_mask=mask, rank=rank, num_adapters=na, slice_bounds=bounds)
    present = [a for a in range(1, na + 1) if (row_adapter == a).any()]
    for a in present:  # columns of present adapters are written for every token
        for sl in range(3):
            c0 = sl * na * rank + (a - 1) * rank
            _close(s[:, c0:c0 + rank], s_ref[:, c0:c0 + rank])
    ref = G.switched_gemm_reference(x, w, s=s_ref, lb=lb, rank=rank, num_adapters=na, slice_bounds=bounds)
    with _DecodeMaxM(0):
        s_gen = G.lora_shrink(x, a_all, row_adapter, rank, na, tile_mask=mask)
        general = G.switched_gemm(x, w, s=s_gen, lb=lb, tile_mask=mask, rank=rank, num_adapters=na,
                                  slice_bounds=bounds)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    _close(out, ref)
    _close(out, general)
    from granite_switch_b200._native import check_errors

    check_errors(torch.device("cuda", 0))


@pytest.mark.parametrize("m", [1, 5, 96])
@pytest.mark.parametrize("rank,na,slices", [(32, 12, 3), (8, 3, 3), (16, 5, 1)])
def test_small_shrink_matches_masked_gemm(m, rank, na, slices):
    """The CUDA-core shrink for a few tokens writes what the tensor-core kernel's adapter-mask
    epilogue writes: each row's own adapter columns in every slice (A padded with zero rows,
    so a last partial slice exists when na * rank does not divide 64), zeros elsewhere and for
    base rows."""
    from granite_switch_b200._native import native
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(m + rank)
    k = 1024
    width = slices * na * rank
    n = (width + 63) // 64 * 64
    x = _rand(m, k)
    a_all = torch.zeros(n, k, device="cuda", dtype=torch.bfloat16)
    a_all[:width] = _rand(width, k, scale=0.05)
    ra = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    s = torch.full((m, n), 7.0, device="cuda", dtype=torch.bfloat16)  # every column must be written
    native().lora_shrink_small(x, a_all, ra, s, rank, na)
    ref = G.switched_gemm_reference(x, a_all, epi=G.EPI_MASK_ADAPTER, row_adapter=ra, mask_rank=rank,
                                    mask_num_adapters=na)
    tc = G.switched_gemm(x, a_all, epi=G.EPI_MASK_ADAPTER, row_adapter=ra, mask_rank=rank, mask_num_adapters=na,
                         bn=64)
    torch.cuda.synchronize()
    _close(s, ref)
    _close(s, tc)
    cols = torch.arange(n, device="cuda")
    keep = ((cols // rank) % na + 1).unsqueeze(0) == ra.long().unsqueeze(1)
    assert (s.float()[~keep] == 0).all()  # other adapters' and base rows' columns written as zeros


class _PDL:
    """Temporarily launch the decode GEMMs as programmatic dependents (or not)."""

    def __init__(self, on):
        self.on = on

    def __enter__(self):
        from granite_switch_b200._native import native

        self.old = native().set_pdl(self.on)

    def __exit__(self, *a):
        from granite_switch_b200._native import native

        native().set_pdl(self.old)


@pytest.mark.parametrize("m", [16, 130, 222])
def test_pdl_chain_matches_serial(m):
    """A decode layer's chain of dependent kernels (RMSNorm -> LoRA shrink -> projection
    with the LoRA expand -> gate/up with SwiGLU -> down with the residual add), each GEMM
    launched as a programmatic dependent of the kernel before it, eagerly and replayed from
    a CUDA graph, equals the same chain launched in plain stream order bit for bit."""
    from granite_switch_b200._native import check_errors, native
    from granite_switch_b200.ops import elementwise as E
    from granite_switch_b200.ops import gemm as G

    torch.manual_seed(11)
    h0 = _rand(m, 4096)
    norm_w = (1.0 + 0.1 * torch.randn(4096, device="cuda")).bfloat16()
    na, rank = 12, 32
    a_all = _rand(na * rank, 4096, scale=0.02)
    w_o = _rand(4096, 4096, scale=0.02)
    lb = _rand(4096, na * rank, scale=0.05)
    w_gu = _rand(2 * 12800, 4096, scale=0.02)
    w_d = _rand(4096, 12800, scale=0.02)
    ids = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    mask = _tile_mask(ids, m)
    x = torch.empty(m, 4096, device="cuda", dtype=torch.bfloat16)
    s = torch.empty(m, na * rank, device="cuda", dtype=torch.bfloat16)
    act = torch.empty(m, 12800, device="cuda", dtype=torch.bfloat16)

    def chain(h):
        E.rmsnorm(h, norm_w, 1e-5, out=x)
        G.lora_shrink(x, a_all, ids, rank, na, out=s, tile_mask=mask)
        G.switched_gemm(x, w_o, h, epi=G.EPI_RESADD, residual=h, s=s, lb=lb, tile_mask=mask, rank=rank,
                        num_adapters=na)
        E.rmsnorm(h, norm_w, 1e-5, out=x)
        G.switched_gemm(x, w_gu, act, epi=G.EPI_SWIGLU, bn=128)
        G.switched_gemm(act, w_d, h, epi=G.EPI_RESADD, residual=h)
        return h

    with _PDL(False):
        ref = chain(h0.clone())
        torch.cuda.synchronize()
    with _PDL(True):
        eager = chain(h0.clone())
        torch.cuda.synchronize()
        hg = h0.clone()
        chain(hg.clone())  # warm-up outside capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            chain(hg)
        results = []
        for _ in range(3):
            hg.copy_(h0)
            graph.replay()
            torch.cuda.synchronize()
            results.append(hg.clone())
        del graph
    check_errors(torch.device("cuda", 0))
    assert native().gemm_decode_plan(m, 4096, 4096, G.EPI_RESADD, 0)[0] > 0  # the decode kernel ran
    assert torch.equal(eager, ref)
    for r in results:
        assert torch.equal(r, ref)
