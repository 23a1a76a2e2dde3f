"""Block-scaled fp8 tcgen05 GEMM and its quantiser vs fp32 PyTorch oracles (GPU)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200 import _native

    _native.native()  # fail loudly if the extension is missing


def _rows(m, k, seed):
    """bf16 rows whose magnitudes span six decades, so every row and block gets its own scale."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=g)
    mag = 10.0 ** (torch.rand(m, k // 128, 1, device="cuda", generator=g) * 6 - 3)
    return (x.view(m, k // 128, 128) * mag).view(m, k).to(torch.bfloat16)


def _weights(n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.05
    mag = 2.0 ** torch.randint(-6, 7, (n // 128, 1, k // 128, 1), device="cuda", generator=g).float()
    return (w.view(n // 128, 128, k // 128, 128) * mag).view(n, k).to(torch.bfloat16)


def _close(a, b, tol=1e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= tol * ref, f"max err {err} vs max |ref| {ref}"


@pytest.mark.parametrize("m", [1, 77, 300])
def test_quantize_rows_matches_reference(m):
    """The device quantiser writes the same e4m3 bytes and scales as the PyTorch statement."""
    from granite_switch_b200.ops import gemm_fp8 as F

    k = 512
    x = _rows(m, k, seed=m)
    x8, sfa = F.quantize_rows_fp8(x)
    r8, rsfa = F.quantize_rows_reference(x)
    torch.cuda.synchronize()
    assert torch.equal(x8, r8)
    assert torch.equal(F._exponents_from_atoms(sfa, m), F._exponents_from_atoms(rsfa, m))
    deq = F.dequantize_fp8(x8, sfa)
    # e4m3 keeps 3 mantissa bits: relative error per element within 2^-4 of the block max
    blk = x.float().view(m, k // 128, 128).abs().amax(-1, keepdim=True)
    assert ((deq - x.float()).view(m, k // 128, 128).abs() <= blk / 16 + 1e-30).all()


@pytest.mark.parametrize("m", [1, 77, 128, 300])
@pytest.mark.parametrize("n", [256, 384, 1024])
@pytest.mark.parametrize("k", [128, 1024])
def test_fp8_gemm_store(m, n, k):
    """Every block's scale differs (both 128-row halves of a 256-row tile included), so a
    misplaced scale atom shows; partial token and weight tiles included."""
    from granite_switch_b200.ops import gemm_fp8 as F

    x = _rows(m, k, seed=1)
    w = _weights(n, k, seed=2)
    x8, sfa = F.quantize_rows_fp8(x)
    w8, sfb = F.quantize_weight_fp8(w)
    out = F.fp8_gemm(x8, sfa, w8, sfb, scale=0.5)
    ref = F.fp8_gemm_reference(x8, sfa, w8, sfb, scale=0.5)
    torch.cuda.synchronize()
    _close(out, ref)


def test_fp8_gemm_resadd_many_tiles_per_cta():
    """More tiles than SMs (each CTA reuses its accumulator and scale ring) with a residual add."""
    from granite_switch_b200.ops import gemm_fp8 as F

    m, n, k = 2048, 4096, 512
    x = _rows(m, k, seed=3)
    w = _weights(n, k, seed=4)
    res = (torch.randn(m, n, device="cuda") * 4).to(torch.bfloat16)
    x8, sfa = F.quantize_rows_fp8(x)
    w8, sfb = F.quantize_weight_fp8(w)
    out = F.fp8_gemm(x8, sfa, w8, sfb, epi=F.EPI_RESADD, residual=res, scale=0.25)
    ref = F.fp8_gemm_reference(x8, sfa, w8, sfb, epi=F.EPI_RESADD, residual=res, scale=0.25)
    torch.cuda.synchronize()
    _close(out, ref)


@pytest.mark.parametrize("m", [5, 300])
def test_fp8_gemm_lora_slices(m):
    """fp8 base + bf16 switched LoRA expand over three slices, adapters present per 128-row
    tile from the bitmask (one adapter absent)."""
    from granite_switch_b200.ops import gemm_fp8 as F

    torch.manual_seed(5)
    k, na, rank = 512, 5, 32
    bounds = [0, 1024, 1280, 1536]
    n = bounds[-1]
    x = _rows(m, k, seed=6)
    w = _weights(n, k, seed=7)
    row_adapter = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    row_adapter[row_adapter == 2] = 3
    s = torch.zeros(m, 3 * na * rank, device="cuda")
    for sl in range(3):
        for i in range(m):
            a = int(row_adapter[i])
            if a > 0:
                c = sl * na * rank + (a - 1) * rank
                s[i, c:c + rank] = torch.randn(rank, device="cuda")
    s = s.to(torch.bfloat16)
    lb = (torch.randn(n, na * rank, device="cuda") * 0.05).to(torch.bfloat16)
    tiles = (m + 127) // 128
    mask = torch.zeros(tiles, dtype=torch.int64, device="cuda")
    for t in range(tiles):
        bits = 0
        for a in row_adapter[t * 128:(t + 1) * 128].unique().tolist():
            if a > 0:
                bits |= 1 << (a - 1)
        mask[t] = bits
    x8, sfa = F.quantize_rows_fp8(x)
    w8, sfb = F.quantize_weight_fp8(w)
    kw = dict(s=s, lb=lb, rank=rank, num_adapters=na, slice_bounds=bounds)
    out = F.fp8_gemm(x8, sfa, w8, sfb, tile_mask=mask, **kw)
    ref = F.fp8_gemm_reference(x8, sfa, w8, sfb, **kw)
    torch.cuda.synchronize()
    _close(out, ref)
