"""fp8 block-scale format (CPU): scale-atom layout, exponent rule and round trip."""
import torch

from granite_switch_b200.ops import gemm_fp8 as F


def test_exponent_rule():
    amax = torch.tensor([0.0, 1e-30, 1.0, 448.0, 449.0, 896.0, 3.0e4])
    e = F._exponent(amax)
    scaled = amax / torch.ldexp(torch.ones(7), e)
    assert (scaled <= 448).all()
    # smallest such power of two: one step down would overflow (for non-tiny maxima)
    big = amax > 1e-20
    assert (amax[big] / torch.ldexp(torch.ones(7), e - 1)[big] > 448).all()
    assert int(e[0]) == -127 and int(e[3]) == 0 and int(e[4]) == 1 and int(e[5]) == 1


def test_atom_layout():
    """Byte 16 (r % 32) + 4 (r // 32) + j of an atom holds row r's scale, for j = 0..3."""
    rows, kb = 200, 3
    e = torch.randint(-20, 20, (rows, kb))
    atoms = F._atoms_from_exponents(e, 256)
    assert atoms.shape == (2, kb, 512)
    for r in (0, 1, 31, 32, 63, 64, 127, 128, 199):
        t, rr = divmod(r, 128)
        for j in range(4):
            assert int(atoms[t, 1, 16 * (rr % 32) + 4 * (rr // 32) + j]) == int(e[r, 1]) + 127
    assert torch.equal(F._exponents_from_atoms(atoms, rows), e)


def test_weight_round_trip():
    torch.manual_seed(0)
    n, k = 384, 256
    w = torch.randn(n, k) * (10.0 ** torch.randint(-2, 3, (n, 1)).float())
    w8, sfb = F.quantize_weight_fp8(w.bfloat16())
    assert w8.dtype == torch.uint8 and sfb.shape == (4, k // 128, 512)
    deq = F.dequantize_fp8(w8, sfb)
    blk = w.bfloat16().float().view(n // 128, 128, k // 128, 128).abs().amax(dim=(1, 3))
    tol = blk.repeat_interleave(128, 0).repeat_interleave(128, 1) / 16
    assert ((deq - w.bfloat16().float()).abs() <= tol).all()


def test_rows_reference_round_trip():
    torch.manual_seed(1)
    x = (torch.randn(77, 256) * 3).bfloat16()
    x8, sfa = F.quantize_rows_reference(x)
    assert sfa.shape == (1, 2, 512)
    deq = F.dequantize_fp8(x8, sfa)
    rel = (deq - x.float()).abs().max() / x.float().abs().max()
    assert rel < 1 / 16
