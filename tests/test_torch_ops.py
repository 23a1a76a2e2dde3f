"""The native kernels as torch.library custom ops: schemas and fake implementations (CPU),
values, opcheck and torch.compile opacity (GPU)."""
import pytest
import torch

from granite_switch_b200.ops import gemm as G
from granite_switch_b200.ops import torch_ops as T


def test_registered_with_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    ops = T.ops()
    for name in ("switched_lora_linear", "lora_shrink", "paged_attention"):
        assert hasattr(ops, name)
    with FakeTensorMode():
        x = torch.empty(300, 256, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(512, 256, dtype=torch.bfloat16, device="cuda")
        a = torch.empty(64, 256, dtype=torch.bfloat16, device="cuda")
        lb = torch.empty(512, 32, dtype=torch.bfloat16, device="cuda")
        ra = torch.empty(300, dtype=torch.int32, device="cuda")
        for epi, shape, dt in ((G.EPI_STORE, (300, 512), torch.bfloat16), (G.EPI_SWIGLU, (300, 256), torch.bfloat16),
                               (G.EPI_F32, (300, 512), torch.float32)):
            y = ops.switched_lora_linear(x, w, a, lb, ra, None, 8, 4, [0, 512], epi, 1.0, None, 128)
            assert tuple(y.shape) == shape and y.dtype == dt
        assert tuple(ops.lora_shrink(x, a, ra, 8, 4, None).shape) == (300, 64)


def _case(m=200):
    torch.manual_seed(5)
    k, na, rank = 256, 3, 32
    bounds = [0, 256, 384, 512]
    x = (torch.randn(m, k, device="cuda")).bfloat16()
    w = (torch.randn(bounds[-1], k, device="cuda") * 0.05).bfloat16()
    ra = torch.randint(0, na + 1, (m,), device="cuda", dtype=torch.int32)
    a_all = torch.zeros(320, k, device="cuda", dtype=torch.bfloat16)
    a_all[:3 * na * rank] = (torch.randn(3 * na * rank, k, device="cuda") * 0.05).bfloat16()
    lb = (torch.randn(bounds[-1], na * rank, device="cuda") * 0.05).bfloat16()
    tiles = (m + 127) // 128
    mask = torch.zeros(tiles, dtype=torch.int64, device="cuda")
    for t in range(tiles):
        bits = 0
        for a in ra[t * 128:(t + 1) * 128].unique().tolist():
            if a > 0:
                bits |= 1 << (a - 1)
        mask[t] = bits
    return x, w, a_all, lb, ra, mask, rank, na, bounds


@pytest.mark.gpu
def test_switched_lora_linear_values_opcheck_and_compile():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200 import _native

    _native.native()
    x, w, a_all, lb, ra, mask, rank, na, bounds = _case()
    ops = T.ops()
    y = ops.switched_lora_linear(x, w, a_all, lb, ra, mask, rank, na, bounds, G.EPI_STORE, 1.0, None, 0)
    s = G.switched_gemm_reference(x, a_all, epi=G.EPI_MASK_ADAPTER, row_adapter=ra, mask_rank=rank,
                                  mask_num_adapters=na).to(torch.bfloat16)
    ref = G.switched_gemm_reference(x, w, s=s, lb=lb, rank=rank, num_adapters=na, slice_bounds=bounds)
    err = (y.float() - ref.float()).abs().max().item()
    assert err <= 2e-2 * ref.float().abs().max().item() + 1e-2
    torch.library.opcheck(T.switched_lora_linear,
                          (x, w, a_all, lb, ra, mask, rank, na, bounds, G.EPI_STORE, 1.0, None, 0),
                          test_utils=("test_schema", "test_faketensor"))

    def f(x):
        return ops.switched_lora_linear(x * 2, w, a_all, lb, ra, mask, rank, na, bounds, G.EPI_STORE, 0.5,
                                        None, 0) + 1

    got = torch.compile(f, backend="aot_eager", fullgraph=True)(x)
    torch.testing.assert_close(got, f(x), rtol=0, atol=0)
