"""Allocation-free decode attention, called through its exported C symbol.

``gsb_decode_attention_noalloc`` keeps the split-KV partial results in a
static device array instead of caller workspaces. Two calls in a row (with
different shapes, so the second sees the first one's leftovers in the shared
scratch) must match the regular ``paged_attention`` op with explicit
workspaces, and a request larger than the fixed scratch must be rejected.
The file name sorts last so the test also runs after the rest of the suite.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, EINVAL, ETOOBIG = 0, 1, 2
SCRATCH_FLOATS = 1 << 20


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200 import _native

    _native.native()  # imports the in-tree extension (fails loudly if it is missing)
    import granite_switch_b200._C as C

    so = ctypes.CDLL(C.__file__)  # same library handle as the imported module
    fn = so.gsb_decode_attention_noalloc
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    fn.argtypes = [vp, i64, vp, vp, i64, i32, i32, vp, i64, vp, vp, vp, vp, i32, i32, i32, ctypes.c_float, i32,
                   vp, i64, vp, vp, ctypes.c_char_p, ctypes.c_size_t]
    fn.restype = ctypes.c_int
    return fn


def _case(d, hq, hkv, q_lens, kv_lens, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    nblk = sum((l + 15) // 16 for l in kv_lens) + 3
    kc = torch.randn(nblk, hkv, 16, d, generator=g).bfloat16().cuda()
    vc = torch.randn(nblk, hkv, 16, d, generator=g).bfloat16().cuda()
    perm = torch.randperm(nblk, generator=g).tolist()
    maxb = max((l + 15) // 16 for l in kv_lens)
    bt = torch.zeros(len(kv_lens), maxb, dtype=torch.int32)
    p = 0
    for i, l in enumerate(kv_lens):
        for j in range((l + 15) // 16):
            bt[i, j] = perm[p]
            p += 1
    T = sum(q_lens)
    q = torch.randn(T, (hq + 2 * hkv) * d, generator=g).bfloat16().cuda()  # q at the front of a qkv row
    qs = [0]
    for l in q_lens:
        qs.append(qs[-1] + l)
    from granite_switch_b200.ops import attention as A

    ws, wr = A.build_work(q_lens, hq // hkv, 16)
    i32 = dict(dtype=torch.int32, device="cuda")
    return dict(q=q, kc=kc, vc=vc, bt=bt.cuda(), qs=torch.tensor(qs, **i32), kv=torch.tensor(kv_lens, **i32),
                ws=torch.tensor(ws, **i32), wr=torch.tensor(wr, **i32), T=T, d=d, hq=hq, hkv=hkv,
                q_lens=q_lens, kv_lens=kv_lens)


def _regular(c, nsplit, scale):
    from granite_switch_b200.ops import attention as A

    out = torch.zeros(c["T"], c["hq"] * c["d"], device="cuda").bfloat16()
    ws_o = torch.empty(nsplit * c["T"] * c["hq"] * c["d"], device="cuda")
    ws_l = torch.empty(nsplit * c["T"] * c["hq"], device="cuda")
    A.paged_attention(c["q"], c["kc"], c["vc"], c["bt"], c["qs"], c["kv"], c["ws"], c["wr"], 16, c["hq"], scale,
                      out, nsplit, ws_o, ws_l)
    return out


def _noalloc(fn, c, nsplit, scale, out, err):
    msg = ctypes.create_string_buffer(512)
    rc = fn(c["q"].data_ptr(), c["q"].stride(0), c["kc"].data_ptr(), c["vc"].data_ptr(), c["kc"].shape[0],
            c["hkv"], c["d"], c["bt"].data_ptr(), c["bt"].stride(0), c["qs"].data_ptr(), c["kv"].data_ptr(),
            c["ws"].data_ptr(), c["wr"].data_ptr(), c["ws"].numel(), c["T"], c["hq"], scale, nsplit,
            out.data_ptr(), out.stride(0), err.data_ptr(), torch.cuda.current_stream().cuda_stream, msg, 512)
    return rc, msg.value.decode()


def test_noalloc_matches_regular_twice(lib):
    from granite_switch_b200._native import check_errors
    from granite_switch_b200.ops import attention as A

    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    cases = [
        (_case(128, 32, 8, [1, 1, 2, 1], [1, 900, 2500, 4100], seed=1), 16, 0.088),
        (_case(128, 32, 8, [1, 1], [300, 77], seed=2), 5, 0.088),
    ]
    for i, (c, nsplit, scale) in enumerate(cases):
        ref = _regular(c, nsplit, scale)
        out = torch.full_like(ref, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc, msg = _noalloc(lib, c, nsplit, scale, out, err)
        torch.cuda.synchronize()
        assert rc == OK, msg
        if i > 0:  # the first call on the device did its one-time set-up
            assert torch.cuda.mem_get_info()[0] == free_before
        assert int(err.abs().sum()) == 0
        assert torch.allclose(out.float(), ref.float(), atol=2e-3, rtol=0), (out.float() - ref.float()).abs().max()
        oracle = A.paged_attention_reference(c["q"], c["kc"], c["vc"], c["bt"], c["q_lens"], c["kv_lens"], c["hq"],
                                             scale)
        assert (out.float() - oracle).abs().max().item() < 3e-2
    check_errors(torch.device("cuda"))


def test_noalloc_head_dim_64_single_split(lib):
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    for nsplit in (1, 3):
        c = _case(64, 8, 2, [1, 4, 1], [40, 333, 1025], seed=3)
        ref = _regular(c, nsplit, 0.125)
        out = torch.zeros_like(ref)
        rc, msg = _noalloc(lib, c, nsplit, 0.125, out, err)
        torch.cuda.synchronize()
        assert rc == OK, msg
        assert torch.allclose(out.float(), ref.float(), atol=2e-3, rtol=0)
    assert int(err.abs().sum()) == 0


def test_noalloc_rejects_oversized_split(lib):
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    c = _case(128, 32, 8, [1] * 40, [64] * 40, seed=4)
    assert 64 * c["T"] * 32 * 129 > SCRATCH_FLOATS
    out = torch.zeros(c["T"], 32 * 128, device="cuda").bfloat16()
    rc, msg = _noalloc(lib, c, 64, 0.088, out, err)
    torch.cuda.synchronize()
    assert rc == ETOOBIG
    assert "scratch" in msg and str(SCRATCH_FLOATS) in msg
    assert int(out.float().abs().sum()) == 0  # nothing was launched
    rc, msg = _noalloc(lib, c, 0, 0.088, out, err)
    assert rc == EINVAL and "nsplit" in msg
