"""Tensor-parallel weight sharding (pack_linear) reproduces the unsharded projection.

Simulated on CPU: every rank's packed shard runs through the PyTorch statement
of the switched GEMM, and the ranks are combined the way the runtime combines
them (concatenation for column-parallel, summation for row-parallel).
"""
import pytest
import torch

from granite_switch_b200.models.packing import interleave_gate_up, pack_linear


def _apply(pl, x, idx):
    """fp32 statement of a packed projection incl. the per-row LoRA delta."""
    y = x @ pl.w.float().t()
    if pl.has_lora:
        local = torch.tensor(pl.remap)[idx]
        nl, rp, ns = pl.n_local, pl.rank, pl.num_slices
        s = x @ pl.a_all.float().t()
        for row in range(x.shape[0]):
            a = int(local[row])
            if a == 0:
                continue
            for sl in range(ns):
                cols = slice(pl.slice_bounds[sl], pl.slice_bounds[sl + 1])
                sv = s[row, (sl * nl + a - 1) * rp:(sl * nl + a) * rp]
                y[row, cols] += pl.lb.float()[cols, (a - 1) * rp:a * rp] @ sv
    return y


def _full(w, la, lb, x, idx, sizes):
    y = x @ w.t()
    off = 0
    for s, n in enumerate(sizes):
        for row in range(x.shape[0]):
            a = int(idx[row])
            if a:
                y[row, off:off + n] += (x[row] @ la[s][a - 1, 0].t()) @ lb[s][a - 1, 0].t()
        off += n
    return y


@pytest.mark.parametrize("tp", [2, 4])
def test_column_parallel_qkv(tp):
    torch.manual_seed(0)
    k, sizes, na, r = 64, [64, 32, 32], 3, 8
    w = torch.randn(sum(sizes), k)
    la = [torch.randn(na, 1, r, k) * 0.1 for _ in sizes]
    lb = [torch.randn(na, 1, n, r) * 0.1 for n in sizes]
    x = torch.randn(7, k)
    idx = torch.tensor([0, 1, 2, 3, 1, 0, 2])
    ref = _full(w, la, lb, x, idx, sizes)
    parts = []
    for rank in range(tp):
        pl = pack_linear(w, la, lb, sizes, na, "cpu", dtype=torch.float32, tp_rank=rank, tp_size=tp,
                         parallel="column")
        parts.append(_apply(pl, x, idx))
    # each rank holds its slice of q, of k and of v; compare slice by slice
    off = 0
    for s, n in enumerate(sizes):
        m = n // tp
        local_off = sum(nn // tp for nn in sizes[:s])
        for rank in range(tp):
            torch.testing.assert_close(parts[rank][:, local_off:local_off + m], ref[:, off + rank * m:off + (rank + 1) * m],
                                       rtol=1e-4, atol=1e-4)
        off += n


@pytest.mark.parametrize("tp", [2, 4])
def test_row_parallel_o(tp):
    torch.manual_seed(1)
    k, n, na, r = 64, 48, 2, 8
    w = torch.randn(n, k)
    la = [torch.randn(na, 1, r, k) * 0.1]
    lb = [torch.randn(na, 1, n, r) * 0.1]
    x = torch.randn(5, k)
    idx = torch.tensor([1, 0, 2, 2, 1])
    ref = _full(w, la, lb, x, idx, [n])
    total = torch.zeros_like(ref)
    for rank in range(tp):
        pl = pack_linear(w, la, lb, [n], na, "cpu", dtype=torch.float32, tp_rank=rank, tp_size=tp, parallel="row")
        xs = x[:, rank * (k // tp):(rank + 1) * (k // tp)]
        total += _apply(pl, xs, idx)
    torch.testing.assert_close(total, ref, rtol=1e-4, atol=1e-4)


def test_gate_up_interleave_roundtrip():
    w = torch.arange(2 * 256 * 3, dtype=torch.float32).view(512, 3)
    out = interleave_gate_up(w, 128)
    # tile t holds gate rows [64t, 64t+64) then up rows [256 + 64t, ...)
    assert torch.equal(out[:64], w[:64]) and torch.equal(out[64:128], w[256:320])
    assert torch.equal(out[128:192], w[64:128])


def test_adapter_not_touching_module_is_dropped():
    k, n, na, r = 32, 32, 3, 8
    la = [torch.zeros(na, 1, r, k)]
    lb = [torch.zeros(na, 1, n, r)]
    la[0][1] = 0.5
    lb[0][1] = 0.5
    pl = pack_linear(torch.randn(n, k), la, lb, [n], na, "cpu", dtype=torch.float32)
    assert pl.n_local == 1 and pl.remap == [0, 0, 1, 0]


def test_pipeline_layer_split():
    from granite_switch_b200.models.native import split_layers

    assert [split_layers(40, s, 2) for s in range(2)] == [(0, 20), (20, 40)]
    assert [split_layers(10, s, 3) for s in range(3)] == [(0, 4), (4, 7), (7, 10)]
    spans = [split_layers(7, s, 4) for s in range(4)]
    assert spans[0][0] == 0 and spans[-1][1] == 7
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


@pytest.mark.parametrize("fault", ["lora_a_wrong_shard", "lora_b_wrong_shard", "skip_row_reduce", "base_wrong_shard"])
def test_sharding_faults_are_detected(fault):
    """Sensitivity guard (reference: tests/vllm/_tp_integration_worker.py:56-144, GS_TP_FAULT):
    the row-parallel comparison must fail when a shard or the reduction is wrong."""
    torch.manual_seed(3)
    tp, k, n, na, r = 2, 64, 48, 2, 8
    w = torch.randn(n, k)
    la = [torch.randn(na, 1, r, k) * 0.3]
    lb = [torch.randn(na, 1, n, r) * 0.3]
    x = torch.randn(5, k)
    idx = torch.tensor([1, 0, 2, 2, 1])
    ref = _full(w, la, lb, x, idx, [n])
    pls = [pack_linear(w, la, lb, [n], na, "cpu", dtype=torch.float32, tp_rank=rk, tp_size=tp, parallel="row")
           for rk in range(tp)]
    if fault == "lora_a_wrong_shard":
        pls[0].a_all, pls[1].a_all = pls[1].a_all, pls[0].a_all
    elif fault == "lora_b_wrong_shard":
        pls[0].lb = pls[0].lb * 0.5
    elif fault == "base_wrong_shard":
        pls[0].w, pls[1].w = pls[1].w, pls[0].w
    parts = [_apply(pl, x[:, rk * (k // tp):(rk + 1) * (k // tp)], idx) for rk, pl in enumerate(pls)]
    total = parts[0] if fault == "skip_row_reduce" else parts[0] + parts[1]
    assert not torch.allclose(total, ref, rtol=1e-3, atol=1e-3)
