"""Exact latest-wins routing vs the coded-memory algorithm it replaces."""
import random

import pytest
import torch

from granite_switch_b200.routing import (
    apply_token_exchange,
    build_control_to_substitute_lut,
    expert_table,
    probe_slot_mask,
    route_flat,
    route_sequence,
    split_probe_stream,
)
from granite_switch_b200.routing.codebook import KerdockDGCodeGenerator, verify_coherence
from granite_switch_b200.routing.coded_switch import coded_switch_route


@pytest.fixture(scope="module")
def codebook():
    return KerdockDGCodeGenerator(6).precompute_codebook()


def _stream(rng, length, ctrl, p=0.08, vocab=300):
    ids = []
    for _ in range(length):
        if rng.random() < p:
            ids.append(rng.choice(ctrl))
        else:
            ids.append(rng.randrange(0, vocab))
    return ids


@pytest.mark.parametrize("base_reset", [False, True])
def test_scan_matches_coded_memory(codebook, base_reset):
    rng = random.Random(0)
    na = 5
    ctrl = [300 + i for i in range(na + (1 if base_reset else 0))]
    table = expert_table(ctrl, na)
    for trial in range(40):
        ids = _stream(rng, rng.randrange(1, 120), ctrl)
        if trial % 5 == 0:
            ids[0] = rng.choice(ctrl)  # control token at position 0
        if trial % 7 == 0 and len(ids) > 3:
            ids[1] = ids[2] = rng.choice(ctrl)  # adjacent control tokens
        got, _ = route_sequence(ids, table)
        want = coded_switch_route(torch.tensor(ids), ctrl, na, codebook)
        assert torch.equal(got, want), (ids, got.tolist(), want.tolist())


def test_chunked_carry_equals_whole():
    rng = random.Random(1)
    na = 4
    ctrl = [500, 501, 502, 503]
    table = expert_table(ctrl, na)
    for _ in range(30):
        ids = _stream(rng, 200, ctrl, p=0.05)
        whole, _ = route_sequence(ids, table)
        cuts = sorted(rng.sample(range(1, 200), 5))
        carry = 0
        parts = []
        prev = 0
        for c in cuts + [200]:
            part, carry = route_sequence(ids[prev:c], table, carry)
            parts.append(part)
            prev = c
        assert torch.equal(torch.cat(parts), whole)


def test_route_flat_multiple_requests():
    table = expert_table([10, 11], 2)
    ids = torch.tensor([1, 10, 2, 3, 11, 4, 5, 6])
    out, carries = route_flat(ids, [0, 3, 6, 8], [0, 2, 1], table)
    assert out.tolist() == [0, 1, 1, 2, 2, 2, 1, 1]
    assert carries == [1, 2, 1]


def test_latest_wins_semantics_examples():
    # T A T B T -> 0 1 1 2 2 (reference docs example)
    table = expert_table([100, 101], 2)
    got, _ = route_sequence([5, 100, 6, 101, 7], table)
    assert got.tolist() == [0, 1, 1, 2, 2]
    # base-reset layout: slot 0 resets to base
    table = expert_table([99, 100, 101], 2)
    got, _ = route_sequence([5, 100, 6, 99, 7, 101], table)
    assert got.tolist() == [0, 1, 1, 0, 0, 2]


def test_codebook_properties(codebook):
    assert codebook.shape == (2048, 64)
    assert torch.allclose(codebook.norm(dim=1), torch.ones(2048))
    assert abs(verify_coherence(codebook) - 0.125) < 1e-9


def test_dg1_codebook_small():
    g = KerdockDGCodeGenerator(4, "dg1")
    cb = g.precompute_codebook()
    assert cb.shape == (g.capacity, 16)
    assert torch.unique(cb, dim=0).shape[0] == g.capacity
    assert verify_coherence(cb) <= 0.5 + 1e-9


class _Cfg:
    vocab_size = 50
    adapter_token_ids = [50, 51]
    adapter_substitute_token_ids = [7, 8]
    adapter_kinds = ["lora", "probe"]


def test_token_exchange_and_probe_split():
    lut = build_control_to_substitute_lut(_Cfg)
    assert lut.numel() == 52 and lut[50] == 7 and lut[51] == 8 and lut[3] == -1
    ids = torch.tensor([[1, 50, 2, 51, 60]])
    assert apply_token_exchange(lut, ids).tolist() == [[1, 7, 2, 8, 60]]
    kind = probe_slot_mask(_Cfg.adapter_kinds)
    assert kind.tolist() == [False, False, True]
    assert probe_slot_mask(["lora", "lora"]) is None
    lora, probe = split_probe_stream(torch.tensor([0, 1, 2, 1]), kind)
    assert lora.tolist() == [0, 1, 0, 1] and probe.tolist() == [0, 0, 2, 0]


def test_codebook_size_limit():
    """DG(6, 1) (65,536 x 64, coherence 1/4) is written; DG(8, 1) (4.2M x 256, 4 GB) is refused."""
    import pytest
    import torch

    from granite_switch_b200.routing.codebook import KerdockDGCodeGenerator

    cb = KerdockDGCodeGenerator(m=6, code_type="dg1").precompute_codebook(torch.float32)
    assert tuple(cb.shape) == (65536, 64)
    with pytest.raises(ValueError, match="MB"):
        KerdockDGCodeGenerator(m=8, code_type="dg1").precompute_codebook(torch.float32)
