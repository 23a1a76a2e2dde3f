"""Checkpoint IO: lazy per-tensor reads and the load audit (CPU)."""
import os

import pytest
import torch
from safetensors.torch import load_file, save_file

from granite_switch_b200.checkpoint import LazyCheckpoint, save_state_dict
from granite_switch_b200.composer.synthetic import compose_synthetic
from granite_switch_b200.config import GraniteSwitchConfig
from granite_switch_b200.models.native import audit_unread


@pytest.fixture(scope="module")
def ckpt_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("ckpt"))
    compose_synthetic(d, "tiny", num_adapters=2, rank=8, targets=("q", "k", "v", "o"), seed=0,
                      dtype=torch.float32, num_hidden_layers=2)
    return d


def test_lazy_reads_only_what_is_asked(ckpt_dir):
    ck = LazyCheckpoint(ckpt_dir)
    names = list(ck.keys())
    assert "model.embed_tokens.weight" in ck and "nope" not in ck
    t = ck["model.norm.weight"]
    full = {}
    for f in os.listdir(ckpt_dir):
        if f.endswith(".safetensors"):
            full.update(load_file(os.path.join(ckpt_dir, f)))
    assert torch.equal(t, full["model.norm.weight"])
    assert ck.read == {"model.norm.weight"} and len(ck.unread()) == len(names) - 1
    with pytest.raises(KeyError, match="missing"):
        ck["model.layers.9.mlp.weight"]


def test_sharded_checkpoint_reads(tmp_path):
    sd = {f"t{i}": torch.full((64, 64), float(i)) for i in range(6)}
    save_state_dict(sd, str(tmp_path), max_shard_bytes=40000)  # several shards + index
    ck = LazyCheckpoint(str(tmp_path))
    assert sorted(ck.keys()) == sorted(sd) and float(ck["t4"][0, 0]) == 4.0


def test_load_audit(ckpt_dir):
    cfg = GraniteSwitchConfig.from_pretrained(ckpt_dir)
    n = cfg.num_decoder_layers
    # unused by design: codebook, tied LM head, other pipeline stages' layers
    audit_unread(cfg, ["model.switch.codebook", "model.layers.1.self_attn.o_proj.lora_A"], 0, 1)
    with pytest.raises(ValueError, match="does not use"):
        audit_unread(cfg, ["model.layers.0.self_attn.q_proj.weight"], 0, n)
    with pytest.raises(ValueError, match="does not use"):
        audit_unread(cfg, ["some.extra.tensor"], 0, n)


def test_audit_catches_an_unknown_tensor_in_a_checkpoint(ckpt_dir, tmp_path):
    """A checkpoint with an extra (for example unfused) projection is refused at load time
    instead of being served without it: every tensor the packer reads is recorded, the rest
    is audited."""
    d = str(tmp_path / "extra")
    os.makedirs(d)
    for f in os.listdir(ckpt_dir):
        src = os.path.join(ckpt_dir, f)
        if f.endswith(".safetensors"):
            sd = load_file(src)
            sd["model.layers.0.self_attn.q_proj.weight"] = torch.zeros(4, 4)
            save_file(sd, os.path.join(d, f))
        elif os.path.isfile(src):
            with open(src, "rb") as a, open(os.path.join(d, f), "wb") as b:
                b.write(a.read())
    cfg = GraniteSwitchConfig.from_pretrained(d)
    ck = LazyCheckpoint(d)
    for k in ck.keys():  # what the packer reads for a dense LoRA checkpoint
        if "q_proj" not in k and k != "model.switch.codebook":
            ck[k]
    with pytest.raises(ValueError, match="q_proj"):
        audit_unread(cfg, ck.unread(), 0, cfg.num_decoder_layers)
