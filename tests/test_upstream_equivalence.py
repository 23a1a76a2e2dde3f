"""A switch checkpoint with no adapter active reproduces upstream transformers' Granite model.

Independent oracle for the Granite numerics (embedding / residual / attention
multipliers, logits scaling, RoPE, GQA, SwiGLU): the base weights are loaded into
``transformers.GraniteForCausalLM`` and into the composed switch model; for
prompts without a control token the logits must agree (reference:
tests/shared/vllm_equivalence.py upstream-equivalence checks).
"""

import pytest
import torch

from granite_switch_b200.composer.compose import compose_checkpoint
from granite_switch_b200.composer.synthetic import base_config, random_base_state, synthetic_adapters
from granite_switch_b200.models import GraniteSwitchForCausalLM

transformers = pytest.importorskip("transformers")


def _granite_multipliers():
    # non-trivial values, as real Granite checkpoints have
    return dict(embedding_multiplier=12.0, residual_multiplier=0.22, logits_scaling=8.0, attention_multiplier=0.015625)


@pytest.mark.parametrize("tied", [True, False])
def test_no_adapter_matches_transformers_granite(tmp_path, tied):
    cfg = base_config("tiny", tie_word_embeddings=tied, **_granite_multipliers())
    base = random_base_state(cfg, seed=4)
    if not tied and "lm_head.weight" not in base:
        base["lm_head.weight"] = torch.randn(cfg["vocab_size"], cfg["hidden_size"]) * 0.02
    hf_cfg = transformers.GraniteConfig(**{k: v for k, v in cfg.items() if k != "head_dim"}, hidden_act="silu",
                                        attention_bias=False, mlp_bias=False)
    hf_cfg.head_dim = cfg["head_dim"]
    up = transformers.GraniteForCausalLM(hf_cfg).eval()
    missing, unexpected = up.load_state_dict(base, strict=False)
    assert not unexpected and all("rotary" in k or (tied and k == "lm_head.weight") for k in missing), missing
    if tied:
        up.tie_weights()
    out = str(tmp_path / "sw")
    ads = synthetic_adapters(cfg, 2, 8, ("q", "k", "v", "o", "gate", "up", "down"), seed=5)
    compose_checkpoint(cfg, base, ads, out, dtype=torch.float32)
    sw = GraniteSwitchForCausalLM.from_pretrained(out).eval()
    ids = torch.randint(1, cfg["vocab_size"], (2, 37), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        a = up(ids).logits.float()
        b = sw(ids).logits.float()
    # the switch vocabulary appends the control tokens; the base vocabulary must agree
    torch.testing.assert_close(b[..., : cfg["vocab_size"]], a, rtol=1e-4, atol=1e-4)
