"""Synthetic base models and PEFT adapters of a named shape (random init).

Used by the tests (the tiny CPU config), the benchmark (Granite-3B / 8B
shapes) and anyone who wants to try the runtime without downloading weights.
Base weights and adapters are drawn from seeded normals, written in the base
model's own (unfused) naming so the composer's fuse/stack path is exercised.
"""
from __future__ import annotations

import torch

from .compose import AdapterSpec, compose_checkpoint

PRESETS = {
    # CPU fp32 tiny model
    "tiny": dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                 num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=10000.0),
    # Granite-3B-shape
    "granite-3b": dict(vocab_size=49152, hidden_size=2048, intermediate_size=8192, num_hidden_layers=40,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=64, rope_theta=10000.0),
    # Granite-8B-shape
    "granite-8b": dict(vocab_size=49152, hidden_size=4096, intermediate_size=12800, num_hidden_layers=40,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=10000.0),
    # unit-test shapes
    "micro": dict(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=16, rope_theta=10000.0),
}

_MODS = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
         "o": "self_attn.o_proj", "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}


def base_config(preset: str | dict, **overrides) -> dict:
    cfg = dict(PRESETS[preset]) if isinstance(preset, str) else dict(preset)
    cfg.setdefault("rms_norm_eps", 1e-5)
    cfg.setdefault("tie_word_embeddings", True)
    cfg.setdefault("residual_multiplier", 1.0)
    cfg.setdefault("embedding_multiplier", 1.0)
    cfg.setdefault("logits_scaling", 1.0)
    cfg.setdefault("attention_multiplier", 1.0 / float(cfg["head_dim"]) ** 0.5)
    cfg.setdefault("max_position_embeddings", 131072)
    cfg.setdefault("bos_token_id", 0)
    cfg.setdefault("eos_token_id", 0)
    cfg.setdefault("pad_token_id", 0)
    cfg.update(overrides)
    return cfg


def _shapes(cfg: dict) -> dict[str, tuple[int, int]]:
    h, hd = cfg["hidden_size"], cfg["head_dim"]
    q, kv, i = cfg["num_attention_heads"] * hd, cfg["num_key_value_heads"] * hd, cfg["intermediate_size"]
    return {"q": (q, h), "k": (kv, h), "v": (kv, h), "o": (h, q), "gate": (i, h), "up": (i, h), "down": (h, i)}


def random_base_state(cfg: dict, seed: int = 0, std: float = 0.02, dtype=torch.float32,
                      device="cpu") -> dict[str, torch.Tensor]:
    """N(0, std) base weights in dense-Granite naming; norms are ones."""
    g = torch.Generator(device=device).manual_seed(seed)
    sd = {}

    def rnd(*shape):
        return (torch.randn(*shape, generator=g, device=device) * std).to(dtype)

    sd["model.embed_tokens.weight"] = rnd(cfg["vocab_size"], cfg["hidden_size"])
    if not cfg.get("tie_word_embeddings", True):
        sd["lm_head.weight"] = rnd(cfg["vocab_size"], cfg["hidden_size"])
    sd["model.norm.weight"] = torch.ones(cfg["hidden_size"], dtype=dtype)
    shp = _shapes(cfg)
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = torch.ones(cfg["hidden_size"], dtype=dtype)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(cfg["hidden_size"], dtype=dtype)
        for k, mod in _MODS.items():
            sd[p + mod + ".weight"] = rnd(*shp[k])
    return sd


def random_peft_adapter(cfg: dict, rank: int, targets=("q", "k", "v"), seed: int = 1, std_a: float = 0.02,
                        std_b: float = 0.01, dtype=torch.float32) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    shp = _shapes(cfg)
    out = {}
    for i in range(cfg["num_hidden_layers"]):
        for t in targets:
            n_out, n_in = shp[t]
            pre = f"base_model.model.model.layers.{i}.{_MODS[t]}"
            out[pre + ".lora_A.weight"] = (torch.randn(rank, n_in, generator=g) * std_a).to(dtype)
            out[pre + ".lora_B.weight"] = (torch.randn(n_out, rank, generator=g) * std_b).to(dtype)
    return out


def synthetic_adapters(cfg: dict, n: int, rank: int, targets=("q", "k", "v"), alpha: float | None = None,
                       invocation_len: int = 4, technology: str = "alora", seed: int = 1,
                       std_a: float = 0.02, std_b: float = 0.01) -> list[AdapterSpec]:
    g = torch.Generator().manual_seed(seed + 1000)
    out = []
    for a in range(n):
        inv = torch.randint(1, cfg["vocab_size"] - 1, (invocation_len,), generator=g).tolist()
        out.append(AdapterSpec(
            name=f"adapter_{a}", tensors=random_peft_adapter(cfg, rank, targets, seed + a, std_a, std_b),
            r=rank, alpha=alpha if alpha is not None else 2.0 * rank, technology=technology,
            invocation_tokens=inv))
    return out


def compose_synthetic(out_dir: str, preset: str | dict = "tiny", num_adapters: int = 3, rank: int = 8,
                      targets=("q", "k", "v"), seed: int = 0, dtype=torch.float32, invocation_len: int = 4,
                      base_reset: bool = False, technology: str = "alora", alpha: float | None = None,
                      **cfg_overrides):
    """Write a composed checkpoint with random base + random adapters; returns the config."""
    cfg = base_config(preset, **cfg_overrides)
    base = random_base_state(cfg, seed=seed)
    ads = synthetic_adapters(cfg, num_adapters, rank, targets, alpha=alpha, invocation_len=invocation_len,
                             technology=technology, seed=seed + 1)
    return compose_checkpoint(cfg, base, ads, out_dir, dtype=dtype, base_reset=base_reset,
                              base_model_name=f"synthetic-{preset if isinstance(preset, str) else 'custom'}")
