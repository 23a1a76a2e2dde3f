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
    # benchmark config 1: CPU fp32 tiny model
    "tiny": dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                 num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=10000.0),
    # benchmark config 2: Granite-3B-shape
    "granite-3b": dict(vocab_size=49152, hidden_size=2048, intermediate_size=8192, num_hidden_layers=40,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=64, rope_theta=10000.0),
    # benchmark config 3: Granite-8B-shape
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


def _mlp_size(cfg: dict) -> int:
    """Width of the dense (shared) MLP: intermediate_size for dense bases; for
    mixture-of-experts bases shared_intermediate_size (0 = no shared MLP)."""
    if int(cfg.get("num_local_experts", 0) or 0):
        return int(cfg.get("shared_intermediate_size") or 0)
    return int(cfg["intermediate_size"])


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
    n_exp = int(cfg.get("num_local_experts", 0) or 0)
    h = cfg["hidden_size"]
    # mixture-of-experts bases: experts use intermediate_size, the optional shared
    # MLP (dense mlp.* names) uses shared_intermediate_size
    shared = _mlp_size(cfg)
    shp = _shapes(dict(cfg, intermediate_size=shared)) if shared else _shapes(cfg)
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = torch.ones(h, dtype=dtype)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(h, dtype=dtype)
        for k, mod in _MODS.items():
            if k in ("gate", "up", "down") and not shared:
                continue
            sd[p + mod + ".weight"] = rnd(*shp[k])
        if n_exp:
            ie = cfg["intermediate_size"]
            sd[p + "block_sparse_moe.experts.gate_up_proj"] = rnd(n_exp, 2 * ie, h)
            sd[p + "block_sparse_moe.experts.down_proj"] = rnd(n_exp, h, ie)
            sd[p + "block_sparse_moe.router.weight"] = rnd(n_exp, h) * 10.0
    return sd


def random_peft_adapter(cfg: dict, rank: int, targets=("q", "k", "v"), seed: int = 1, std_a: float = 0.02,
                        std_b: float = 0.01, dtype=torch.float32, cross_rank: int = 0) -> dict[str, torch.Tensor]:
    """PEFT-named random LoRA tensors; ``cross_rank > 0`` adds a Shadow-Residual ``cross_stream``."""
    g = torch.Generator().manual_seed(seed)
    shared = _mlp_size(cfg)
    shp = _shapes(dict(cfg, intermediate_size=shared or cfg["intermediate_size"]))
    if not shared:  # no dense MLP to adapt
        targets = [t for t in targets if t not in ("gate", "up", "down")]
    if cross_rank:  # the Shadow-Residual adapter stream reads the base stream's K/V
        targets = [t for t in targets if t not in ("k", "v")]
    out = {}
    for i in range(cfg["num_hidden_layers"]):
        for t in targets:
            n_out, n_in = shp[t]
            pre = f"base_model.model.model.layers.{i}.{_MODS[t]}"
            out[pre + ".lora_A.weight"] = (torch.randn(rank, n_in, generator=g) * std_a).to(dtype)
            out[pre + ".lora_B.weight"] = (torch.randn(n_out, rank, generator=g) * std_b).to(dtype)
        if cross_rank:
            h = cfg["hidden_size"]
            pre = f"base_model.model.model.layers.{i}.cross_stream"
            out[pre + ".lora_A.weight"] = (torch.randn(cross_rank, h, generator=g) * std_a).to(dtype)
            out[pre + ".lora_B.weight"] = (torch.randn(h, cross_rank, generator=g) * std_b).to(dtype)
    return out


def synthetic_probes(cfg: dict, n: int, num_labels: int = 3, read_layers=None, seed: int = 7) -> list[AdapterSpec]:
    """``n`` probe slots: random label token ids and a random linear head each.

    ``read_layers[i]`` is the decoder layer whose output the probe reads, or
    ``None`` for the final-norm hidden state.
    """
    g = torch.Generator().manual_seed(seed)
    h = cfg["hidden_size"]
    out = []
    for i in range(n):
        labels = torch.randperm(cfg["vocab_size"] - 2, generator=g)[:num_labels].add(1).tolist()
        layer = read_layers[i] if read_layers is not None else None
        out.append(AdapterSpec(
            name=f"probe_{i}", tensors={}, r=1, alpha=1.0, technology="lora", kind="probe",
            probe_label_token_ids=labels, probe_read_layer=layer,
            probe_weight=torch.randn(num_labels, h, generator=g) * 0.1, probe_bias=torch.randn(num_labels, generator=g)))
    return out


def synthetic_adapters(cfg: dict, n: int, rank: int, targets=("q", "k", "v"), alpha: float | None = None,
                       invocation_len: int = 4, technology: str = "alora", seed: int = 1,
                       std_a: float = 0.02, std_b: float = 0.01, cross_rank: int = 0) -> list[AdapterSpec]:
    g = torch.Generator().manual_seed(seed + 1000)
    out = []
    for a in range(n):
        inv = torch.randint(1, cfg["vocab_size"] - 1, (invocation_len,), generator=g).tolist()
        out.append(AdapterSpec(
            name=f"adapter_{a}",
            tensors=random_peft_adapter(cfg, rank, targets, seed + a, std_a, std_b, cross_rank=cross_rank),
            r=rank, alpha=alpha if alpha is not None else 2.0 * rank, technology=technology,
            invocation_tokens=inv))
    return out


def compose_synthetic(out_dir: str, preset: str | dict = "tiny", num_adapters: int = 3, rank: int = 8,
                      targets=("q", "k", "v"), seed: int = 0, dtype=torch.float32, invocation_len: int = 4,
                      base_reset: bool = False, technology: str = "alora", alpha: float | None = None,
                      num_probes: int = 0, probe_read_layers=None, probe_labels: int = 3, cross_rank: int = 0,
                      std_b: float = 0.01, **cfg_overrides):
    """Write a composed checkpoint with random base + random adapters; returns the config.

    ``num_probes`` appends probe slots after the LoRA slots; ``cross_rank > 0``
    makes every adapter a Shadow-Residual one (dual-stream checkpoint).
    """
    cfg = base_config(preset, **cfg_overrides)
    base = random_base_state(cfg, seed=seed)
    ads = synthetic_adapters(cfg, num_adapters, rank, targets, alpha=alpha, invocation_len=invocation_len,
                             technology=technology, seed=seed + 1, cross_rank=cross_rank, std_b=std_b)
    if num_probes:
        ads += synthetic_probes(cfg, num_probes, probe_labels, probe_read_layers, seed=seed + 7)
    return compose_checkpoint(cfg, base, ads, out_dir, dtype=dtype, base_reset=base_reset,
                              base_model_name=f"synthetic-{preset if isinstance(preset, str) else 'custom'}")


def write_random_checkpoint(out_dir: str, config, device="cuda", seed: int = 0, std: float = 0.02,
                            lora_groups=("qkv_proj", "o_proj"), rank: int = 32,
                            max_shard_bytes: int = 4 * 1024 ** 3) -> None:
    """Write a composed checkpoint of ``config`` with random weights, generated on ``device``.

    For large shapes (the Granite-8B benchmark model) where composing from a
    random base on the CPU would be slow: tensors are drawn in bf16 directly
    in the composed layout and written shard by shard.
    """
    import json
    import os

    from safetensors.torch import save_file

    from ..routing.codebook import KerdockDGCodeGenerator
    from ..routing.token_exchange import build_control_to_substitute_lut

    os.makedirs(out_dir, exist_ok=True)
    g = torch.Generator(device=device).manual_seed(seed)
    h, d = config.hidden_size, config.head_dim_eff
    q, kv = config.num_attention_heads * d, config.num_key_value_heads * d
    inter = config.shared_intermediate_size
    na, r = config.num_adapters, config.max_lora_rank

    def rnd(*shape, s=std):
        return (torch.randn(*shape, generator=g, device=device) * s).to(torch.bfloat16)

    shards, cur, size = [], {}, 0

    def put(name, t):
        nonlocal cur, size
        n = t.numel() * t.element_size()
        if cur and size + n > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[name] = t.cpu()
        size += n

    put("model.embed_tokens.weight", rnd(config.vocab_size, h))
    put("model.norm.weight", torch.ones(h, dtype=torch.bfloat16))
    if not config.tie_word_embeddings:
        put("lm_head.weight", rnd(config.vocab_size, h))
    groups = {"qkv_proj": ("self_attn.qkv_proj", [q, kv, kv], h), "o_proj": ("self_attn.o_proj", [h], q),
              "shared_input_linear": ("shared_mlp.input_linear", [inter, inter], h),
              "shared_output_linear": ("shared_mlp.output_linear", [h], inter)}
    for i in range(config.num_decoder_layers):
        p = f"model.layers.{i}."
        put(p + "input_layernorm.weight", torch.ones(h, dtype=torch.bfloat16))
        put(p + "post_attention_layernorm.weight", torch.ones(h, dtype=torch.bfloat16))
        for gname, (mod, sizes, k) in groups.items():
            lora = gname in config.lora_target_modules
            put(p + mod + (".base_layer.weight" if lora else ".weight"), rnd(sum(sizes), k))
            if not lora:
                continue
            if len(sizes) > 1:
                for s, n in enumerate(sizes):
                    put(f"{p}{mod}.lora_A_slices.{s}", rnd(na, 1, r, k, s=0.02))
                    put(f"{p}{mod}.lora_B_slices.{s}", rnd(na, 1, n, r, s=0.02))
            else:
                put(f"{p}{mod}.lora_A", rnd(na, 1, r, k, s=0.02))
                put(f"{p}{mod}.lora_B", rnd(na, 1, sizes[0], r, s=0.02))
    if na > 0:
        put("model.switch.codebook", KerdockDGCodeGenerator(config.ms_code_m, config.ms_code_type)
            .precompute_codebook(torch.float32))
        put("model.switch.control_to_substitute_lut", build_control_to_substitute_lut(config))
    if cur:
        shards.append(cur)
    weight_map = {}
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(out_dir, name), metadata={"format": "pt"})
        for k in sh:
            weight_map[k] = name
    with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    config.save_pretrained(out_dir)
