"""Compose a base Granite checkpoint and N adapters into one Granite Switch checkpoint.

Core of the composer (reference: src/granite_switch/composer/compose_utils.py:30-369
and compose_granite_switch.py:1075-1769), independent of where the adapters
come from (PEFT directories, an adapter library, or the synthetic generator):

1. one control token per adapter is appended to the vocabulary (plus a leading
   ``<|base_reset|>`` on request); each gets a substitute id (aLoRA: the first
   invocation token, which the control token replaces in the prompt);
2. the config is inflated by the two switch cache slots and records ids, ranks,
   names, kinds and target module groups;
3. base weights are fused (q|k|v, gate|up) and adapters stacked with
   ``lora_B`` pre-scaled by alpha / r;
4. the output row of every control token is copied from a reserved row so the
   model never emits one; the switch buffers are written; then config,
   safetensors, ``adapter_index.json`` and ``compose_report.json`` are saved.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch

from ..checkpoint import save_state_dict
from ..config import SWITCH_CACHE_LAYERS, GraniteSwitchConfig
from ..routing.codebook import KerdockDGCodeGenerator
from ..routing.scan import probe_slot_mask
from ..routing.token_exchange import build_control_to_substitute_lut, validate_control_lut
from .arch import resolve_arch
from .validators import audit_saved_checkpoint, validate_cross_stream_population, validate_parameters
from .weight_transfer import GROUP_PREFIX, fuse_base_weights, module_group, parse_peft_name, stack_adapters


@dataclass
class AdapterSpec:
    name: str
    tensors: dict[str, torch.Tensor]
    r: int
    alpha: float
    technology: str = "alora"            # "alora" | "lora"
    invocation_tokens: list[int] | None = None
    kind: str = "lora"                   # "lora" | "probe"
    rank_pattern: dict = field(default_factory=dict)
    alpha_pattern: dict = field(default_factory=dict)
    substitute_token_id: int | None = None
    probe_label_token_ids: list[int] | None = None
    probe_read_layer: int | None = None
    probe_weight: torch.Tensor | None = None   # [L, H]
    probe_bias: torch.Tensor | None = None     # [L]
    io_config: dict | None = None
    source: str | None = None
    last_context_token: str | None = None      # Shadow Residual activation anchor
    last_context_token_id: int | None = None

    def target_groups(self) -> set[str]:
        groups = set()
        for n in self.tensors:
            p = parse_peft_name(n)
            if p:
                groups.add(module_group(p[1])[0])
        return groups

    def max_rank(self) -> int:
        ranks = [self.r] + [int(v) for v in self.rank_pattern.values()]
        found = [t.shape[0] for n, t in self.tensors.items() if (p := parse_peft_name(n)) and p[2] == "A"]
        return max(ranks + found)


def control_token_names(adapters: list[AdapterSpec], base_reset: bool) -> list[str]:
    names = [f"<|{a.name}|>" for a in adapters]
    return (["<|base_reset|>"] + names) if base_reset else names


def compose_checkpoint(base_config: dict, base_state: dict[str, torch.Tensor], adapters: list[AdapterSpec],
                       out_dir: str, *, dtype: torch.dtype = torch.bfloat16, base_reset: bool = False,
                       reserved_output_row: int | None = None, default_substitute: int | None = None,
                       base_model_name: str = "synthetic", ms_code_m: int = 6, ms_memory_gain: float = 28.0,
                       switch_head_dim: int = 32, extra_config: dict | None = None,
                       max_shard_bytes: int = 5 * 1024 ** 3,
                       control_token_ids: list[int] | None = None,
                       extra_token_ids: list[int] | None = None,
                       vocab_size: int | None = None) -> GraniteSwitchConfig:
    """``extra_token_ids``: other added tokens that need an embedding row and a
    never-emitted output row (the audio marker), like the control tokens.
    ``vocab_size``: rows of the composed embedding (the tokenizer's length after
    the control tokens were added, as the reference's resize does; rows past it
    are dropped); by default the base rows, grown to cover the added ids."""
    na = len(adapters)
    cfg = dict(base_config)
    base_vocab = int(cfg["vocab_size"])
    h = int(cfg["hidden_size"])
    nh, nkv = int(cfg["num_attention_heads"]), int(cfg["num_key_value_heads"])
    hd = int(cfg.get("head_dim") or h // nh)
    inter = int(cfg.get("shared_intermediate_size") or cfg["intermediate_size"])
    n_layers = int(cfg["num_hidden_layers"])
    lora_adapters = [a for a in adapters if a.kind == "lora"]
    groups: set[str] = set()
    for a in lora_adapters:
        groups |= a.target_groups()
    dual = any("cross_stream" in a.target_groups() for a in lora_adapters)
    if dual and any("cross_stream" not in a.target_groups() for a in lora_adapters):
        raise ValueError("Shadow Residual and plain LoRA/aLoRA adapters cannot be composed together")
    arch = resolve_arch(base_config, dual_stream=dual)
    for a in lora_adapters:
        arch.check_adapter_modules(a.name, {p[1] for n in a.tensors if (p := parse_peft_name(n))})
        if dual and {p[1] for n in a.tensors if (p := parse_peft_name(n))} & {"k_proj", "v_proj"}:
            raise ValueError(f"Shadow Residual adapter {a.name!r} trains k/v: the adapter stream reuses the "
                             f"base stream's K/V, so k/v LoRA would never apply")
    groups.discard("cross_stream")
    order = ["qkv_proj", "o_proj", "shared_input_linear", "shared_output_linear"]
    target_modules = [g for g in order if g in groups]

    # ---- control tokens and substitutes
    n_ctrl = na + (1 if base_reset else 0)
    if control_token_ids is not None:
        if len(control_token_ids) != n_ctrl:
            raise ValueError(f"{len(control_token_ids)} control token ids for {n_ctrl} control tokens")
        ctrl_ids = [int(t) for t in control_token_ids]
    else:
        ctrl_ids = list(range(base_vocab, base_vocab + n_ctrl))
    subs = []
    if base_reset:
        subs.append(default_substitute if default_substitute is not None else 0)
    for a in adapters:
        if a.substitute_token_id is not None:
            subs.append(int(a.substitute_token_id))
        elif a.technology == "alora" and a.invocation_tokens:
            subs.append(int(a.invocation_tokens[0]))
        else:
            subs.append(default_substitute if default_substitute is not None else 0)
    extra_ids = [int(t) for t in (extra_token_ids or [])]
    new_vocab = max([base_vocab] + [t + 1 for t in ctrl_ids + extra_ids])
    if vocab_size is not None:
        if vocab_size < max([0] + [t + 1 for t in ctrl_ids + extra_ids]):
            raise ValueError(f"vocab_size {vocab_size} does not cover the added token ids")
        new_vocab = int(vocab_size)
    ranks = [a.max_rank() if a.kind == "lora" else 1 for a in adapters]
    max_rank = max(ranks) if ranks else 8
    kinds = [a.kind for a in adapters]
    probe_labels = [a.probe_label_token_ids if a.kind == "probe" else None for a in adapters]
    probe_layers = [a.probe_read_layer if a.kind == "probe" else None for a in adapters]
    cross_rank = None
    if dual:
        cross_rank = max(a.tensors[n].shape[0] for a in lora_adapters for n in a.tensors
                         if (p := parse_peft_name(n)) and p[1] == "cross_stream" and p[2] == "A")

    cfg.update(
        num_adapters=na,
        adapter_token_ids=ctrl_ids,
        adapter_substitute_token_ids=subs,
        adapter_names=[a.name for a in adapters],
        adapter_ranks=ranks,
        max_lora_rank=max_rank,
        lora_target_modules=target_modules,
        num_hidden_layers=n_layers + (SWITCH_CACHE_LAYERS if na > 0 else 0),
        vocab_size=new_vocab,
        ms_code_m=ms_code_m,
        ms_memory_gain=ms_memory_gain,
        switch_head_dim=switch_head_dim,
        adapter_kinds=kinds,
        probe_label_token_ids=probe_labels if any(k == "probe" for k in kinds) else None,
        probe_read_layers=probe_layers if any(l is not None for l in probe_layers) else None,
        dual_stream=dual,
        cross_stream_rank=cross_rank,
        torch_dtype=str(dtype).replace("torch.", ""),
    )
    cfg.pop("layer_types", None)
    cfg.update(extra_config or {})
    config = GraniteSwitchConfig(**cfg)

    # ---- weights
    sd = fuse_base_weights(base_state, n_layers, target_modules)
    sizes, in_sizes = arch.sizes(cfg)
    slice_sizes = {g: sizes[g] for g in target_modules + (["cross_stream"] if dual else [])}
    padded = [AdapterSpec(a.name, a.tensors, a.r, a.alpha, rank_pattern=a.rank_pattern,
                          alpha_pattern=a.alpha_pattern) if a.kind == "lora"
              else AdapterSpec(a.name, {}, 1, 1.0) for a in adapters]
    sd.update(stack_adapters([vars(p) for p in padded], n_layers, slice_sizes, in_sizes, max_rank,
                             torch.float32, cross_rank))
    if dual:
        for i in range(n_layers):
            sd[f"model.layers.{i}.cross_stream.base_layer.weight"] = torch.zeros(h, h)

    # grow embeddings to cover the control ids; every control-token output row is
    # a copy of a reserved (never emitted) row, so the model does not emit them
    reserved = reserved_output_row if reserved_output_row is not None else base_vocab - 1
    for key in ("model.embed_tokens.weight", "lm_head.weight"):
        if key not in sd:
            continue
        t = sd[key]
        if new_vocab > t.shape[0]:
            t = torch.cat([t, t[reserved:reserved + 1].expand(new_vocab - t.shape[0], -1).clone()], 0)
        else:
            t = t[:new_vocab].clone()
        if ctrl_ids or extra_ids:
            t[torch.tensor(ctrl_ids + extra_ids, dtype=torch.long)] = t[reserved].clone()
        sd[key] = t

    if any(k == "probe" for k in kinds):
        lmax = config.max_probe_labels
        pw = torch.zeros(na, lmax, h)
        pb = torch.zeros(na, lmax)
        for i, a in enumerate(adapters):
            if a.kind == "probe" and a.probe_weight is not None:
                pw[i, :a.probe_weight.shape[0]] = a.probe_weight
                if a.probe_bias is not None:
                    pb[i, :a.probe_bias.shape[0]] = a.probe_bias
        sd["model.probe_head.weight"] = pw
        sd["model.probe_head.bias"] = pb

    sd = {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in sd.items()}
    if na > 0:
        gen = KerdockDGCodeGenerator(m=ms_code_m, code_type=config.ms_code_type)
        sd["model.switch.codebook"] = gen.precompute_codebook(torch.float32)
        lut = build_control_to_substitute_lut(config)
        validate_control_lut(lut, config)
        sd["model.switch.control_to_substitute_lut"] = lut
        kind_lut = probe_slot_mask(getattr(config, "adapter_kinds", None))
        if kind_lut is not None:
            sd["model.switch.adapter_kind_lut"] = kind_lut
    if config.tie_word_embeddings:
        sd.pop("lm_head.weight", None)

    validation = validate_parameters(sd, config, arch, adapters, cfg)
    validation["cross_stream_layers"] = validate_cross_stream_population(sd, config, adapters)
    os.makedirs(out_dir, exist_ok=True)
    config.save_pretrained(out_dir)
    save_state_dict(sd, out_dir, max_shard_bytes=max_shard_bytes)
    validation["saved_tensors"] = audit_saved_checkpoint(out_dir, sd)
    validation["arch"] = arch.model_type
    config.compose_validation = validation
    write_adapter_index(out_dir, config, adapters, base_model_name)
    write_generation_config(out_dir, config)
    return config


def write_adapter_index(out_dir: str, config: GraniteSwitchConfig, adapters: list[AdapterSpec],
                        base_model_name: str) -> None:
    """``adapter_index.json`` (reference: compose_granite_switch.py:446-524)."""
    off = len(config.adapter_token_ids or []) - config.num_adapters
    entries = []
    for i, a in enumerate(adapters):
        tok_id = config.adapter_token_ids[i + off]
        e = {
            "adapter_index": i + 1,
            "adapter_name": a.name,
            "technology": a.technology if a.kind == "lora" else "probe",
            "control_token": {"token": f"<|{a.name}|>", "id": tok_id},
        }
        if a.io_config is not None:
            e["io_config"] = f"io_configs/{a.name}.yaml"
        if a.invocation_tokens:
            e["invocation_token_ids"] = list(a.invocation_tokens)
        entries.append(e)
    idx = {"model_info": {"num_adapters": config.num_adapters, "base_model": base_model_name},
           "adapters": entries}
    with open(os.path.join(out_dir, "adapter_index.json"), "w") as f:
        json.dump(idx, f, indent=2)


def write_generation_config(out_dir: str, config: GraniteSwitchConfig) -> None:
    gc = {"bos_token_id": config.bos_token_id, "eos_token_id": config.eos_token_id,
          "pad_token_id": config.pad_token_id}
    with open(os.path.join(out_dir, "generation_config.json"), "w") as f:
        json.dump(gc, f, indent=2)


__all__ = ["AdapterSpec", "compose_checkpoint", "control_token_names", "GROUP_PREFIX"]
