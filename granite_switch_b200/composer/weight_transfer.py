"""Weight transfer into the composed layout: fuse base projections, stack adapters.

* Base: ``q|k|v`` are concatenated into ``self_attn.qkv_proj.base_layer.weight``
  and ``gate|up`` into ``shared_mlp.input_linear.base_layer.weight``; ``o`` and
  ``down`` map to ``o_proj`` / ``shared_mlp.output_linear``. A module that no
  adapter targets keeps a plain ``.weight`` (no ``base_layer``).
* Adapters: each PEFT ``lora_A [r, in]`` / ``lora_B [out, r]`` is zero-padded
  to ``max_lora_rank`` and stacked into ``[NA, 1, R, in]`` / ``[NA, 1, out, R]``;
  ``lora_B`` is pre-scaled by ``alpha / r`` so the runtime applies no scaling.
(reference: src/granite_switch/composer/weight_transfer.py:59-200, :401-534,
:567-613.)
"""
from __future__ import annotations

import re

import torch

# PEFT module name -> (composed module group, slice index, number of slices)
ATTN_SLICES = {"q_proj": ("qkv_proj", 0), "k_proj": ("qkv_proj", 1), "v_proj": ("qkv_proj", 2),
               "o_proj": ("o_proj", None)}
MLP_SLICES = {"gate_proj": ("shared_input_linear", 0), "up_proj": ("shared_input_linear", 1),
              "down_proj": ("shared_output_linear", None)}
GROUP_PREFIX = {
    "qkv_proj": "self_attn.qkv_proj",
    "o_proj": "self_attn.o_proj",
    "shared_input_linear": "shared_mlp.input_linear",
    "shared_output_linear": "shared_mlp.output_linear",
    "cross_stream": "cross_stream",
}
GROUP_SLICES = {"qkv_proj": 3, "o_proj": 1, "shared_input_linear": 2, "shared_output_linear": 1,
                "cross_stream": 1}

_PEFT_RE = re.compile(
    r"(?:base_model\.model\.)?model\.layers\.(\d+)\.(?:self_attn|mlp|shared_mlp)?\.?"
    r"(q_proj|k_proj|v_proj|o_proj|gate_proj|up_proj|down_proj|input_linear|output_linear|cross_stream)"
    r"\.lora_([AB])(?:\.default)?\.weight$"
)
# PEFT modules of a fused MoE-hybrid shared MLP: input_linear (gate|up) is split into
# two slices (A duplicated, B chunked on its output dim), output_linear is down.
FUSED_SPLIT = {"input_linear": ("shared_input_linear", 2), "output_linear": ("shared_output_linear", 1)}


def parse_peft_name(name: str):
    """``(layer, module, 'A'|'B')`` for a PEFT LoRA tensor name, else ``None``."""
    m = _PEFT_RE.search(name)
    if not m:
        return None
    return int(m.group(1)), m.group(2), m.group(3)


def module_group(module: str) -> tuple[str, int | None]:
    if module == "input_linear":
        return "shared_input_linear", -1  # both slices
    if module == "output_linear":
        return "shared_output_linear", None
    if module in ATTN_SLICES:
        return ATTN_SLICES[module]
    if module in MLP_SLICES:
        return MLP_SLICES[module]
    if module == "cross_stream":
        return "cross_stream", None
    raise KeyError(module)


def fuse_base_weights(base: dict[str, torch.Tensor], num_layers: int, lora_groups: list[str]) -> dict[str, torch.Tensor]:
    """Map a dense Granite base state dict to composed names (fused qkv / gate-up)."""
    out: dict[str, torch.Tensor] = {}
    for k in ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"):
        if k in base:
            out[k] = base[k]
    for i in range(num_layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = base[p + "input_layernorm.weight"]
        out[p + "post_attention_layernorm.weight"] = base[p + "post_attention_layernorm.weight"]
        if p + "self_attn.qkv_proj.weight" in base:
            qkv = base[p + "self_attn.qkv_proj.weight"]
        else:
            qkv = torch.cat([base[p + f"self_attn.{n}.weight"] for n in ("q_proj", "k_proj", "v_proj")], 0)
        suffix = ".base_layer.weight" if "qkv_proj" in lora_groups else ".weight"
        out[p + "self_attn.qkv_proj" + suffix] = qkv
        suffix = ".base_layer.weight" if "o_proj" in lora_groups else ".weight"
        out[p + "self_attn.o_proj" + suffix] = base[p + "self_attn.o_proj.weight"]
        if p + "mlp.gate_proj.weight" in base:
            gu = torch.cat([base[p + "mlp.gate_proj.weight"], base[p + "mlp.up_proj.weight"]], 0)
            down = base[p + "mlp.down_proj.weight"]
        elif p + "shared_mlp.input_linear.weight" in base:
            gu = base[p + "shared_mlp.input_linear.weight"]
            down = base[p + "shared_mlp.output_linear.weight"]
        else:
            gu = down = None
        if gu is not None:
            suffix = ".base_layer.weight" if "shared_input_linear" in lora_groups else ".weight"
            out[p + "shared_mlp.input_linear" + suffix] = gu
            suffix = ".base_layer.weight" if "shared_output_linear" in lora_groups else ".weight"
            out[p + "shared_mlp.output_linear" + suffix] = down
        for moe in ("block_sparse_moe.experts.gate_up_proj", "block_sparse_moe.experts.down_proj",
                    "block_sparse_moe.router.weight"):
            if p + moe in base:
                out[p + moe] = base[p + moe]
    return out


def stack_adapters(adapters: list[dict], num_layers: int, slice_sizes: dict[str, list[int]],
                   in_sizes: dict[str, int], max_rank: int, dtype=torch.float32,
                   cross_rank: int | None = None) -> dict[str, torch.Tensor]:
    """Stack PEFT adapters into the composed ``lora_A*/lora_B*`` tensors.

    ``adapters[a]`` = ``{"tensors": {peft name: tensor}, "r": int, "alpha": float,
    "rank_pattern": {...}, "alpha_pattern": {...}}``. ``slice_sizes[group]`` lists
    the output size of each slice; ``in_sizes[group]`` the input size.
    """
    na = len(adapters)
    out: dict[str, torch.Tensor] = {}
    groups = [g for g in slice_sizes]
    for i in range(num_layers):
        for g in groups:
            rank = cross_rank if g == "cross_stream" else max_rank
            pre = f"model.layers.{i}.{GROUP_PREFIX[g]}"
            ns = GROUP_SLICES[g]
            if ns == 1:
                out[pre + ".lora_A"] = torch.zeros(na, 1, rank, in_sizes[g], dtype=dtype)
                out[pre + ".lora_B"] = torch.zeros(na, 1, slice_sizes[g][0], rank, dtype=dtype)
            else:
                for s in range(ns):
                    out[pre + f".lora_A_slices.{s}"] = torch.zeros(na, 1, rank, in_sizes[g], dtype=dtype)
                    out[pre + f".lora_B_slices.{s}"] = torch.zeros(na, 1, slice_sizes[g][s], rank, dtype=dtype)
    for a, ad in enumerate(adapters):
        pairs: dict[tuple[int, str], dict[str, torch.Tensor]] = {}
        for name, t in ad["tensors"].items():
            parsed = parse_peft_name(name)
            if parsed is None:
                continue
            layer, mod, ab = parsed
            pairs.setdefault((layer, mod), {})[ab] = t
        for (layer, mod), ab in pairs.items():
            if "A" not in ab or "B" not in ab:
                raise ValueError(f"adapter {a}: layer {layer} {mod} has only lora_{list(ab)}")
            g, s = module_group(mod)
            if g not in slice_sizes:
                continue
            A, B = ab["A"].to(dtype), ab["B"].to(dtype)
            r = A.shape[0]
            key = f"model.layers.{layer}.{mod}"
            r_pat = (ad.get("rank_pattern") or {})
            a_pat = (ad.get("alpha_pattern") or {})
            alpha = ad.get("alpha", r)
            for pat, val in a_pat.items():
                if pat in key:
                    alpha = val
            r_cfg = ad.get("r", r)
            for pat, val in r_pat.items():
                if pat in key:
                    r_cfg = val
            scale = float(alpha) / float(r_cfg)
            pre = f"model.layers.{layer}.{GROUP_PREFIX[g]}"
            if s is None:
                out[pre + ".lora_A"][a, 0, :r] = A
                out[pre + ".lora_B"][a, 0, :, :r] = B * scale
            elif s == -1:  # fused gate|up: duplicate A, chunk B
                half = B.shape[0] // 2
                for si in range(2):
                    out[pre + f".lora_A_slices.{si}"][a, 0, :r] = A
                    out[pre + f".lora_B_slices.{si}"][a, 0, :, :r] = B[si * half:(si + 1) * half] * scale
            else:
                out[pre + f".lora_A_slices.{s}"][a, 0, :r] = A
                out[pre + f".lora_B_slices.{s}"][a, 0, :, :r] = B * scale
    return out
