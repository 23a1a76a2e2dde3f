"""Checks on a composed checkpoint before and after it is written.

(reference: src/granite_switch/composer/validator.py:17-286 and the save audit
compose_granite_switch.py:775-812.)

* :func:`validate_parameters` - every expected tensor exists with its shape and
  is finite; base weights are not all zero; each adapter's LoRA slice is
  non-zero exactly where the adapter trains a module (and exactly zero where it
  does not); probe and switch buffers are present.
* :func:`validate_cross_stream_population` - every Shadow-Residual slot has a
  non-zero ``cross_stream`` delta in at least one layer.
* :func:`audit_saved_checkpoint` - the files on disk hold exactly the tensors
  that were meant to be saved (names, shapes, dtypes).
"""
from __future__ import annotations

import os

import torch

from ..routing.token_exchange import validate_control_lut
from .arch import ArchSpec
from .weight_transfer import parse_peft_name


def _lora_keys(prefix: str, slices: int) -> list[tuple[str, str]]:
    if slices == 1:
        return [(prefix + ".lora_A", prefix + ".lora_B")]
    return [(prefix + f".lora_A_slices.{s}", prefix + f".lora_B_slices.{s}") for s in range(slices)]


def validate_parameters(sd: dict[str, torch.Tensor], config, arch: ArchSpec, adapters, base_cfg: dict) -> dict:
    """Raise ``ValueError`` listing every problem; return a summary for the report."""
    problems: list[str] = []
    n_layers = config.num_decoder_layers
    na = config.num_adapters
    slice_sizes, in_sizes = arch.sizes(base_cfg)
    groups = list(config.lora_target_modules or [])
    if config.dual_stream:
        groups.append("cross_stream")
    h = config.hidden_size

    def need(name, shape=None):
        t = sd.get(name)
        if t is None:
            problems.append(f"missing {name}")
            return None
        if shape is not None and tuple(t.shape) != tuple(shape):
            problems.append(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
        if t.is_floating_point() and not torch.isfinite(t).all():
            problems.append(f"{name}: non-finite values")
        return t

    need("model.embed_tokens.weight", (config.vocab_size, h))
    need("model.norm.weight", (h,))
    if not config.tie_word_embeddings:
        need("lm_head.weight", (config.vocab_size, h))
    base_zero = []
    populated = {}
    for i in range(n_layers):
        p = f"model.layers.{i}."
        need(p + "input_layernorm.weight", (h,))
        need(p + "post_attention_layernorm.weight", (h,))
        for g in arch.groups:
            if g.name == "cross_stream":
                continue
            if g.name.startswith("shared_") and not arch.shared_mlp:
                continue
            lora = g.name in groups
            out_total = sum(slice_sizes[g.name])
            w = need(p + g.prefix + (".base_layer.weight" if lora else ".weight"), (out_total, in_sizes[g.name]))
            if w is not None and w.is_floating_point() and not bool(w.abs().amax() > 0):
                base_zero.append(p + g.prefix)
        for gname in groups:
            g = arch.group(gname)
            rank = config.cross_stream_rank if gname == "cross_stream" else config.max_lora_rank
            for s, (ka, kb) in enumerate(_lora_keys(p + g.prefix, g.slices)):
                a = need(ka, (na, 1, rank, in_sizes[gname]))
                b = need(kb, (na, 1, slice_sizes[gname][s if g.slices > 1 else 0], rank))
                if a is None or b is None:
                    continue
                nz = (a.flatten(1).abs().amax(1) > 0) & (b.flatten(1).abs().amax(1) > 0)
                for k in range(na):
                    populated.setdefault((k, gname, s), set())
                    if bool(nz[k]):
                        populated[(k, gname, s)].add(i)
    if base_zero:
        problems.append(f"base weights all zero (uninitialised?): {base_zero[:5]}")
    # each adapter: every (module slice, layer) it trains is populated, nothing else is
    summary = {}
    for k, ad in enumerate(adapters):
        trained: dict[tuple[str, int], set[int]] = {}
        for n in ad.tensors:
            pp = parse_peft_name(n)
            if pp is None:
                continue
            g, sl = arch.group_of(pp[1])
            for s in (range(g.slices) if sl == -1 else [sl or 0]):
                trained.setdefault((g.name, s), set()).add(pp[0])
        row = {}
        for gname in groups:
            layers = set()
            for s in range(arch.group(gname).slices):
                have = populated.get((k, gname, s), set())
                want = trained.get((gname, s), set())
                if ad.kind == "lora" and want - have:
                    problems.append(f"adapter {ad.name}: {gname}[{s}] is trained but all zero in layers "
                                    f"{sorted(want - have)[:5]}")
                if have - want:
                    problems.append(f"adapter {ad.name}: {gname}[{s}] populated in layers "
                                    f"{sorted(have - want)[:5]} it does not train")
                layers |= have
            row[gname] = len(layers)
        summary[ad.name] = row
    if config.probe_label_token_ids is not None:
        lmax = config.max_probe_labels
        need("model.probe_head.weight", (na, lmax, h))
        need("model.probe_head.bias", (na, lmax))
    if na > 0:
        lut = need("model.switch.control_to_substitute_lut")
        if lut is not None:
            try:
                validate_control_lut(lut, config)
            except ValueError as e:
                problems.append(str(e))
        need("model.switch.codebook")
    if problems:
        raise ValueError("composed checkpoint failed validation:\n  " + "\n  ".join(problems))
    return {"layers_populated": summary, "tensors": len(sd),
            "parameters": int(sum(t.numel() for t in sd.values()))}


def validate_cross_stream_population(sd: dict[str, torch.Tensor], config, adapters) -> dict[str, int]:
    """Layers with a non-zero ``cross_stream`` delta per Shadow-Residual slot; raises when a slot has none."""
    if not config.dual_stream:
        return {}
    out = {}
    empty = []
    for k, ad in enumerate(adapters):
        if ad.kind != "lora":
            continue
        n = 0
        for i in range(config.num_decoder_layers):
            a = sd.get(f"model.layers.{i}.cross_stream.lora_A")
            b = sd.get(f"model.layers.{i}.cross_stream.lora_B")
            if a is not None and b is not None and bool(a[k].abs().amax() > 0) and bool(b[k].abs().amax() > 0):
                n += 1
        out[ad.name] = n
        if n == 0:
            empty.append(ad.name)
    if empty:
        raise ValueError(f"Shadow Residual adapters with no cross_stream weights in any layer: {empty}")
    return out


def audit_saved_checkpoint(out_dir: str, sd: dict[str, torch.Tensor]) -> int:
    """Re-read the written safetensors; raise if a tensor is missing, extra or differs in shape/dtype."""
    from safetensors import safe_open

    from ..checkpoint import checkpoint_files

    files = checkpoint_files(out_dir)
    seen = {}
    for f in files:
        with safe_open(os.path.join(out_dir, f), framework="pt") as fh:
            for k in fh.keys():
                sl = fh.get_slice(k)
                seen[k] = (tuple(sl.get_shape()), sl.get_dtype())
    missing = sorted(set(sd) - set(seen))
    extra = sorted(set(seen) - set(sd))
    dt = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16", torch.int64: "I64",
          torch.int32: "I32", torch.bool: "BOOL", torch.int8: "I8", torch.uint8: "U8"}
    bad = [k for k, t in sd.items() if k in seen and (seen[k][0] != tuple(t.shape) or
                                                      seen[k][1] != dt.get(t.dtype, seen[k][1]))]
    if missing or extra or bad:
        raise ValueError(f"saved checkpoint differs from the composed state: missing {missing[:5]}, "
                         f"extra {extra[:5]}, shape/dtype {bad[:5]}")
    return len(seen)


__all__ = ["validate_parameters", "validate_cross_stream_population", "audit_saved_checkpoint"]
