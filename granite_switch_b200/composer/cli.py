"""Composer command line: ``python -m granite_switch_b200.composer --adapters ... --base-model ... --output ...``.

Same flags as the reference composer (reference:
src/granite_switch/composer/compose_granite_switch.py:815-1073). Adapters come
from adapter libraries, single adapter directories, YAML manifests, or Hugging
Face repos already in the local cache (no network access is attempted).
Steps: resolve and filter adapters -> load PEFT weights -> add control tokens
to the tokenizer and wrap its chat template -> fuse/stack weights -> write the
checkpoint, tokenizer, ``adapter_index.json``, ``io_configs/``,
``compose_report.json`` and ``BUILD.md``.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import time

import torch

from ..checkpoint import load_state_dict
from ..config import DEFAULT_ASR_MODEL_ID, DEFAULT_ASR_MODEL_REVISION
from .adapter_discovery import filter_adapters, resolve
from .adapter_loader import empty_adapter, load_adapter
from .compose import AdapterSpec, compose_checkpoint

# base-config fields copied into the composed config (reference: composer/arch.py:282-330)
_BASE_FIELDS = ["vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
                "num_key_value_heads", "hidden_act", "max_position_embeddings", "initializer_range",
                "rms_norm_eps", "use_cache", "pad_token_id", "bos_token_id", "eos_token_id",
                "tie_word_embeddings", "rope_theta", "rope_scaling", "attention_bias", "attention_dropout",
                "torch_dtype", "residual_multiplier", "embedding_multiplier", "logits_scaling",
                "attention_multiplier", "num_local_experts", "num_experts_per_tok", "shared_intermediate_size",
                "head_dim"]


def build_argparser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Compose a Granite Switch model with embedded LoRA / aLoRA adapters")
    p.add_argument("--adapters", nargs="*", default=[], help="adapter libraries, adapter dirs, YAML manifests")
    p.add_argument("--technology", choices=["alora", "lora"], default=None)
    p.add_argument("--base-model", default="ibm-granite/granite-4.1-3b")
    p.add_argument("--target-model", default=None)
    p.add_argument("--output", default="./granite-with-all-aloras")
    p.add_argument("--switch-head-dim", type=int, default=None)
    p.add_argument("--ms-code-m", type=int, choices=[6, 8], default=None)
    p.add_argument("--ms-memory-gain", type=float, default=None)
    p.add_argument("--base-reset-token", action="store_true")
    p.add_argument("--built-in-adapters", nargs="*", default=[])
    p.add_argument("--lora-rank", type=int, default=8)
    p.add_argument("--lora-alpha", type=float, default=None)
    p.add_argument("--include-adapters", nargs="*", default=None)
    p.add_argument("--exclude-adapters", nargs="*", default=None)
    p.add_argument("--technology-filter", choices=["alora", "lora"], default=None)
    p.add_argument("--list-adapters", action="store_true")
    p.add_argument("--debug-fields", action="store_true")
    p.add_argument("--create-ioyaml", action="store_true")
    p.add_argument("--dtype", default=None, choices=["bfloat16", "float16", "float32"],
                   help="weight dtype of the composed checkpoint (default: the base config's dtype, else float32, "
                        "as the reference's composer)")
    p.add_argument("--enable-audio", action="store_true")
    p.add_argument("--asr-model", default=None)
    p.add_argument("--asr-revision", default=None)
    p.add_argument("--bundle-asr", action="store_true")
    p.add_argument("--asr-device", default="cuda")
    p.add_argument("--asr-dtype", default=None, choices=[None, "auto", "float16", "bfloat16", "float32"])
    p.add_argument("--asr-pipeline-kwargs", default=None, help="JSON object")
    p.add_argument("--asr-generate-kwargs", default=None, help="JSON object")
    p.add_argument("--asr-max-audio-clips", type=int, default=32)
    p.add_argument("--asr-self-chunks", dest="asr_self_chunks", action="store_true", default=False)
    p.add_argument("--asr-no-self-chunks", dest="asr_self_chunks", action="store_false")
    p.add_argument("--asr-chunk-length-s", type=float, default=120.0)
    p.add_argument("--asr-chunk-overlap-s", type=float, default=5.0)
    return p


def _resolve_local(path: str) -> str:
    if os.path.isdir(path):
        return path
    try:
        from huggingface_hub import snapshot_download

        return snapshot_download(path, local_files_only=True)
    except Exception as e:
        raise FileNotFoundError(f"base model {path!r} is not a local directory nor in the local HF cache") from e


def load_base(path: str) -> tuple[dict, dict[str, torch.Tensor]]:
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    cfg = {k: raw[k] for k in _BASE_FIELDS if k in raw}
    if raw.get("model_type") == "granitemoehybrid":
        lt = raw.get("layer_types")
        if lt and any(t != "attention" and t != "full_attention" for t in lt):
            raise ValueError("the switch model is attention-only; this base has mamba layers")
    return cfg, load_state_dict(path)


def _probe_adapter(found, tokenizer) -> AdapterSpec:
    from safetensors.torch import load_file

    ph = os.path.join(found.path, "probe_head.safetensors")
    sd = load_file(ph) if os.path.exists(ph) else {}
    labels = found.labels or []
    if tokenizer is not None:
        from .tokenizer_setup import resolve_label_token_ids

        label_ids = resolve_label_token_ids(tokenizer, [str(x) for x in labels])
    else:
        label_ids = [int(lab) for lab in labels]
    return AdapterSpec(name=found.name, tensors={}, r=1, alpha=1.0, technology="lora", kind="probe",
                       probe_label_token_ids=label_ids, probe_read_layer=found.layer,
                       probe_weight=sd.get("weight"), probe_bias=sd.get("bias"), source=found.path)


_TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "vocab.json", "tokenizer.model")


def compose_main(argv=None) -> int:
    args = build_argparser().parse_args(argv)
    base_path = _resolve_local(args.base_model) if not args.list_adapters else args.base_model
    target = args.target_model or args.base_model
    found = resolve(args.adapters, target, args.technology_filter, args.include_adapters,
                    args.exclude_adapters) if args.adapters else []
    found = filter_adapters(found, args.include_adapters, args.exclude_adapters, args.technology_filter)
    if args.list_adapters:
        for a in found:
            print(f"{a.name:40s} {a.technology:6s} {a.kind:6s} {a.path}")
        return 0
    t0 = time.time()
    tokenizer = None
    # a directory without tokenizer files would give an empty placeholder tokenizer
    if any(os.path.exists(os.path.join(base_path, f)) for f in _TOKENIZER_FILES):
        try:
            from transformers import AutoTokenizer

            tokenizer = AutoTokenizer.from_pretrained(base_path)
        except Exception:
            tokenizer = None
    adapters: list[AdapterSpec] = []
    for f in found:
        if f.kind == "probe":
            adapters.append(_probe_adapter(f, tokenizer))
            continue
        a = load_adapter(f.path, name=f.name, technology=args.technology or f.technology,
                         require_io_yaml=not args.create_ioyaml)
        if a.io_config is None:
            a.io_config = {"name": a.name, "model": None, "response_format": None, "transformations": None,
                           "instruction": None, "parameters": None, "sentence_boundaries": None}
        adapters.append(a)
    for name in args.built_in_adapters:
        adapters.append(empty_adapter(name, args.lora_rank, args.lora_alpha))
    if not adapters:
        print("no adapters selected", file=sys.stderr)
        return 2
    # LoRA slots first, probes last (reference: compose_granite_switch.py:1265-1267)
    adapters.sort(key=lambda a: 1 if a.kind == "probe" else 0)
    base_cfg, base_sd = load_base(base_path)
    ctrl_ids = None
    reserved_row = default_sub = None
    extra_ids: list[int] = []
    if tokenizer is not None:
        from .tokenizer_setup import configure_tokenizer, find_reserved_never_emitted_token_id

        ctrl_ids, setup = configure_tokenizer(tokenizer, adapters, args.base_reset_token, audio=args.enable_audio)
        reserved_row = find_reserved_never_emitted_token_id(tokenizer)
        if args.enable_audio:
            extra_ids = [int(tokenizer.convert_tokens_to_ids("<|audio|>"))]
        if setup is not None:
            default_sub = setup.lora_substitute
            print(f"chat template: {setup.format.name}; placements: "
                  + ", ".join(f"{n}={p.mode}" for n, p in setup.placements.items()))
    extra = {}
    if args.enable_audio:
        extra.update(asr_enabled=True, asr_model_id=args.asr_model or DEFAULT_ASR_MODEL_ID,
                     asr_model_revision=args.asr_revision or (None if args.asr_model else DEFAULT_ASR_MODEL_REVISION),
                     asr_device=args.asr_device, asr_dtype=args.asr_dtype,
                     asr_pipeline_kwargs=json.loads(args.asr_pipeline_kwargs) if args.asr_pipeline_kwargs else None,
                     asr_generate_kwargs=json.loads(args.asr_generate_kwargs) if args.asr_generate_kwargs else None,
                     asr_max_audio_clips=args.asr_max_audio_clips, asr_chunk_length_s=args.asr_chunk_length_s,
                     asr_chunk_overlap_s=args.asr_chunk_overlap_s, asr_self_chunks=args.asr_self_chunks)
        if args.bundle_asr:
            extra["asr_bundled_path"] = "asr"
    dtype_name = args.dtype or str(base_cfg.get("torch_dtype") or base_cfg.get("dtype") or "float32")
    dtype = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[
        dtype_name.replace("torch.", "")]
    config = compose_checkpoint(base_cfg, base_sd, adapters, args.output, dtype=dtype,
                                base_reset=args.base_reset_token, base_model_name=args.base_model,
                                ms_code_m=args.ms_code_m or 6, ms_memory_gain=args.ms_memory_gain or 28.0,
                                switch_head_dim=args.switch_head_dim or 32, extra_config=extra,
                                control_token_ids=ctrl_ids, reserved_output_row=reserved_row,
                                default_substitute=default_sub, extra_token_ids=extra_ids,
                                vocab_size=len(tokenizer) if tokenizer is not None else None)
    if tokenizer is not None:
        tokenizer.save_pretrained(args.output)
    io_dir = os.path.join(args.output, "io_configs")
    for a in adapters:
        if a.io_config is not None:
            import yaml

            os.makedirs(io_dir, exist_ok=True)
            with open(os.path.join(io_dir, f"{a.name}.yaml"), "w") as f:
                yaml.safe_dump(a.io_config, f, sort_keys=False)
    if args.debug_fields:
        p = os.path.join(args.output, "adapter_index.json")
        idx = json.load(open(p))
        for e, a in zip(idx["adapters"], adapters):
            e["original_path"] = a.source
        json.dump(idx, open(p, "w"), indent=2)
    from .reporting import write_reports

    write_reports(args.output, config, adapters, base_model=args.base_model, seconds=time.time() - t0)
    if args.bundle_asr and args.enable_audio and args.asr_model and os.path.isdir(args.asr_model):
        shutil.copytree(args.asr_model, os.path.join(args.output, "asr"), dirs_exist_ok=True)
    print(f"composed {len(adapters)} adapters into {args.output}")
    return 0


def main():
    sys.exit(compose_main())


if __name__ == "__main__":
    main()
