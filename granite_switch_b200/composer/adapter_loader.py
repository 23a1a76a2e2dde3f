"""Read PEFT adapter directories (LoRA / aLoRA / Shadow-Residual) into :class:`AdapterSpec`.

An adapter directory holds ``adapter_config.json`` (``r``, ``lora_alpha``,
``rank_pattern``, ``alpha_pattern``, ``target_modules`` and, for activated
LoRA, ``alora_invocation_tokens``), ``adapter_model.safetensors`` (or
``adapter_model.bin``) and optionally ``io.yaml`` (reference:
src/granite_switch/composer/adapter_loader.py:44-360). Shadow-Residual
adapters are recognised by ``cross_stream`` tensors.
"""
from __future__ import annotations

import json
import os

import torch

from .compose import AdapterSpec
from .weight_transfer import parse_peft_name


def read_adapter_config(path: str) -> dict:
    with open(os.path.join(path, "adapter_config.json")) as f:
        return json.load(f)


def read_adapter_tensors(path: str) -> dict[str, torch.Tensor]:
    st = os.path.join(path, "adapter_model.safetensors")
    if os.path.exists(st):
        from safetensors.torch import load_file

        return load_file(st)
    binf = os.path.join(path, "adapter_model.bin")
    if os.path.exists(binf):
        return torch.load(binf, map_location="cpu", weights_only=True)
    raise FileNotFoundError(f"no adapter_model.safetensors / .bin in {path}")


def read_io_yaml(path: str) -> dict | None:
    p = os.path.join(path, "io.yaml")
    if not os.path.exists(p):
        return None
    import yaml

    with open(p) as f:
        return yaml.safe_load(f)


def is_shadow_residual(tensors: dict[str, torch.Tensor]) -> bool:
    return any(".cross_stream." in k for k in tensors)


def detect_technology(cfg: dict, path: str = "") -> str:
    if cfg.get("alora_invocation_tokens"):
        return "alora"
    low = path.lower()
    if "/alora" in low or low.endswith("alora"):
        return "alora"
    return "lora"


def detect_present_modules(tensors: dict[str, torch.Tensor]) -> set[str]:
    mods = set()
    for n in tensors:
        p = parse_peft_name(n)
        if p:
            mods.add(p[1])
    return mods


def load_adapter(path: str, name: str | None = None, technology: str | None = None,
                 require_io_yaml: bool = False, kind: str = "lora") -> AdapterSpec:
    cfg = read_adapter_config(path)
    tensors = read_adapter_tensors(path)
    io = read_io_yaml(path)
    if io is None and require_io_yaml:
        raise FileNotFoundError(f"{path}: io.yaml is missing (pass --create-ioyaml to synthesise one)")
    tech = technology or detect_technology(cfg, path)
    inv = cfg.get("alora_invocation_tokens")
    nm = name or (io or {}).get("name") or os.path.basename(os.path.dirname(os.path.dirname(path.rstrip("/")))) \
        or os.path.basename(path.rstrip("/"))
    return AdapterSpec(
        name=nm, tensors=tensors, r=int(cfg.get("r", 8)), alpha=float(cfg.get("lora_alpha", cfg.get("r", 8))),
        technology=tech, invocation_tokens=list(inv) if inv else None, kind=kind,
        rank_pattern=dict(cfg.get("rank_pattern") or {}), alpha_pattern=dict(cfg.get("alpha_pattern") or {}),
        io_config=io, source=path, last_context_token=cfg.get("last_context_token"),
        last_context_token_id=cfg.get("last_context_token_id"))


def empty_adapter(name: str, rank: int, alpha: float | None = None) -> AdapterSpec:
    """A built-in adapter slot with no weights (a control token that routes to base weights)."""
    return AdapterSpec(name=name, tensors={}, r=rank, alpha=alpha if alpha is not None else float(rank),
                       technology="lora", io_config=None, source="built-in")
