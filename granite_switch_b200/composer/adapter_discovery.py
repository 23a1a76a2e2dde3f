"""Find adapters: library trees, single adapter directories and YAML manifests.

* Library layout: ``<root>/<adapter>/<target model>/<technology>/{adapter_config.json,
  adapter_model.safetensors, io.yaml}``; when an adapter has both ``alora`` and
  ``lora`` builds, ``alora`` is preferred (reference:
  src/granite_switch/composer/adapter_discovery.py:16-106).
* A single adapter directory (it holds ``adapter_config.json``).
* A YAML manifest: a list (or ``{"adapters": [...]}``) of entries with
  ``path``, optional ``name``, ``type`` (alora|lora), ``kind: probe`` with
  ``labels`` and ``layer`` (reference: adapter_discovery.py:109-175).
Filters: ``include`` / ``exclude`` fnmatch patterns on names, and a technology
filter (reference: adapter_discovery.py:223).
"""
from __future__ import annotations

import fnmatch
import os
from dataclasses import dataclass, field


@dataclass
class FoundAdapter:
    name: str
    path: str
    technology: str
    kind: str = "lora"
    labels: list[str] | None = None
    layer: int | None = None
    extra: dict = field(default_factory=dict)


def _is_adapter_dir(p: str) -> bool:
    return os.path.isfile(os.path.join(p, "adapter_config.json"))


def discover_library(root: str, target_model: str | None = None, technology: str | None = None) -> list[FoundAdapter]:
    out = []
    if _is_adapter_dir(root):
        tech = "alora" if "alora" in root.lower().split(os.sep)[-1] else None
        return [FoundAdapter(os.path.basename(root.rstrip("/")), root, technology or tech or "alora")]
    for name in sorted(os.listdir(root)):
        adir = os.path.join(root, name)
        if not os.path.isdir(adir):
            continue
        models = sorted(m for m in os.listdir(adir) if os.path.isdir(os.path.join(adir, m)))
        if target_model is not None:
            short = target_model.rstrip("/").split("/")[-1]
            models = [m for m in models if m == short or m == target_model]
        for m in models:
            mdir = os.path.join(adir, m)
            techs = [t for t in ("alora", "lora") if _is_adapter_dir(os.path.join(mdir, t))]
            if technology is not None:
                techs = [t for t in techs if t == technology]
            if not techs:
                continue
            t = techs[0]  # alora preferred
            out.append(FoundAdapter(name, os.path.join(mdir, t), t))
            break
    return out


def discover_from_yaml(path: str) -> list[FoundAdapter]:
    import yaml

    with open(path) as f:
        doc = yaml.safe_load(f)
    entries = doc.get("adapters", doc) if isinstance(doc, dict) else doc
    base = os.path.dirname(os.path.abspath(path))
    out = []
    for e in entries:
        p = e["path"]
        if not os.path.isabs(p):
            p = os.path.join(base, p)
        kind = e.get("kind", "lora")
        name = e.get("name") or os.path.basename(p.rstrip("/"))
        out.append(FoundAdapter(name, p, e.get("type", "alora" if kind != "probe" else "lora"), kind,
                                e.get("labels"), e.get("layer"), {k: v for k, v in e.items() if k not in
                                                                   ("path", "name", "type", "kind", "labels", "layer")}))
    return out


def filter_adapters(found: list[FoundAdapter], include=None, exclude=None, technology=None) -> list[FoundAdapter]:
    out = list(found)
    if include:
        out = [a for a in out if any(fnmatch.fnmatch(a.name, pat) for pat in include)]
    if exclude:
        out = [a for a in out if not any(fnmatch.fnmatch(a.name, pat) for pat in exclude)]
    if technology:
        out = [a for a in out if a.technology == technology]
    return out


def resolve(sources: list[str], target_model: str | None = None, technology: str | None = None,
            include=None, exclude=None) -> list[FoundAdapter]:
    """Resolve each ``--adapters`` source (library dir, adapter dir, YAML file, or a Hugging Face repo)."""
    found: list[FoundAdapter] = []
    for src in sources:
        if src.endswith((".yaml", ".yml")) and os.path.isfile(src):
            found += discover_from_yaml(src)
        elif os.path.isdir(src):
            found += discover_library(src, target_model, technology)
        else:
            local = _hf_snapshot(src, target_model, include, exclude, technology)
            if local is None:
                raise FileNotFoundError(
                    f"adapter source {src!r} is neither a local path nor a reachable or cached Hugging Face repo")
            found += discover_library(local, target_model, technology)
    return found


def hf_patterns(target_model: str | None, include=None, exclude=None, technology: str | None = None):
    """``(allow_patterns, ignore_patterns)`` for a selective download of an adapter library laid
    out ``<adapter>/<model>/<technology>/...`` (reference: adapter_discovery.py:488-571): only
    the target model's adapters, the requested technology and the included names."""
    if not target_model:
        allow = None
    else:
        techs = [technology] if technology in ("alora", "lora") else ["alora", "lora"]
        short = target_model.rstrip("/").split("/")[-1]  # library dirs use the model's short name
        allow = [f"{n}/{short}/{t}/*" for n in (include or ["*"]) for t in techs]
        allow += ["*.yaml", "*.yml", "README*"]
    ignore = [f"{e}/*" for e in (exclude or [])] or None
    return allow, ignore


def _hf_snapshot(repo: str, target_model=None, include=None, exclude=None, technology=None) -> str | None:
    """Download (selectively) or find in the local cache; None when neither works."""
    try:
        from huggingface_hub import snapshot_download
    except ImportError:
        return None
    allow, ignore = hf_patterns(target_model, include, exclude, technology)
    offline = os.environ.get("HF_HUB_OFFLINE", "0") not in ("0", "", "false")
    for local_only in ((True,) if offline else (False, True)):
        try:
            return snapshot_download(repo, allow_patterns=allow, ignore_patterns=ignore, local_files_only=local_only)
        except Exception:
            continue
    return None
