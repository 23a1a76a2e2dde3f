"""Composed-checkpoint IO in the HF safetensors layout.

One ``model.safetensors`` or ``model-0000i-of-0000n.safetensors`` shards with a
``model.safetensors.index.json`` weight map (the layout ``save_pretrained``
writes; the reference composes with ``max_shard_size="5GB"``, reference:
src/granite_switch/composer/compose_granite_switch.py:1691-1693). Loading is
lazy (``safe_open``) so the serving runtime can stream one tensor at a time
into its kernel layouts without holding the whole checkpoint in host memory.
"""
from __future__ import annotations

import json
import os
from collections.abc import Iterator

import torch
from safetensors import safe_open
from safetensors.torch import save_file

INDEX_NAME = "model.safetensors.index.json"
SINGLE_NAME = "model.safetensors"


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def save_state_dict(sd: dict[str, torch.Tensor], path: str, max_shard_bytes: int = 5 * 1024 ** 3,
                    metadata: dict[str, str] | None = None) -> list[str]:
    """Write ``sd`` as safetensors shards; returns the file names written."""
    os.makedirs(path, exist_ok=True)
    meta = {"format": "pt", **(metadata or {})}
    items = [(k, v.detach().contiguous().cpu()) for k, v in sd.items()]
    shards: list[list[tuple[str, torch.Tensor]]] = [[]]
    size = 0
    for k, v in items:
        n = _nbytes(v)
        if shards[-1] and size + n > max_shard_bytes:
            shards.append([])
            size = 0
        shards[-1].append((k, v))
        size += n
    # remove stale files of a previous save
    for f in os.listdir(path):
        if f.endswith(".safetensors") or f == INDEX_NAME:
            os.remove(os.path.join(path, f))
    if len(shards) == 1:
        save_file(dict(shards[0]), os.path.join(path, SINGLE_NAME), metadata=meta)
        return [SINGLE_NAME]
    names = []
    weight_map = {}
    total = 0
    for i, shard in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(dict(shard), os.path.join(path, name), metadata=meta)
        names.append(name)
        for k, v in shard:
            weight_map[k] = name
            total += _nbytes(v)
    with open(os.path.join(path, INDEX_NAME), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)
    return names


def checkpoint_files(path: str) -> list[str]:
    idx = os.path.join(path, INDEX_NAME)
    if os.path.exists(idx):
        with open(idx) as f:
            wm = json.load(f)["weight_map"]
        return sorted(set(wm.values()))
    if os.path.exists(os.path.join(path, SINGLE_NAME)):
        return [SINGLE_NAME]
    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors files under {path}")
    return files


def iter_tensors(path: str, device: str = "cpu") -> Iterator[tuple[str, torch.Tensor]]:
    """Yield ``(name, tensor)`` for every tensor of the checkpoint, one at a time."""
    for fname in checkpoint_files(path):
        with safe_open(os.path.join(path, fname), framework="pt", device=device) as f:
            for k in f.keys():
                yield k, f.get_tensor(k)


def tensor_names(path: str) -> list[str]:
    names = []
    for fname in checkpoint_files(path):
        with safe_open(os.path.join(path, fname), framework="pt") as f:
            names.extend(f.keys())
    return names


def load_state_dict(path: str, device: str = "cpu") -> dict[str, torch.Tensor]:
    return dict(iter_tensors(path, device))


class LazyCheckpoint:
    """Read-on-demand view of a composed checkpoint: ``ckpt[name]`` reads one tensor
    from its shard (memory-mapped by safetensors), so a rank materialises only the
    tensors it packs, one at a time, never the whole state dict. Every read is
    recorded; :meth:`unread` lists the tensors nothing asked for (the load audit).
    """

    def __init__(self, path: str):
        self.path = path
        self._where: dict[str, str] = {}
        for fname in checkpoint_files(path):
            with safe_open(os.path.join(path, fname), framework="pt") as f:
                for k in f.keys():
                    self._where[k] = fname
        self._open: dict[str, object] = {}
        self.read: set[str] = set()

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def keys(self):
        return self._where.keys()

    def __getitem__(self, name: str) -> torch.Tensor:
        fname = self._where.get(name)
        if fname is None:
            raise KeyError(f"tensor {name!r} is missing from the checkpoint at {self.path}")
        h = self._open.get(fname)
        if h is None:
            h = self._open[fname] = safe_open(os.path.join(self.path, fname), framework="pt")
        self.read.add(name)
        return h.get_tensor(name)

    def unread(self) -> list[str]:
        return sorted(k for k in self._where if k not in self.read)

    def close(self) -> None:
        self._open.clear()


def total_bytes(path: str) -> int:
    n = 0
    for fname in checkpoint_files(path):
        n += os.path.getsize(os.path.join(path, fname))
    return n
