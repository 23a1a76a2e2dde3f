"""PyTorch building blocks of the HF-style Granite Switch model (CPU oracle).

Parameter names match the composed checkpoint layout exactly (reference:
src/granite_switch/hf/core/lora.py:23-348 for ``SwitchedLoRALinear`` /
``MergedSwitchedLoRALinear``), so ``load_state_dict`` reads a composed
``model.safetensors`` directly. ``lora_B`` is stored pre-scaled by alpha / r.
"""
from __future__ import annotations

import math

import torch
from torch import nn
from torch.nn import functional as F


class RMSNorm(nn.Module):
    """Granite RMSNorm: fp32 statistics, weight applied in the input dtype."""

    def __init__(self, hidden: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = x.dtype
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * h.to(dt)


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float, dtype=torch.float32):
    """NeoX-style (rotate-half) cos/sin tables for integer positions ``[..., S]``."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64, device=positions.device) / head_dim))
    f = positions.double().unsqueeze(-1) * inv
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x ``[B, S, heads, d]``; cos/sin ``[B, S, d]``."""
    return x * cos.unsqueeze(2) + rotate_half(x) * sin.unsqueeze(2)


def _lora_delta(x: torch.Tensor, idx: torch.Tensor, A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """Per-token ``B_a A_a x`` for adapter ``a = idx`` (0 = none). x ``[T, K]``."""
    out = x.new_zeros(x.shape[0], B.shape[2])
    for a in idx.unique().tolist():
        if a <= 0:
            continue
        rows = (idx == a).nonzero(as_tuple=True)[0]
        xa = x[rows]
        out[rows] = (xa @ A[a - 1, 0].t()) @ B[a - 1, 0].t()
    return out


class SwitchedLoRALinear(nn.Module):
    """Base linear plus stacked per-adapter LoRA ``lora_A [NA,1,R,K]``, ``lora_B [NA,1,N,R]``."""

    def __init__(self, in_features: int, out_features: int, num_adapters: int, max_rank: int,
                 bias: bool = False):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.base_layer = nn.Linear(in_features, out_features, bias=bias)
        self.lora_A = nn.Parameter(torch.zeros(num_adapters, 1, max_rank, in_features))
        self.lora_B = nn.Parameter(torch.zeros(num_adapters, 1, out_features, max_rank))

    def forward(self, x: torch.Tensor, adapter_indices: torch.Tensor | None = None) -> torch.Tensor:
        out = self.base_layer(x)
        if adapter_indices is None or not bool((adapter_indices > 0).any()):
            return out
        shp = out.shape
        flat = out.reshape(-1, shp[-1]).clone()
        flat += _lora_delta(x.reshape(-1, x.shape[-1]), adapter_indices.reshape(-1), self.lora_A, self.lora_B).to(flat.dtype)
        return flat.view(shp)


class MergedSwitchedLoRALinear(nn.Module):
    """Fused projection (q|k|v or gate|up) with one LoRA pair per output slice."""

    def __init__(self, in_features: int, output_slices: tuple[int, ...], num_adapters: int,
                 max_rank: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.output_slices = tuple(output_slices)
        self.base_layer = nn.Linear(in_features, sum(output_slices), bias=bias)
        self.lora_A_slices = nn.ParameterList(
            [nn.Parameter(torch.zeros(num_adapters, 1, max_rank, in_features)) for _ in output_slices])
        self.lora_B_slices = nn.ParameterList(
            [nn.Parameter(torch.zeros(num_adapters, 1, n, max_rank)) for n in output_slices])

    def forward(self, x: torch.Tensor, adapter_indices: torch.Tensor | None = None) -> torch.Tensor:
        out = self.base_layer(x)
        if adapter_indices is None or not bool((adapter_indices > 0).any()):
            return out
        shp = out.shape
        flat = out.reshape(-1, shp[-1]).clone()
        xf = x.reshape(-1, x.shape[-1])
        idx = adapter_indices.reshape(-1)
        off = 0
        for s, n in enumerate(self.output_slices):
            flat[:, off:off + n] += _lora_delta(xf, idx, self.lora_A_slices[s], self.lora_B_slices[s]).to(flat.dtype)
            off += n
        return flat.view(shp)


def attention(q, k, v, scale: float, q_pos: torch.Tensor, k_pos: torch.Tensor,
              key_valid: torch.Tensor | None = None) -> torch.Tensor:
    """Causal GQA attention. q ``[B,S,Hq,d]``, k/v ``[B,L,Hkv,d]``; positions ``[B,S]``/``[B,L]``."""
    b, s, hq, d = q.shape
    hkv = k.shape[2]
    g = hq // hkv
    k = k.repeat_interleave(g, dim=2)
    v = v.repeat_interleave(g, dim=2)
    att = torch.einsum("bshd,blhd->bhsl", q.float(), k.float()) * scale
    mask = k_pos.unsqueeze(1) <= q_pos.unsqueeze(2)  # [B,S,L]
    if key_valid is not None:
        mask = mask & key_valid.unsqueeze(1)
    att = att.masked_fill(~mask.unsqueeze(1), float("-inf"))
    p = torch.softmax(att, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    o = torch.einsum("bhsl,blhd->bshd", p, v.float())
    return o.to(q.dtype)


def init_normal_(module: nn.Module, std: float, generator: torch.Generator | None = None):
    for p in module.parameters():
        with torch.no_grad():
            p.normal_(0.0, std, generator=generator)


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate) * up


__all__ = [
    "RMSNorm", "SwitchedLoRALinear", "MergedSwitchedLoRALinear", "attention", "apply_rope",
    "rope_cos_sin", "rotate_half", "silu_mul", "init_normal_", "math",
]
