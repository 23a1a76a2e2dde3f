"""Per-request sampling: native kernel on CUDA, PyTorch statement for the CPU oracle."""
from __future__ import annotations

import torch

from .._native import native


def _params(params, reqs, device):
    temp = torch.tensor([p.temperature if not p.greedy else 0.0 for p in params], dtype=torch.float32)
    top_k = torch.tensor([p.top_k for p in params], dtype=torch.int32)
    top_p = torch.tensor([p.top_p for p in params], dtype=torch.float32)
    seeds = torch.tensor([(p.seed if p.seed is not None else hash(r.request_id) & 0x7FFFFFFF) for p, r in zip(params, reqs)],
                         dtype=torch.long)
    offs = torch.tensor([len(r.output_ids) for r in reqs], dtype=torch.long)
    return [t.to(device, non_blocking=True) for t in (temp, top_k, top_p, seeds, offs)]


def sample(logits: torch.Tensor, params, reqs, out: torch.Tensor | None = None) -> torch.Tensor:
    """Sample one token per row of ``logits`` ([B, V] fp32 CUDA) with the native kernel."""
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
    temp, top_k, top_p, seeds, offs = _params(params, reqs, logits.device)
    native().sample(logits.contiguous(), temp, top_k, top_p, seeds, offs, out)
    return out


def sample_reference(logits: torch.Tensor, params, reqs) -> torch.Tensor:
    """Same distribution as the kernel (different random stream): temperature, top-k, top-p."""
    outs = []
    for row, p, r in zip(logits.float(), params, reqs):
        if p.greedy:
            outs.append(int(row.argmax()))
            continue
        x = row / p.temperature
        if p.top_k and p.top_k < x.numel():
            kth = torch.topk(x, p.top_k).values[-1]
            x = torch.where(x >= kth, x, torch.full_like(x, float("-inf")))
        if p.top_p < 1.0:
            sx, si = torch.sort(x, descending=True)
            cp = torch.softmax(sx, 0).cumsum(0)
            keep = cp - torch.softmax(sx, 0) < p.top_p
            x = torch.full_like(x, float("-inf")).scatter(0, si[keep], sx[keep])
        g = torch.Generator().manual_seed((p.seed if p.seed is not None else 0) + len(r.output_ids))
        outs.append(int(torch.multinomial(torch.softmax(x, 0), 1, generator=g)))
    return torch.tensor(outs, dtype=torch.long)
