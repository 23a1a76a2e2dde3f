"""Load-time repack of a composed checkpoint into the native kernels' layouts.

The analogue of the reference's ``finalize_weights`` (reference:
src/granite_switch/vllm/core/lora.py:299-538): per projection it finds the
adapters that actually touch it (nonzero ``lora_A``/``lora_B``), gives them
kernel-local ids 1..n (the per-module remap table), pads ranks to a multiple
of 32 and builds

* ``w``    ``[N, K]``   bf16 base weight (gate/up rows interleaved per GEMM
  tile when the SwiGLU epilogue is used);
* ``a_all`` ``[pad64(S*n*Rp), K]`` stacked shrink weights, rows ordered
  (slice, local adapter, rank);
* ``lb``   ``[N, n*Rp]`` packed expand weights (``lora_B`` already carries
  alpha / r), rows permuted like ``w``.

Tensor-parallel sharding happens here too: column-parallel projections
(qkv, gate/up) split ``w`` and ``lora_B`` on the output dim and replicate
``lora_A``; row-parallel ones (o, down) split ``w`` and ``lora_A`` on the
input dim and replicate ``lora_B``, so each rank adds its partial delta
before the reduction (reference: src/granite_switch/vllm/core/lora.py:270-297,
:568-586).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

RANK_ALIGN = 32


@dataclass
class PackedLinear:
    w: torch.Tensor
    n: int
    k: int
    a_all: torch.Tensor | None = None
    lb: torch.Tensor | None = None
    rank: int = 0              # padded rank (multiple of 32)
    n_local: int = 0           # adapters present in this module
    num_slices: int = 1
    slice_bounds: list[int] = field(default_factory=list)
    remap: list[int] | None = None   # global adapter index -> local id (0 = none)
    map_id: int = -1                 # index into the model's remap table set
    swiglu_tile: int = 0             # > 0: gate/up interleaved per tile of this many rows
    bias: torch.Tensor | None = None

    @property
    def has_lora(self) -> bool:
        return self.n_local > 0


def _pad_to(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def interleave_gate_up(w: torch.Tensor, tile: int) -> torch.Tensor:
    """[2I, ...] (gate rows then up rows) -> per tile: tile/2 gate rows, tile/2 up rows."""
    i = w.shape[0] // 2
    half = tile // 2
    assert i % half == 0, f"I={i} not divisible by {half}"
    g = w[:i].reshape(i // half, half, *w.shape[1:])
    u = w[i:].reshape(i // half, half, *w.shape[1:])
    return torch.stack([g, u], dim=1).reshape(w.shape)


def pack_linear(base_w: torch.Tensor, lora_a: list[torch.Tensor] | None, lora_b: list[torch.Tensor] | None,
                slice_sizes: list[int], num_adapters: int, device, dtype=torch.bfloat16,
                swiglu_tile: int = 0, tp_rank: int = 0, tp_size: int = 1, parallel: str = "none",
                bias: torch.Tensor | None = None) -> PackedLinear:
    """Pack one projection. ``lora_a[s]``: ``[NA,1,R,K]``; ``lora_b[s]``: ``[NA,1,n_s,R]``.

    ``parallel``: ``"column"`` shards outputs (per slice), ``"row"`` shards inputs.
    """
    w = base_w
    sizes = list(slice_sizes)
    la = lora_a
    lbs = lora_b
    if tp_size > 1 and parallel == "column":
        parts, lb_parts, new_sizes, off = [], [], [], 0
        for s, n in enumerate(sizes):
            assert n % tp_size == 0, f"slice {n} not divisible by tp {tp_size}"
            m = n // tp_size
            parts.append(w[off + tp_rank * m: off + (tp_rank + 1) * m])
            if lbs is not None:
                lb_parts.append(lbs[s][:, :, tp_rank * m:(tp_rank + 1) * m])
            new_sizes.append(m)
            off += n
        w = torch.cat(parts, 0)
        sizes = new_sizes
        lbs = lb_parts if lbs is not None else None
        if bias is not None:
            bias = torch.cat([bias[o:o + n][tp_rank * (n // tp_size):(tp_rank + 1) * (n // tp_size)]
                              for o, n in zip([sum(slice_sizes[:i]) for i in range(len(slice_sizes))], slice_sizes)])
    elif tp_size > 1 and parallel == "row":
        k = w.shape[1]
        assert k % tp_size == 0
        m = k // tp_size
        w = w[:, tp_rank * m:(tp_rank + 1) * m]
        if la is not None:
            la = [a[..., tp_rank * m:(tp_rank + 1) * m] for a in la]
        if bias is not None and tp_rank != 0:
            bias = None  # added once, after the reduction
    n_total, k = w.shape
    bounds = [0]
    for n in sizes:
        bounds.append(bounds[-1] + n)

    present: list[int] = []
    if la is not None and lbs is not None:
        for a in range(num_adapters):
            nz = any(bool(la[s][a].abs().sum() > 0) for s in range(len(la))) and \
                any(bool(lbs[s][a].abs().sum() > 0) for s in range(len(lbs)))
            if nz:
                present.append(a)
    pl = PackedLinear(w=None, n=n_total, k=k, num_slices=len(sizes), slice_bounds=bounds,
                      swiglu_tile=swiglu_tile)
    if present:
        r_max = max(int(la[0].shape[2]), 1)
        # effective rank: last nonzero rank row over present adapters
        used = 1
        for a in present:
            for s in range(len(la)):
                nzr = (la[s][a, 0].abs().sum(dim=1) > 0).nonzero()
                if nzr.numel():
                    used = max(used, int(nzr.max()) + 1)
        rp = _pad_to(min(used, r_max), RANK_ALIGN)
        nl = len(present)
        ns = len(sizes)
        rows = ns * nl * rp
        a_all = torch.zeros(_pad_to(rows, 64), k, dtype=torch.float32)
        lb = torch.zeros(n_total, nl * rp, dtype=torch.float32)
        for li, a in enumerate(present):
            for s in range(ns):
                r_here = min(rp, la[s].shape[2])
                a_all[(s * nl + li) * rp:(s * nl + li) * rp + r_here] = la[s][a, 0, :r_here].float()
                lb[bounds[s]:bounds[s + 1], li * rp:li * rp + r_here] = lbs[s][a, 0, :, :r_here].float()
        remap = [0] * (num_adapters + 1)
        for li, a in enumerate(present):
            remap[a + 1] = li + 1
        pl.a_all = a_all.to(device=device, dtype=dtype).contiguous()
        if swiglu_tile:
            lb = interleave_gate_up(lb, swiglu_tile)
        pl.lb = lb.to(device=device, dtype=dtype).contiguous()
        pl.rank = rp
        pl.n_local = nl
        pl.remap = remap
    if swiglu_tile:
        w = interleave_gate_up(w, swiglu_tile)
    pl.w = w.to(device=device, dtype=dtype).contiguous()
    if bias is not None:
        pl.bias = bias.to(device=device, dtype=dtype)
    return pl


def choose_swiglu_tile(inter_local: int) -> int:
    for bn in (256, 128, 64):
        if inter_local % (bn // 2) == 0:
            return bn
    raise ValueError(f"intermediate size {inter_local} is not a multiple of 32")


@dataclass
class PackedMoE:
    """Frozen expert bank in kernel layout (never a LoRA target).

    ``router`` ``[pad64(E), H]`` bf16 (zero rows past E); ``gate_up``
    ``[E, 2 I_local, H]`` with gate/up rows interleaved per SwiGLU tile;
    ``down`` ``[E, H, I_local]``. Under tensor parallelism every rank holds
    ``I / tp`` of each expert (gate/up column-parallel, down row-parallel)
    and the router is replicated.
    """
    router: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    num_experts: int
    top_k: int
    inter: int
    swiglu_tile: int


def pack_moe(gate_up: torch.Tensor, down: torch.Tensor, router: torch.Tensor, top_k: int, device,
             tp_rank: int = 0, tp_size: int = 1, dtype=torch.bfloat16) -> PackedMoE:
    """``gate_up [E, 2I, H]`` (gate rows then up rows), ``down [E, H, I]``, ``router [E, H]``."""
    e, two_i, h = gate_up.shape
    i = two_i // 2
    assert i % tp_size == 0, f"expert intermediate size {i} not divisible by tp {tp_size}"
    il = i // tp_size
    lo, hi = tp_rank * il, (tp_rank + 1) * il
    gu = torch.cat([gate_up[:, lo:hi], gate_up[:, i + lo:i + hi]], dim=1)
    tile = choose_swiglu_tile(il)
    gu = torch.stack([interleave_gate_up(gu[k], tile) for k in range(e)])
    dn = down[:, :, lo:hi]
    r = torch.zeros(_pad_to(e, 64), h, dtype=router.dtype, device=router.device)
    r[:e] = router
    return PackedMoE(router=r.to(device=device, dtype=dtype).contiguous(),
                     gate_up=gu.to(device=device, dtype=dtype).contiguous(),
                     down=dn.to(device=device, dtype=dtype).contiguous(),
                     num_experts=e, top_k=int(top_k), inter=il, swiglu_tile=tile)
