"""The decoder on the native sm_100a kernels: one engine step = one ``forward``.

Per step: routing + LoRA metadata (one launch) -> embedding with token
exchange -> per layer [RMSNorm -> qkv shrink + switched GEMM -> RoPE + paged
KV write -> paged attention -> o_proj switched GEMM with the residual add in
its epilogue -> RMSNorm -> gate/up switched GEMM with SwiGLU in its epilogue
-> down switched GEMM with residual add] -> final RMSNorm on the rows that
need logits -> LM head GEMM (fp32, / logits_scaling).

Tensor parallelism (``tp_size > 1``): heads and the FFN are sharded; the
row-parallel o/down projections write ``residual + partial`` on rank 0 and
``partial`` elsewhere, and one all-reduce per projection sums them (the
reference does the same reduction after its expand,
src/granite_switch/vllm/core/lora.py:568-586). When a symmetric-memory
communicator is attached, that reduction runs in the fused kernels of
:mod:`granite_switch_b200.parallel.fused` instead of NCCL.
"""
from __future__ import annotations

import contextlib
import math
import os
from dataclasses import dataclass

import torch

from .._native import err_buffer, native
from ..config import GraniteSwitchConfig
from ..ops import attention as A
from ..ops import elementwise as E
from ..ops import gemm as G
from ..routing.scan import expert_table
from .packing import PackedLinear, PackedMoE, choose_swiglu_tile, pack_linear, pack_moe


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv: PackedLinear
    o: PackedLinear
    gu: PackedLinear | None             # shared MLP (None for pure mixture-of-experts bases)
    down: PackedLinear | None
    cross: PackedLinear | None = None   # Shadow Residual cross-stream LoRA (no base weight)
    moe: PackedMoE | None = None        # frozen expert bank


@dataclass
class AttnPlan:
    work_seq: torch.Tensor
    work_row0: torch.Tensor
    rows: int
    nsplit: int


@dataclass
class StepBatch:
    """Device-side inputs of one engine step (flattened request chunks)."""

    num_tokens: int
    num_seqs: int
    ids: torch.Tensor          # [T] int64 original ids (control tokens included)
    positions: torch.Tensor    # [T] int64
    slots: torch.Tensor        # [T] int64 KV slot of each token
    seq_starts: torch.Tensor   # [S+1] int32
    carry_in: torch.Tensor     # [S] int32 routing carry at chunk start
    kv_lens: torch.Tensor      # [S] int32 cached + new tokens
    block_table: torch.Tensor  # [S, max_blocks] int32
    logit_rows: torch.Tensor   # [B] int64 rows whose logits are needed
    plans: list                # [AttnPlan]
    # probe markers: per read layer (None = final norm) the device tensors
    # (flat rows, slots, logit rows); plus (logit rows, slots) of all markers
    probe_groups: list | None = None
    probe_all: tuple | None = None


class NativeGraniteSwitch:
    """Kernel-layout weights + persistent activation buffers + the step forward."""

    def __init__(self, config: GraniteSwitchConfig, device: torch.device, max_tokens: int,
                 num_kv_blocks: int, tp_rank: int = 0, tp_size: int = 1, tp_group=None,
                 max_seqs: int = 512, pipeline=None):
        self.cfg = config
        self.device = device
        self.tp_rank, self.tp_size, self.tp_group = tp_rank, tp_size, tp_group
        self.hidden = config.hidden_size
        self.head_dim = config.head_dim_eff
        assert config.num_attention_heads % tp_size == 0
        self.num_q = config.num_attention_heads // tp_size
        self.num_kv = max(1, config.num_key_value_heads // tp_size)
        self.inter = config.shared_intermediate_size // tp_size
        self.has_shared_mlp = config.shared_intermediate_size > 0
        self.has_moe = int(getattr(config, "num_local_experts", 0) or 0) > 0
        self.vocab = config.vocab_size
        # pipeline parallelism: this stage owns decoder layers [layer_lo, layer_hi)
        self.pipeline = pipeline
        if pipeline is not None:
            self.layer_lo, self.layer_hi = split_layers(config.num_decoder_layers, pipeline.rank, pipeline.size)
        else:
            self.layer_lo, self.layer_hi = 0, config.num_decoder_layers
        self.first_stage = pipeline is None or pipeline.rank == 0
        self.last_stage = pipeline is None or pipeline.rank == pipeline.size - 1
        self.num_layers = self.layer_hi - self.layer_lo
        self.max_tokens = max_tokens
        self.max_seqs = max_seqs
        self.num_kv_blocks = num_kv_blocks
        self.layers: list[LayerWeights] = []
        self.remaps: torch.Tensor | None = None
        self.comm = None  # optional fused-collective communicator
        # KV cache storage: bf16, or e4m3 with a per-(token, KV head) scale (kv_fp8.cu)
        self.kv_fp8 = False
        self.prof = None  # optional per-op CUDA-event profiler (utils.step_profile.StepProfiler)
        # prefill attention on tcgen05 (head_dim 64 / 128); False selects the mma.sync kernel (A/B tests)
        self.use_tc_attention = True
        # a step with both decode rows and prefill chunks runs the prefill attention on a
        # second stream, beside the decode attention (set by the engine)
        self.overlap_attention = False
        self._side_stream = None
        # decode tile rows over an fp8 cache: 8 (keys on the MMA's row side) or 16 (row-major)
        self.fp8_decode_rows = 8
        self.err = err_buffer(device)
        na = config.num_adapters
        self.num_adapters = na
        tbl = expert_table(config.adapter_token_ids or [], na, 1)
        self.expert_tbl = tbl.to(device)
        self.lut = None
        self.kind_lut = None
        self.cos_sin = E.rope_cos_sin_table(min(config.max_position_embeddings, 1 << 17), self.head_dim,
                                            config.rope_theta, device)
        # Shadow Residual (dual stream): base stream + adapter stream over base-only K/V
        self.dual = bool(getattr(config, "dual_stream", False))
        # probe heads: weight [NA, L, H] bf16, bias [NA, L] fp32, label ids [NA, L] int32 (-1 pad)
        self.probe_w = self.probe_b = self.probe_labels = None

    # ------------------------------------------------------------------ weights
    def _finish_weights(self, embed: torch.Tensor, final_norm: torch.Tensor, lm_head: torch.Tensor | None):
        self.embed_w = embed
        self.final_norm = final_norm
        self.lm_head_w = lm_head if lm_head is not None else embed
        # LM head is vocab-parallel under TP
        if self.tp_size > 1:
            v = self.lm_head_w.shape[0]
            per = (v + self.tp_size - 1) // self.tp_size
            per = (per + 255) // 256 * 256
            lo = self.tp_rank * per
            shard = torch.zeros(per, self.hidden, dtype=self.lm_head_w.dtype, device=self.device)
            hi = min(v, lo + per)
            if hi > lo:
                shard[: hi - lo] = self.lm_head_w[lo:hi]
            self.lm_vocab_lo, self.lm_vocab_hi = lo, hi
            self.lm_head_w = shard
        else:
            v = self.lm_head_w.shape[0]
            pad = (v + 255) // 256 * 256
            if pad != v:
                w = torch.zeros(pad, self.hidden, dtype=self.lm_head_w.dtype, device=self.device)
                w[:v] = self.lm_head_w
                self.lm_head_w = w
            self.lm_vocab_lo, self.lm_vocab_hi = 0, v
        # remap tables (deduplicated) for the routing kernel
        maps: list[list[int]] = []
        for lw in self.layers:
            for pl in (lw.qkv, lw.o, lw.gu, lw.down, lw.cross):
                if pl is not None and pl.has_lora:
                    if pl.remap not in maps:
                        maps.append(pl.remap)
                    pl.map_id = maps.index(pl.remap)
        self.remaps = torch.tensor(maps, dtype=torch.int32, device=self.device) if maps else None
        self.n_maps = len(maps)
        self._alloc_buffers()

    def _set_probes(self, weight: torch.Tensor, bias: torch.Tensor) -> None:
        cfg = self.cfg
        na, lmax = weight.shape[0], weight.shape[1]
        labels = torch.full((na, lmax), -1, dtype=torch.int32)
        for i, ids in enumerate(cfg.probe_label_token_ids or []):
            if ids:
                labels[i, : len(ids)] = torch.tensor(ids, dtype=torch.int32)
        self.probe_w = weight.to(self.device, torch.bfloat16).contiguous()
        self.probe_b = bias.to(self.device, torch.float32).contiguous()
        self.probe_labels = labels.to(self.device)

    def _pack_cross(self, la: torch.Tensor, lb: torch.Tensor) -> PackedLinear:
        """Cross-stream LoRA (replicated under TP). Its base weight is all zeros and
        never multiplied; ``lb`` is padded to the shrink width so the expand is one
        plain GEMM ``S @ lb^T`` over every adapter column."""
        h = self.hidden
        pl = pack_linear(torch.zeros(h, h), [la], [lb], [h], self.num_adapters, self.device)
        pl.w = None
        if pl.has_lora:
            pad = torch.zeros(h, pl.a_all.shape[0], dtype=pl.lb.dtype, device=self.device)
            pad[:, : pl.lb.shape[1]] = pl.lb
            pl.lb = pad
        return pl

    @classmethod
    def from_state_dict(cls, config: GraniteSwitchConfig, sd, device, max_tokens: int, num_kv_blocks: int,
                        tp_rank: int = 0, tp_size: int = 1, tp_group=None, max_seqs: int = 512, pipeline=None):
        """Pack a composed checkpoint (``sd``: name -> tensor, or a lazy getter).

        With ``pipeline`` only this stage's decoder layers are read.
        """
        self = cls(config, device, max_tokens, num_kv_blocks, tp_rank, tp_size, tp_group, max_seqs, pipeline)
        get = sd.__getitem__ if hasattr(sd, "__getitem__") else sd
        if hasattr(sd, "__contains__"):
            def has(k):
                return k in sd
        else:  # a bare getter: probe by reading
            def has(k):
                try:
                    get(k)
                    return True
                except KeyError:
                    return False
        na = config.num_adapters
        h, d = config.hidden_size, config.head_dim_eff
        q, kv = config.num_attention_heads * d, config.num_key_value_heads * d
        inter = config.shared_intermediate_size
        tiles = choose_swiglu_tile(inter // tp_size) if inter > 0 else 0

        def lin(prefix, slices, parallel, swiglu=0):
            base = prefix + ".base_layer.weight"
            if has(base):
                w = get(base)
                ns = len(slices)
                if ns > 1:
                    la = [get(f"{prefix}.lora_A_slices.{s}") for s in range(ns)]
                    lb = [get(f"{prefix}.lora_B_slices.{s}") for s in range(ns)]
                else:
                    la, lb = [get(prefix + ".lora_A")], [get(prefix + ".lora_B")]
            else:
                w, la, lb = get(prefix + ".weight"), None, None
            return pack_linear(w, la, lb, slices, na, device, swiglu_tile=swiglu, tp_rank=tp_rank,
                               tp_size=tp_size, parallel=parallel)

        for i in range(self.layer_lo, self.layer_hi):
            p = f"model.layers.{i}."
            lw = LayerWeights(
                in_norm=get(p + "input_layernorm.weight").to(device, torch.bfloat16),
                post_norm=get(p + "post_attention_layernorm.weight").to(device, torch.bfloat16),
                qkv=lin(p + "self_attn.qkv_proj", [q, kv, kv], "column"),
                o=lin(p + "self_attn.o_proj", [h], "row"),
                gu=lin(p + "shared_mlp.input_linear", [inter, inter], "column", swiglu=tiles) if inter > 0 else None,
                down=lin(p + "shared_mlp.output_linear", [h], "row") if inter > 0 else None,
            )
            if self.has_moe:
                e = p + "block_sparse_moe."
                lw.moe = pack_moe(get(e + "experts.gate_up_proj"), get(e + "experts.down_proj"),
                                  get(e + "router.weight"), config.num_experts_per_tok, device, tp_rank, tp_size)
            self.layers.append(lw)
        if self.dual:
            for i, lw in zip(range(self.layer_lo, self.layer_hi), self.layers):
                p = f"model.layers.{i}.cross_stream."
                lw.cross = self._pack_cross(get(p + "lora_A"), get(p + "lora_B"))
        if has("model.probe_head.weight"):
            self._set_probes(get("model.probe_head.weight"), get("model.probe_head.bias"))
        embed = get("model.embed_tokens.weight").to(device, torch.bfloat16)
        lm = None
        if not config.tie_word_embeddings and has("lm_head.weight"):
            lm = get("lm_head.weight").to(device, torch.bfloat16)
        if has("model.switch.control_to_substitute_lut"):
            self.lut = get("model.switch.control_to_substitute_lut").to(device, torch.long)
        if has("model.switch.adapter_kind_lut"):
            self.kind_lut = get("model.switch.adapter_kind_lut").to(device, torch.bool)
        self._finish_weights(embed, get("model.norm.weight").to(device, torch.bfloat16), lm)
        if hasattr(sd, "unread"):
            audit_unread(config, sd.unread(), self.layer_lo, self.layer_hi)
        return self

    @classmethod
    def from_random(cls, config: GraniteSwitchConfig, device, max_tokens: int, num_kv_blocks: int,
                    lora_modules=("qkv",), rank: int = 32, seed: int = 0, std: float = 0.02,
                    tp_rank: int = 0, tp_size: int = 1, tp_group=None, max_seqs: int = 512, pipeline=None):
        """Random-init weights of the architecture, generated directly in kernel layout on the GPU.

        Every rank draws the full (unsharded) tensors of every layer from the same
        seed and keeps its shard (and, under pipeline parallelism, its stage's
        layers), so TP / PP runs are numerically the same model as one GPU.
        """
        self = cls(config, device, max_tokens, num_kv_blocks, tp_rank, tp_size, tp_group, max_seqs, pipeline)
        g = torch.Generator(device=device).manual_seed(seed)
        na = config.num_adapters
        h, d = config.hidden_size, config.head_dim_eff
        q, kv = config.num_attention_heads * d, config.num_key_value_heads * d
        inter = config.shared_intermediate_size
        tiles = choose_swiglu_tile(inter // tp_size) if inter > 0 else 0
        scale = 2.0  # alpha / r
        n_exp = int(getattr(config, "num_local_experts", 0) or 0)

        def rnd(*shape, s=std):
            return (torch.randn(*shape, generator=g, device=device) * s).to(torch.bfloat16)

        def lin(n_out_slices, k, parallel, lora, swiglu=0):
            n = sum(n_out_slices)
            w = rnd(n, k)
            la = lb = None
            if lora and na > 0:
                la = [rnd(na, 1, rank, k, s=0.02) for _ in n_out_slices]
                lb = [rnd(na, 1, ns, rank, s=0.01 * scale) for ns in n_out_slices]
            return pack_linear(w, la, lb, n_out_slices, na, device, swiglu_tile=swiglu, tp_rank=tp_rank,
                               tp_size=tp_size, parallel=parallel)

        for i in range(config.num_decoder_layers):
            lw = LayerWeights(
                in_norm=torch.ones(h, dtype=torch.bfloat16, device=device),
                post_norm=torch.ones(h, dtype=torch.bfloat16, device=device),
                qkv=lin([q, kv, kv], h, "column", "qkv" in lora_modules),
                o=lin([h], q, "row", "o" in lora_modules),
                gu=lin([inter, inter], h, "column", "gu" in lora_modules, swiglu=tiles) if inter > 0 else None,
                down=lin([h], inter, "row", "down" in lora_modules) if inter > 0 else None,
            )
            if n_exp:
                ie = config.intermediate_size
                lw.moe = pack_moe(rnd(n_exp, 2 * ie, h), rnd(n_exp, h, ie), rnd(n_exp, h),
                                  config.num_experts_per_tok, device, tp_rank, tp_size)
            if self.layer_lo <= i < self.layer_hi:
                self.layers.append(lw)
        if self.dual and na > 0:
            rc = int(config.cross_stream_rank or 32)
            for i in range(config.num_decoder_layers):
                cross = self._pack_cross(rnd(na, 1, rc, h).float().cpu(), rnd(na, 1, h, rc, s=0.01).float().cpu())
                if self.layer_lo <= i < self.layer_hi:
                    self.layers[i - self.layer_lo].cross = cross
        if config.probe_control_token_ids:
            lmax = max(1, config.max_probe_labels)
            self._set_probes(rnd(na, lmax, h, s=0.1), torch.randn(na, lmax, generator=g, device=device))
        embed = rnd(config.vocab_size, h)
        if config.adapter_token_ids:
            from ..routing.token_exchange import build_control_to_substitute_lut

            lut = build_control_to_substitute_lut(config)
            self.lut = lut.to(device) if lut is not None else None
        self._finish_weights(embed, torch.ones(h, dtype=torch.bfloat16, device=device), None)
        return self

    # ------------------------------------------------------------------ buffers
    def _alloc_buffers(self):
        t, dev = self.max_tokens, self.device
        bf = torch.bfloat16
        qkv_n = (self.num_q + 2 * self.num_kv) * self.head_dim
        # one extra block past the managed ones: a scratch page for padding rows of
        # CUDA-graph decode steps (the block manager never hands it out)
        self.scratch_block = self.num_kv_blocks
        if self.kv_fp8:
            # [layer, K | V, block, head, ...]: K pages [16, D] bytes, V pages transposed [D, 16]
            self.kv_cache = torch.zeros(self.num_layers, 2, self.num_kv_blocks + 1, self.num_kv, 16, self.head_dim,
                                        dtype=torch.uint8, device=dev)
            self.kv_scale = torch.ones(self.num_layers, 2, self.num_kv_blocks + 1, self.num_kv, 16,
                                       dtype=torch.float32, device=dev)
        else:
            self.kv_cache = torch.zeros(self.num_layers, 2, self.num_kv_blocks + 1, self.num_kv, 16, self.head_dim,
                                        dtype=bf, device=dev)
            self.kv_scale = None
        self.h = torch.empty(t, self.hidden, dtype=bf, device=dev)
        self.h2 = torch.empty(t, self.hidden, dtype=bf, device=dev) if self.tp_size > 1 else None
        self.x = torch.empty(t, self.hidden, dtype=bf, device=dev)
        self.qkv = torch.empty(t, qkv_n, dtype=bf, device=dev)
        self.attn = torch.empty(t, self.num_q * self.head_dim, dtype=bf, device=dev)
        self.act = torch.empty(t, max(self.inter, 1), dtype=bf, device=dev)
        moe = next((lw.moe for lw in self.layers if lw.moe is not None), None)
        if moe is not None:
            e, k = moe.num_experts, moe.top_k
            self.moe_pmax = (t * k + 127 * e + 127) // 128 * 128   # worst case of the padded segments
            self.moe_logits = torch.empty(t, moe.router.shape[0], dtype=torch.float32, device=dev)
            self.moe_ids = torch.empty(t * k, dtype=torch.int32, device=dev)
            self.moe_wts = torch.empty(t * k, dtype=torch.float32, device=dev)
            self.moe_slot = torch.empty(t * k, dtype=torch.int32, device=dev)
            self.moe_counts = torch.zeros(e, dtype=torch.int32, device=dev)
            self.moe_offsets = torch.empty(e, dtype=torch.int32, device=dev)
            self.moe_cursor = torch.empty(e, dtype=torch.int32, device=dev)
            self.moe_tiles = torch.empty(self.moe_pmax // 128, dtype=torch.int32, device=dev)
            self.moe_xp = torch.zeros(self.moe_pmax, self.hidden, dtype=bf, device=dev)
            self.moe_ap = torch.zeros(self.moe_pmax, moe.inter, dtype=bf, device=dev)
            self.moe_yp = torch.zeros(self.moe_pmax, self.hidden, dtype=bf, device=dev)
            self.moe_y = torch.empty(t, self.hidden, dtype=bf, device=dev)
        self.x2 = (torch.empty(t, self.hidden, dtype=bf, device=dev)
                   if moe is not None and self.has_shared_mlp else None)
        s_cols = 64
        for lw in self.layers:
            for pl in (lw.qkv, lw.o, lw.gu, lw.down, lw.cross):
                if pl is not None and pl.has_lora:
                    s_cols = max(s_cols, pl.a_all.shape[0])
        self.s_buf = torch.empty(t, s_cols, dtype=bf, device=dev)
        if self.dual:
            self.hbase = torch.empty(t, self.hidden, dtype=bf, device=dev)
            self.hbase2 = torch.empty(t, self.hidden, dtype=bf, device=dev) if self.tp_size > 1 else None
            self.qa = torch.empty(t, self.num_q * self.head_dim, dtype=bf, device=dev)
        if self.probe_w is not None:
            self.verdict = torch.zeros(self.max_seqs, self.probe_w.shape[1], dtype=torch.float32, device=dev)
        self.adapter_idx = torch.empty(t, dtype=torch.int32, device=dev)
        self.lora_idx = torch.empty(t, dtype=torch.int32, device=dev)
        self.mod_ids = torch.empty(t, dtype=torch.long, device=dev)
        self.carry_out = torch.empty(self.max_seqs, dtype=torch.int32, device=dev)
        n_tiles = (t + 127) // 128
        self.row_adapter = torch.empty(max(self.n_maps, 1), t, dtype=torch.int32, device=dev)
        self.tile_mask = torch.empty(max(self.n_maps, 1), n_tiles, dtype=torch.int64, device=dev)
        self.max_logit_rows = self.max_seqs
        self.xf = torch.empty(self.max_seqs, self.hidden, dtype=bf, device=dev)
        self.logits = torch.empty(self.max_seqs, self.lm_head_w.shape[0], dtype=torch.float32, device=dev)
        max_split = 32
        self.ws_o = torch.empty(max_split * min(t, 4 * self.max_seqs) * self.num_q * self.head_dim,
                                dtype=torch.float32, device=dev)
        self.ws_lse = torch.empty(max_split * min(t, 4 * self.max_seqs) * self.num_q, dtype=torch.float32, device=dev)
        self.ws_tokens = min(t, 4 * self.max_seqs)

    def kv_cache_bytes(self) -> int:
        n = self.kv_cache.numel() * self.kv_cache.element_size()
        if self.kv_scale is not None:
            n += self.kv_scale.numel() * 4
        return n

    def _layer_cache(self, li: int):
        """``(k_cache, v_cache, k_scale, v_scale)`` views of layer ``li`` (scales None for bf16)."""
        kc, vc = self.kv_cache[li, 0], self.kv_cache[li, 1]
        if not self.kv_fp8:
            return kc, vc, None, None
        nb = kc.shape[0]
        return kc, vc.view(nb, self.num_kv, self.head_dim, 16), self.kv_scale[li, 0], self.kv_scale[li, 1]

    def _rope_and_cache(self, b, qkv, li: int) -> None:
        """RoPE on q / k and the write of the step's K / V into layer ``li``'s cache."""
        kc, vc, ks, vs = self._layer_cache(li)
        if self.kv_fp8:
            A.rope_kv_fp8(qkv, b.positions, self.cos_sin, b.slots, kc, vc, ks, vs, self.num_q, self.num_kv,
                          self.head_dim)
        else:
            E.rope_kv(qkv, b.positions, self.cos_sin, self.num_q, self.num_kv, self.head_dim, kc, vc, b.slots)

    def _region(self, name: str):
        return self.prof.region(name) if self.prof is not None else contextlib.nullcontext()

    # ------------------------------------------------------------------ forward pieces
    def _proj(self, pl: PackedLinear, x: torch.Tensor, out: torch.Tensor, epi=G.EPI_STORE, residual=None,
              scale=1.0, mc_out: int = 0, lora: bool = True, n_rows: int | None = None):
        """``out <- epi(x @ W^T (+ switched LoRA))``.

        ``lora=False`` runs the base weight only (the Shadow-Residual base
        stream); ``n_rows`` restricts the projection to the first output rows
        of ``W``, which must be the first slice (the adapter stream's Q).
        """
        m = x.shape[0]
        w, lb, bounds = pl.w, pl.lb, pl.slice_bounds
        if n_rows is not None:
            assert n_rows == pl.slice_bounds[1], "n_rows must cover exactly the first slice"
            w, bounds = w[:n_rows], [0, n_rows]
            lb = lb[:n_rows] if lb is not None else None
        bn = pl.swiglu_tile if epi == G.EPI_SWIGLU else None
        if pl.has_lora and lora:
            ra = self.row_adapter[pl.map_id, :m]
            tm = self.tile_mask[pl.map_id, : (m + 127) // 128]
            a_all = pl.a_all
            if n_rows is not None:  # shrink of the first slice only
                a_all = a_all[: (pl.n_local * pl.rank + 63) // 64 * 64]
            s = self.s_buf[:m, : a_all.shape[0]]
            G.lora_shrink(x, a_all, ra, pl.rank, pl.n_local, out=s, tile_mask=tm)
            G.switched_gemm(x, w, out, epi=epi, residual=residual, scale=scale, s=s, lb=lb, tile_mask=tm,
                            rank=pl.rank, num_adapters=pl.n_local,
                            slice_bounds=[0, pl.n] if epi == G.EPI_SWIGLU else bounds, bn=bn,
                            mc_out=mc_out)
        else:
            G.switched_gemm(x, w, out, epi=epi, residual=residual, scale=scale, bn=bn, mc_out=mc_out)
        return out

    def _row_parallel(self, pl: PackedLinear, x: torch.Tensor, h: torch.Tensor, mult: float, lora: bool = True,
                      partial: torch.Tensor | None = None):
        """h <- h + x @ W^T * mult, summed over TP ranks."""
        m = x.shape[0]
        if self.tp_size == 1:
            self._proj(pl, x, h, epi=G.EPI_RESADD, residual=h, scale=mult, lora=lora)
            return
        y = (partial if partial is not None else self.h2)[:m]
        if self.tp_rank == 0:
            self._proj(pl, x, y, epi=G.EPI_RESADD, residual=h, scale=mult, lora=lora)
        else:
            self._proj(pl, x, y, epi=G.EPI_STORE, scale=mult, lora=lora)
        torch.distributed.all_reduce(y, group=self.tp_group)
        h.copy_(y)

    def _cross_stream(self, pl: PackedLinear, hbase: torch.Tensor, h: torch.Tensor) -> None:
        """Shadow Residual injection ``h <- h + (hbase A_a^T) B_a^T`` on rows routed to adapter a.

        The shrink is computed for every column (no tile mask), so S is exactly
        zero outside each row's own adapter, and the expand is one plain GEMM
        over all adapter columns (reference K4: kernels/switch_lora_kernel.py:883-1091).
        """
        if pl is None or not pl.has_lora:
            return
        m = hbase.shape[0]
        ra = self.row_adapter[pl.map_id, :m]
        s = self.s_buf[:m, : pl.a_all.shape[0]]
        G.lora_shrink(hbase, pl.a_all, ra, pl.rank, pl.n_local, out=s)
        G.switched_gemm(s, pl.lb, h, epi=G.EPI_RESADD, residual=h, scale=1.0)

    def _mlp(self, lw: LayerWeights, x: torch.Tensor, act: torch.Tensor, h: torch.Tensor, mult: float,
             lora: bool = True, reuse_routing: bool = False, partial: torch.Tensor | None = None) -> None:
        """``h <- h + MLP(x) * mult``: shared MLP, expert bank, or their sum (summed over TP ranks).

        ``lora=False`` runs base weights only; ``reuse_routing`` sends ``x`` to the
        experts (and slots) chosen by the previous call, which is how the
        Shadow-Residual adapter stream shares the base stream's routing
        (reference: src/granite_switch/hf/modeling_granite_switch.py:232-340).
        """
        R = self._region
        if lw.moe is None:
            with R("gate_up+swiglu"):
                self._proj(lw.gu, x, act, epi=G.EPI_SWIGLU, lora=lora)
            with R("down"):
                self._row_parallel(lw.down, act, h, mult, lora=lora, partial=partial)
            return
        m = x.shape[0]
        moe = lw.moe
        nat = native()
        k = moe.top_k
        with R("moe_route"):
            if reuse_routing:
                nat.moe_scatter_slots(x, self.moe_slot[: m * k], k, self.moe_xp)
            else:
                logits = self.moe_logits[:m]
                G.switched_gemm(x, moe.router, logits, epi=G.EPI_F32)
                nat.moe_route(logits, moe.num_experts, k, self.moe_ids[: m * k], self.moe_wts[: m * k],
                              self.moe_counts, self.moe_offsets, self.moe_cursor, self.moe_tiles)
                nat.moe_scatter(x, self.moe_ids[: m * k], self.moe_offsets, self.moe_cursor,
                                self.moe_slot[: m * k], self.moe_xp)
        rows = min(self.moe_pmax, (m * k + 127 * moe.num_experts + 127) // 128 * 128)
        tiles = self.moe_tiles[: rows // 128]
        with R("moe_experts"):
            G.switched_gemm(self.moe_xp[:rows], moe.gate_up, self.moe_ap[:rows], epi=G.EPI_SWIGLU,
                            bn=moe.swiglu_tile, tile_expert=tiles)
            G.switched_gemm(self.moe_ap[:rows], moe.down, self.moe_yp[:rows], tile_expert=tiles)
        shared = None
        if lw.gu is not None:
            with R("gate_up+swiglu"):
                self._proj(lw.gu, x, act, epi=G.EPI_SWIGLU, lora=lora)
            with R("down"):
                shared = self.x2[:m]
                self._proj(lw.down, act, shared, epi=G.EPI_STORE, lora=lora)
        with R("moe_combine"):
            if self.tp_size == 1:
                nat.moe_combine(self.moe_yp, self.moe_slot[: m * k], self.moe_wts[: m * k], k, shared, h, mult, h)
            else:
                y = self.moe_y[:m]
                nat.moe_combine(self.moe_yp, self.moe_slot[: m * k], self.moe_wts[: m * k], k, shared, None, 1.0, y)
                torch.distributed.all_reduce(y, group=self.tp_group)
                E.residual_axpy(h, y, mult)

    def _probe_layer(self, b: StepBatch, layer, hidden: torch.Tensor) -> None:
        """Probe scores of the markers that read ``layer`` (None: the final-norm rows)."""
        for lay, rows, slots, outj in b.probe_groups:
            if lay == layer:
                native().probe_verdict(hidden, rows, slots, outj, self.probe_w, self.probe_b, self.verdict)

    @torch.no_grad()
    def forward(self, b: StepBatch) -> torch.Tensor:
        """Run one step; returns fp32 logits ``[B, vocab(_shard)]`` for ``b.logit_rows``."""
        cfg = self.cfg
        t = b.num_tokens
        nat = native()
        R = self._region
        with R("routing+embed"):
            # every pipeline stage recomputes the routing metadata from the ids
            if self.n_maps:
                nat.routing(b.ids, b.seq_starts, b.carry_in, self.expert_tbl, None, self.kind_lut,
                            self.num_adapters, self.remaps, self.adapter_idx[:t], self.lora_idx[:t],
                            self.mod_ids[:t], self.carry_out[: b.num_seqs], self.row_adapter[:, :t],
                            self.tile_mask[:, : (t + 127) // 128])
            if self.first_stage:
                E.embed(b.ids, self.embed_w, self.lut, cfg.embedding_multiplier, out=self.h[:t])
        if not self.first_stage:
            with R("pp_recv"):
                self.pipeline.recv(self.h[:t], self.hbase[:t] if self.dual else None,
                                   self.verdict if self.probe_w is not None else None)
        h, x = self.h[:t], self.x[:t]
        qkv, attn, act = self.qkv[:t], self.attn[:t], self.act[:t]
        mult = float(cfg.residual_multiplier)
        scale = float(cfg.attention_multiplier)
        comm = self.comm
        probes = bool(b.probe_groups)
        if self.dual:
            self._forward_dual(b, h, x, qkv, attn, act, mult, scale)
        else:
            if comm is not None:
                with R("rmsnorm"):
                    E.rmsnorm(h, self.layers[0].in_norm, cfg.rms_norm_eps, out=x)
            for li, lw in enumerate(self.layers):
                if comm is None:
                    with R("rmsnorm"):
                        E.rmsnorm(h, lw.in_norm, cfg.rms_norm_eps, out=x)
                with R("qkv"):
                    self._proj(lw.qkv, x, qkv)
                with R("rope+kv"):
                    self._rope_and_cache(b, qkv, li)
                self._attention(b, qkv, li, attn, scale)
                if comm is not None:
                    with R("o+reduce"):
                        y = comm.row_parallel(self, lw.o, attn, h, mult)
                    with R("finish+rmsnorm"):
                        comm.finish(y, h, lw.post_norm, x, cfg.rms_norm_eps)
                else:
                    with R("o"):
                        self._row_parallel(lw.o, attn, h, mult)
                    with R("rmsnorm"):
                        E.rmsnorm(h, lw.post_norm, cfg.rms_norm_eps, out=x)
                if comm is not None:
                    with R("gate_up+swiglu"):
                        self._proj(lw.gu, x, act, epi=G.EPI_SWIGLU)
                    with R("down+reduce"):
                        y = comm.row_parallel(self, lw.down, act, h, mult)
                    nxt = self.layers[li + 1].in_norm if li + 1 < len(self.layers) else self.final_norm
                    with R("finish+rmsnorm"):
                        comm.finish(y, h, nxt, x, cfg.rms_norm_eps)
                else:
                    self._mlp(lw, x, act, h, mult)
                if probes:
                    self._probe_layer(b, self.layer_lo + li, h)
        if not self.last_stage:
            with R("pp_send"):
                self.pipeline.send(h, self.hbase[:t] if self.dual else None,
                                   self.verdict if self.probe_w is not None else None)
            return None
        nb = b.logit_rows.numel()
        if nb == 0:
            return None
        xf = self.xf[:nb]
        with R("lm_head"):
            E.rmsnorm(h, self.final_norm, cfg.rms_norm_eps, out=xf, rows=b.logit_rows)
            logits = self.logits[:nb]
            G.switched_gemm(xf, self.lm_head_w, logits, epi=G.EPI_F32, scale=1.0 / float(cfg.logits_scaling))
        if probes:
            self._probe_layer(b, None, xf)
            outj, slots = b.probe_all
            native().probe_rewrite(logits, self.lm_vocab_lo, outj, slots, self.probe_labels, self.verdict)
        return logits

    def _attention(self, b: StepBatch, q: torch.Tensor, li: int, attn: torch.Tensor, scale: float) -> None:
        """A step's attention plans. With ``overlap_attention`` and both a decode and a
        prefill plan, the prefill plan (a few CTAs over long key ranges: latency bound)
        runs on a side stream while the decode plan streams the decode rows' pages on the
        current one; the plans write disjoint rows of ``attn`` and of the split
        workspaces, and the current stream waits for the side stream before going on."""
        if self.overlap_attention and len(b.plans) == 2 and self.prof is None:
            main = torch.cuda.current_stream(self.device)
            if self._side_stream is None:
                self._side_stream = torch.cuda.Stream(device=self.device)
            side = self._side_stream
            side.wait_stream(main)
            with torch.cuda.stream(side):
                self._run_plans(b, q, li, attn, scale, b.plans[1:])
            self._run_plans(b, q, li, attn, scale, b.plans[:1])
            main.wait_stream(side)
            return
        self._run_plans(b, q, li, attn, scale, b.plans)

    def _run_plans(self, b: StepBatch, q: torch.Tensor, li: int, attn: torch.Tensor, scale: float,
                   plans) -> None:
        R = self._region
        kc, vc, ks, vs = self._layer_cache(li)
        for plan in plans:
            if plan.rows in (128, 256):
                with R("attn_prefill"):
                    A.prefill_attention_tc(q, kc, vc, b.block_table, b.seq_starts, b.kv_lens, plan.work_seq,
                                           plan.work_row0, self.num_q, scale, attn, plan.rows, plan.nsplit,
                                           self.ws_o, self.ws_lse)
            else:
                with R("attn_decode" if plan.rows in (8, 16) else "attn_prefill"):
                    A.paged_attention(q, kc, vc, b.block_table, b.seq_starts, b.kv_lens, plan.work_seq,
                                      plan.work_row0, plan.rows, self.num_q, scale, attn, plan.nsplit,
                                      self.ws_o, self.ws_lse, ks, vs)

    def _forward_dual(self, b: StepBatch, h, x, qkv, attn, act, mult: float, scale: float) -> None:
        """Shadow Residual layers (reference: src/granite_switch/vllm/decoder/shadow_residual/decoder.py:88-364).

        ``hbase`` is the base stream (no LoRA anywhere; it alone writes K/V),
        ``h`` the adapter stream: its queries (LoRA on the Q slice) attend to
        the base K/V, its o/MLP projections run the switched LoRA, and after
        the MLP it receives the cross-stream delta computed from ``hbase``.
        Logits are read from the adapter stream. Under tensor parallelism both
        streams are reduced over NCCL; the cross stream is replicated.
        """
        cfg = self.cfg
        R = self._region
        t = b.num_tokens
        hb = self.hbase[:t]
        if self.first_stage:
            hb.copy_(h)  # both streams start from the embedding
        qa = self.qa[:t]
        q_n = self.num_q * self.head_dim
        eps = cfg.rms_norm_eps
        hb2 = self.hbase2[:t] if self.hbase2 is not None else None
        for li, lw in enumerate(self.layers):
            # base stream: q, k, v without LoRA; k/v go to the cache
            with R("rmsnorm"):
                E.rmsnorm(hb, lw.in_norm, eps, out=x)
            with R("qkv"):
                self._proj(lw.qkv, x, qkv, lora=False)
            with R("rope+kv"):
                self._rope_and_cache(b, qkv, li)
            self._attention(b, qkv, li, attn, scale)
            with R("o"):
                self._row_parallel(lw.o, attn, hb, mult, lora=False, partial=hb2)
            # adapter stream: switched Q only, same base K/V
            with R("rmsnorm"):
                E.rmsnorm(h, lw.in_norm, eps, out=x)
            with R("qkv"):
                self._proj(lw.qkv, x, qa, n_rows=q_n)
            with R("rope+kv"):
                E.rope_kv(qa, b.positions, self.cos_sin, self.num_q, 0, self.head_dim)
            self._attention(b, qa, li, attn, scale)
            with R("o"):
                self._row_parallel(lw.o, attn, h, mult)
            # MLPs: base stream first (its output feeds the cross stream; with
            # experts, its routing is the adapter stream's too)
            with R("rmsnorm"):
                E.rmsnorm(hb, lw.post_norm, eps, out=x)
            self._mlp(lw, x, act, hb, mult, lora=False, partial=hb2)
            with R("rmsnorm"):
                E.rmsnorm(h, lw.post_norm, eps, out=x)
            self._mlp(lw, x, act, h, mult, reuse_routing=True)
            with R("cross_stream"):
                self._cross_stream(lw.cross, hb, h)
            if b.probe_groups:
                self._probe_layer(b, self.layer_lo + li, h)

    def attention_plans(self, q_lens: list[int], kv_lens: list[int]) -> list[tuple[list[int], list[int], int, int]]:
        """Split requests into decode-layout and prefill-layout CTA work lists."""
        g = self.num_q // self.num_kv
        dec = [i for i, ql in enumerate(q_lens) if ql * g <= 16]
        pre = [i for i, ql in enumerate(q_lens) if ql * g > 16]
        plans = []
        # the tcgen05 prefill kernel reads bf16 pages; an fp8 cache takes the mma.sync layouts
        tc = self.head_dim in (64, 128) and self.use_tc_attention and not self.kv_fp8
        pre_q, pre_kv = [q_lens[i] for i in pre], [kv_lens[i] for i in pre]
        # short chunks over long cached prefixes: split-KV layout (needs the split workspace)
        pre_split = (A.split_prefill(pre_q, pre_kv, g, self.num_kv, rows=128 if tc else 64)
                     if pre and sum(q_lens) <= self.ws_tokens else 0)
        if tc:
            pre_rows = 128 if pre_split else (A.tc_rows_for(pre_q, pre_kv) if pre else 64)
        else:
            pre_rows = 64
        # decode rows over an fp8 cache: 8-row tiles with the keys on the MMA's row side
        # (fp8_decode_rows = 16 selects the row-major layout, for A/B runs)
        dec_rows = getattr(self, "fp8_decode_rows", 8) if self.kv_fp8 else 16
        for idx, rows in ((dec, dec_rows), (pre, pre_rows)):
            if not idx:
                continue
            sub_q = [q_lens[i] for i in idx]
            sw, wr = A.build_work(sub_q, g, rows, [kv_lens[i] for i in idx] if rows != 16 else None)
            ws = [idx[t] for t in sw]
            n_ctas = len(ws) * self.num_kv
            max_kv = max(kv_lens[i] for i in idx)
            ns = A.choose_splits(n_ctas, max_kv) if rows == dec_rows else (pre_split or 1)
            tot = sum(q_lens)
            if ns > 1 and tot > self.ws_tokens:
                ns = 1
            plans.append((ws, wr, rows, ns))
        return plans


def audit_unread(config: GraniteSwitchConfig, unread: list[str], layer_lo: int, layer_hi: int) -> None:
    """Load audit: every checkpoint tensor must have been packed, except those this
    runtime does not use by design. A leftover name means a layout this loader does
    not understand (an unfused projection, a renamed module) whose weights would
    otherwise be dropped silently (reference: src/granite_switch/vllm/decoder/interface.py:95-127
    raises on unloaded parameters).

    Unused by design: the Kerdock codebook (routing is the exact scan), the
    all-zero cross-stream base weight of Shadow-Residual checkpoints, an LM head
    equal to the tied embedding, and other pipeline stages' layers.
    """
    import re

    bad = []
    for k in unread:
        if k == "model.switch.codebook" or k.endswith("cross_stream.base_layer.weight"):
            continue
        if k == "lm_head.weight" and config.tie_word_embeddings:
            continue
        m = re.match(r"model\.layers\.(\d+)\.", k)
        if m and not (layer_lo <= int(m.group(1)) < layer_hi):
            continue
        bad.append(k)
    if bad:
        more = f" (+{len(bad) - 8} more)" if len(bad) > 8 else ""
        raise ValueError(f"checkpoint tensors this loader does not use: {', '.join(bad[:8])}{more}")


def split_layers(num_layers: int, stage: int, stages: int) -> tuple[int, int]:
    """Contiguous layer range of a pipeline stage; earlier stages take the remainder."""
    base, extra = divmod(num_layers, stages)
    lo = stage * base + min(stage, extra)
    return lo, lo + base + (1 if stage < extra else 0)


def default_num_kv_blocks(model_bytes: int, cfg: GraniteSwitchConfig, tp_size: int, mem_fraction: float = 0.85,
                          device=None, reserve_bytes: int = 6 << 30, cap_blocks: int | None = None,
                          num_layers: int | None = None, kv_fp8: bool = False) -> int:
    free, total = torch.cuda.mem_get_info(device)
    d = cfg.head_dim_eff
    kv_heads = max(1, cfg.num_key_value_heads // tp_size)
    # bytes per 16-token block over all layers: bf16 K and V, or e4m3 K and V plus fp32 row scales
    per_row = d + 4 if kv_fp8 else 2 * d
    per_block = (num_layers or cfg.num_decoder_layers) * 2 * kv_heads * 16 * per_row
    budget = int(total * mem_fraction) - (total - free) - reserve_bytes
    n = max(64, budget // per_block)
    if cap_blocks is not None:
        n = min(n, cap_blocks)
    return int(n)


__all__ = ["NativeGraniteSwitch", "StepBatch", "AttnPlan", "default_num_kv_blocks", "split_layers", "math"]
