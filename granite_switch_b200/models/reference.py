"""HF-style ``GraniteSwitchForCausalLM`` in plain PyTorch: prototyping class and CPU oracle.

Same module tree and parameter names as the reference's HF model
(reference: src/granite_switch/hf/modeling_granite_switch.py:50-931), so a
composed checkpoint loads with ``from_pretrained`` and ``state_dict()`` saves
back in the same layout. Routing uses the exact latest-wins scan (see
:mod:`granite_switch_b200.routing.scan`) instead of the coded-memory attention
heads; the switch's persistent buffers (``codebook``,
``control_to_substitute_lut``, ``adapter_kind_lut``) are kept for format parity.

Granite numerics: ``h0 = embed(exchange(ids)) * embedding_multiplier``; per layer
``h += attn(norm(h)) * residual_multiplier``, ``h += mlp(norm(h)) * residual_multiplier``;
attention scale ``attention_multiplier``; ``logits = lm_head(norm(h)) / logits_scaling``.
Shadow Residual (``dual_stream``) runs a frozen base stream next to the adapter
stream, takes K/V from the base stream and adds ``cross_stream(h_base)`` per layer.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch
from torch import nn
from torch.nn import functional as F

from ..config import SWITCH_CACHE_LAYERS, GraniteSwitchConfig
from ..routing.codebook import KerdockDGCodeGenerator
from ..routing.scan import expert_table, probe_slot_mask, route_sequence, split_probe_stream
from ..routing.token_exchange import apply_token_exchange, build_control_to_substitute_lut
from .layers import (
    MergedSwitchedLoRALinear,
    RMSNorm,
    SwitchedLoRALinear,
    apply_rope,
    attention,
    rope_cos_sin,
)


# ----------------------------------------------------------------------------- cache
@dataclass
class SwitchCache:
    """Dense per-layer KV cache plus the routing carry of every batch row."""

    keys: list = field(default_factory=list)     # per layer [B, L, Hkv, d]
    values: list = field(default_factory=list)
    positions: torch.Tensor | None = None        # [B, L]
    valid: torch.Tensor | None = None            # [B, L] bool (padding mask)
    carry: torch.Tensor | None = None            # [B] last expert id seen

    def get_seq_length(self) -> int:
        return 0 if self.positions is None else int(self.positions.shape[1])

    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        if layer < len(self.keys):
            self.keys[layer] = torch.cat([self.keys[layer], k], dim=1)
            self.values[layer] = torch.cat([self.values[layer], v], dim=1)
        else:
            self.keys.append(k)
            self.values.append(v)
        return self.keys[layer], self.values[layer]


@dataclass
class CausalLMOutput:
    logits: torch.Tensor
    past_key_values: SwitchCache | None = None
    hidden_states: tuple | None = None
    adapter_indices: torch.Tensor | None = None


# ----------------------------------------------------------------------------- switch
class GraniteSwitchRouter(nn.Module):
    """Per-token adapter routing + token exchange (module name ``model.switch``)."""

    def __init__(self, config: GraniteSwitchConfig):
        super().__init__()
        self.config = config
        self.num_adapters = config.num_adapters
        gen = KerdockDGCodeGenerator(m=config.ms_code_m, code_type=config.ms_code_type)
        self.register_buffer("codebook", gen.precompute_codebook(torch.float32), persistent=True)
        lut = build_control_to_substitute_lut(config)
        if lut is not None:
            self.register_buffer("control_to_substitute_lut", lut, persistent=True)
        else:
            self.control_to_substitute_lut = None
        kind = probe_slot_mask(getattr(config, "adapter_kinds", None))
        if kind is not None:
            self.register_buffer("adapter_kind_lut", kind, persistent=True)
        else:
            self.adapter_kind_lut = None
        self._table = expert_table(config.adapter_token_ids or [], config.num_adapters)

    def _apply(self, fn, *args, **kwargs):
        # The codebook stays fp32 under .to(dtype) so save/load is idempotent.
        out = super()._apply(fn, *args, **kwargs)
        if self.codebook.dtype != torch.float32:
            self.codebook = self.codebook.float()
        return out

    @property
    def num_cache_layers(self) -> int:
        return SWITCH_CACHE_LAYERS

    def forward(self, input_ids: torch.Tensor, carry: torch.Tensor | None = None):
        """``input_ids [B, S]`` -> ``(adapter_indices [B,S], modified_ids [B,S], carry [B])``."""
        b = input_ids.shape[0]
        out = torch.zeros_like(input_ids, dtype=torch.long)
        new_carry = torch.zeros(b, dtype=torch.long)
        cpu = input_ids.detach().cpu()
        for i in range(b):
            c = int(carry[i]) if carry is not None else 0
            out[i], new_carry[i] = route_sequence(cpu[i], self._table, c)
        out = out.to(input_ids.device)
        modified = apply_token_exchange(self.control_to_substitute_lut, input_ids)
        return out, modified, new_carry

    def split_indices(self, adapter_indices: torch.Tensor):
        return split_probe_stream(adapter_indices, self.adapter_kind_lut)


class SwitchedProbeHead(nn.Module):
    """Probe bank ``weight [NA, Lmax, H]``, ``bias [NA, Lmax]`` indexed by ``slot - 1``."""

    def __init__(self, hidden: int, num_slots: int, max_labels: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(num_slots, max_labels, hidden))
        self.bias = nn.Parameter(torch.zeros(num_slots, max_labels))

    def forward(self, x: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
        w = self.weight[slots - 1]  # [n, L, H]
        return torch.einsum("nlh,nh->nl", w.float(), x.float()) + self.bias[slots - 1].float()


# ----------------------------------------------------------------------------- blocks
class GraniteSwitchAttention(nn.Module):
    def __init__(self, config: GraniteSwitchConfig, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.num_heads = config.num_attention_heads
        self.num_kv = config.num_key_value_heads
        self.head_dim = config.head_dim_eff
        self.scaling = float(config.attention_multiplier)
        q, kv = self.num_heads * self.head_dim, self.num_kv * self.head_dim
        self.q_size, self.kv_size = q, kv
        na, r = config.num_adapters, config.max_lora_rank
        bias = bool(config.attention_bias)
        if "qkv_proj" in config.lora_target_modules:
            self.qkv_proj = MergedSwitchedLoRALinear(config.hidden_size, (q, kv, kv), na, r, bias)
            self.has_qkv_lora = True
        else:
            self.qkv_proj = nn.Linear(config.hidden_size, q + 2 * kv, bias=bias)
            self.has_qkv_lora = False
        if "o_proj" in config.lora_target_modules:
            self.o_proj = SwitchedLoRALinear(q, config.hidden_size, na, r, bias)
            self.has_o_lora = True
        else:
            self.o_proj = nn.Linear(q, config.hidden_size, bias=bias)
            self.has_o_lora = False

    def project_qkv(self, x, idx, cos, sin):
        qkv = self.qkv_proj(x, idx) if self.has_qkv_lora else self.qkv_proj(x)
        b, s, _ = x.shape
        q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
        q = apply_rope(q.view(b, s, self.num_heads, self.head_dim), cos, sin)
        k = apply_rope(k.view(b, s, self.num_kv, self.head_dim), cos, sin)
        return q, k, v.view(b, s, self.num_kv, self.head_dim)

    def out(self, o, idx):
        b, s = o.shape[:2]
        o = o.reshape(b, s, self.num_heads * self.head_dim)
        return self.o_proj(o, idx) if self.has_o_lora else self.o_proj(o)


class GraniteSwitchMLP(nn.Module):
    """Dense shared MLP: ``input_linear`` = fused gate|up, ``output_linear`` = down."""

    def __init__(self, config: GraniteSwitchConfig):
        super().__init__()
        i, h = config.shared_intermediate_size, config.hidden_size
        na, r = config.num_adapters, config.max_lora_rank
        if "shared_input_linear" in config.lora_target_modules:
            self.input_linear = MergedSwitchedLoRALinear(h, (i, i), na, r, False)
            self.in_lora = True
        else:
            self.input_linear = nn.Linear(h, 2 * i, bias=False)
            self.in_lora = False
        if "shared_output_linear" in config.lora_target_modules:
            self.output_linear = SwitchedLoRALinear(i, h, na, r, False)
            self.out_lora = True
        else:
            self.output_linear = nn.Linear(i, h, bias=False)
            self.out_lora = False

    def forward(self, x, idx):
        gu = self.input_linear(x, idx) if self.in_lora else self.input_linear(x)
        g, u = gu.chunk(2, dim=-1)
        a = F.silu(g) * u
        return self.output_linear(a, idx) if self.out_lora else self.output_linear(a)


class GraniteMoEExperts(nn.Module):
    def __init__(self, config: GraniteSwitchConfig):
        super().__init__()
        e, i, h = config.num_local_experts, config.intermediate_size, config.hidden_size
        self.gate_up_proj = nn.Parameter(torch.zeros(e, 2 * i, h))
        self.down_proj = nn.Parameter(torch.zeros(e, h, i))


class GraniteMoERouter(nn.Module):
    def __init__(self, config: GraniteSwitchConfig):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(config.num_local_experts, config.hidden_size))


class GraniteMoE(nn.Module):
    """Frozen top-k routed expert bank (never a LoRA target)."""

    def __init__(self, config: GraniteSwitchConfig):
        super().__init__()
        self.top_k = config.num_experts_per_tok
        self.experts = GraniteMoEExperts(config)
        self.router = GraniteMoERouter(config)

    def route(self, x):
        logits = (x.reshape(-1, x.shape[-1]) @ self.router.weight.t()).float()
        vals, idx = logits.topk(self.top_k, dim=1)
        return idx, torch.softmax(vals, dim=1).to(x.dtype)

    def forward(self, x, routing=None):
        shp = x.shape
        flat = x.reshape(-1, shp[-1])
        idx, w = routing if routing is not None else self.route(x)
        out = torch.zeros_like(flat)
        for e in idx.unique().tolist():
            rows, slot = (idx == e).nonzero(as_tuple=True)
            gu = flat[rows] @ self.experts.gate_up_proj[e].t()
            g, u = gu.chunk(2, dim=-1)
            y = (F.silu(g) * u) @ self.experts.down_proj[e].t()
            out.index_add_(0, rows, y * w[rows, slot].unsqueeze(1))
        return out.view(shp)


class GraniteSwitchDecoderLayer(nn.Module):
    def __init__(self, config: GraniteSwitchConfig, layer_idx: int):
        super().__init__()
        self.residual_multiplier = float(config.residual_multiplier)
        self.self_attn = GraniteSwitchAttention(config, layer_idx)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.block_sparse_moe = GraniteMoE(config) if config.num_local_experts > 0 else None
        self.shared_mlp = GraniteSwitchMLP(config) if config.shared_intermediate_size > 0 else None
        if self.block_sparse_moe is None and self.shared_mlp is None:
            raise ValueError("a decoder layer needs an MLP path (experts or shared MLP)")

    def mlp(self, x, idx, routing=None):
        out = None
        if self.block_sparse_moe is not None:
            out = self.block_sparse_moe(x, routing)
        if self.shared_mlp is not None:
            s = self.shared_mlp(x, idx)
            out = s if out is None else out + s
        return out

    def forward(self, h, idx, cos, sin, cache: SwitchCache | None, q_pos, k_pos, key_valid, layer):
        x = self.input_layernorm(h)
        q, k, v = self.self_attn.project_qkv(x, idx, cos, sin)
        if cache is not None:
            k, v = cache.append(layer, k, v)
        o = attention(q, k, v, self.self_attn.scaling, q_pos, k_pos, key_valid)
        h = h + self.self_attn.out(o, idx) * self.residual_multiplier
        x = self.post_attention_layernorm(h)
        return h + self.mlp(x, idx) * self.residual_multiplier


class SRSwitchDecoderLayer(GraniteSwitchDecoderLayer):
    """Shadow Residual layer: base stream (no LoRA) + adapter stream with base K/V."""

    def __init__(self, config: GraniteSwitchConfig, layer_idx: int):
        super().__init__(config, layer_idx)
        self.cross_stream = SwitchedLoRALinear(config.hidden_size, config.hidden_size,
                                               config.num_adapters, config.cross_stream_rank, False)
        nn.init.zeros_(self.cross_stream.base_layer.weight)

    def forward_dual(self, hb, ha, idx, cos, sin, cache, q_pos, k_pos, key_valid, layer):
        xb = self.input_layernorm(hb)
        xa = self.input_layernorm(ha)
        qb, k, v = self.self_attn.project_qkv(xb, None, cos, sin)
        if cache is not None:
            k, v = cache.append(layer, k, v)
        ob = attention(qb, k, v, self.self_attn.scaling, q_pos, k_pos, key_valid)
        qa, _, _ = self.self_attn.project_qkv(xa, idx, cos, sin)  # only Q of the adapter stream
        oa = attention(qa, k, v, self.self_attn.scaling, q_pos, k_pos, key_valid)
        hb = hb + self.self_attn.out(ob, None) * self.residual_multiplier
        ha = ha + self.self_attn.out(oa, idx) * self.residual_multiplier
        xb = self.post_attention_layernorm(hb)
        xa = self.post_attention_layernorm(ha)
        routing = self.block_sparse_moe.route(xb) if self.block_sparse_moe is not None else None
        hb = hb + self.mlp(xb, None, routing) * self.residual_multiplier
        ha = ha + self.mlp(xa, idx, routing) * self.residual_multiplier
        ha = ha + self.cross_stream(hb, idx)
        return hb, ha


# ----------------------------------------------------------------------------- model
class GraniteSwitchModel(nn.Module):
    def __init__(self, config: GraniteSwitchConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.switch = GraniteSwitchRouter(config) if config.num_adapters > 0 else None
        if "probe" in (config.adapter_kinds or []):
            self.probe_head = SwitchedProbeHead(config.hidden_size, config.num_adapters,
                                                config.max_probe_labels)
        else:
            self.probe_head = None
        cls = SRSwitchDecoderLayer if config.dual_stream else GraniteSwitchDecoderLayer
        offset = SWITCH_CACHE_LAYERS if config.num_adapters > 0 else 0
        self.layers = nn.ModuleList([cls(config, i + offset) for i in range(config.num_decoder_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self._last = {}

    def forward(self, input_ids, attention_mask=None, position_ids=None, past_key_values=None,
                use_cache=False):
        cfg = self.config
        b, s = input_ids.shape
        dev = input_ids.device
        cache = past_key_values
        if use_cache and cache is None:
            cache = SwitchCache()
        past = cache.get_seq_length() if cache is not None else 0
        if attention_mask is None:
            attention_mask = torch.ones(b, past + s, dtype=torch.long, device=dev)
        valid_new = attention_mask[:, -s:].bool()
        if position_ids is None:
            prev = cache.positions[:, -1:] + 1 if (cache is not None and past > 0) else torch.zeros(b, 1, dtype=torch.long, device=dev)
            position_ids = (prev + torch.cumsum(valid_new.long(), dim=1) - 1).clamp(min=0)
        if self.switch is not None:
            carry = cache.carry if cache is not None else None
            idx, ids, new_carry = self.switch(input_ids, carry)
            lora_idx, probe_idx = self.switch.split_indices(idx)
        else:
            idx = torch.zeros_like(input_ids)
            ids, new_carry = input_ids, torch.zeros(b, dtype=torch.long)
            lora_idx, probe_idx = idx, idx
        if cache is not None:
            cache.carry = new_carry
            cache.positions = position_ids if cache.positions is None else torch.cat([cache.positions, position_ids], 1)
            cache.valid = valid_new if cache.valid is None else torch.cat([cache.valid, valid_new], 1)
            k_pos, key_valid = cache.positions, cache.valid
        else:
            k_pos, key_valid = position_ids, valid_new
        self._last = {"adapter_indices": idx, "lora_indices": lora_idx, "probe_indices": probe_idx}

        h = self.embed_tokens(ids) * cfg.embedding_multiplier
        cos, sin = rope_cos_sin(position_ids, cfg.head_dim_eff, cfg.rope_theta, h.dtype)
        markers = self._locate_markers(input_ids, probe_idx, valid_new)
        verdict = None
        if markers is not None:
            verdict = torch.zeros(markers[0].numel(), cfg.max_probe_labels, dtype=torch.float32, device=dev)
        read_layers = cfg.probe_read_layers or [None] * cfg.num_adapters

        def score(layer, hidden):
            if markers is None:
                return
            rows, pos, slots = markers
            for j in range(rows.numel()):
                slot = int(slots[j])
                if read_layers[slot - 1] == layer:
                    verdict[j] = self.probe_head(hidden[rows[j], pos[j]].unsqueeze(0), slots[j:j + 1])[0]

        hb = h if cfg.dual_stream else None
        for li, layer in enumerate(self.layers):
            if cfg.dual_stream:
                hb, h = layer.forward_dual(hb, h, lora_idx, cos, sin, cache, position_ids, k_pos, key_valid, li)
            else:
                h = layer(h, lora_idx, cos, sin, cache, position_ids, k_pos, key_valid, li)
            score(li, h)
        h = self.norm(h)
        score(None, h)
        self._last["probe"] = None if markers is None else (*markers, verdict)
        return h, cache

    # routing introspection of the last forward, under the reference's attribute names
    # (src/granite_switch/hf/modeling_granite_switch.py:679-681,704,756-762)
    @property
    def _last_adapter_indices(self):
        return getattr(self, "_last", {}).get("adapter_indices")

    @property
    def _last_lora_indices(self):
        return getattr(self, "_last", {}).get("lora_indices")

    @property
    def _last_probe_indices(self):
        return getattr(self, "_last", {}).get("probe_indices")

    @property
    def _last_probe_verdict(self):
        probe = getattr(self, "_last", {}).get("probe")
        return None if probe is None else probe[-1]

    def _locate_markers(self, input_ids, probe_idx, valid):
        if self.probe_head is None:
            return None
        ids = torch.tensor(self.config.probe_control_token_ids, device=input_ids.device)
        rows, pos = torch.isin(input_ids, ids).nonzero(as_tuple=True)
        if rows.numel() == 0:
            return None
        cols = torch.arange(input_ids.shape[1], device=input_ids.device)
        last = (valid.long() * cols).max(dim=1).values
        if bool((pos != last[rows]).any()):
            raise RuntimeError("a probe control token must be its request's last token")
        return rows, pos, probe_idx[rows, pos]


class GraniteSwitchForCausalLM(nn.Module):
    """Causal LM head over :class:`GraniteSwitchModel`; ``lm_head`` tied unless configured."""

    def __init__(self, config: GraniteSwitchConfig):
        super().__init__()
        self.config = config
        self.model = GraniteSwitchModel(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight

    # -------------------------------------------------------------- forward
    def forward(self, input_ids, attention_mask=None, position_ids=None, past_key_values=None,
                use_cache=False, logits_to_keep: int = 0):
        h, cache = self.model(input_ids, attention_mask, position_ids, past_key_values, use_cache)
        s = h.shape[1]
        sl = slice(-logits_to_keep, None) if logits_to_keep else slice(None)
        logits = self.lm_head(h[:, sl]).float() / self.config.logits_scaling
        probe = self.model._last.get("probe")
        if probe is not None:
            rows, pos, slots, verdict = probe
            first = s - logits.shape[1]
            for j in range(rows.numel()):
                c = int(pos[j]) - first
                if c < 0:
                    raise RuntimeError("a probe marker's logits were not kept (logits_to_keep)")
                ids = self.config.probe_label_token_ids[int(slots[j]) - 1]
                logits[rows[j], c] = float("-inf")
                logits[rows[j], c, torch.tensor(ids)] = verdict[j, :len(ids)]
        return CausalLMOutput(logits=logits, past_key_values=cache,
                              adapter_indices=self.model._last.get("adapter_indices"))

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 16, attention_mask=None,
                 eos_token_id: int | None = None, do_sample: bool = False, temperature: float = 1.0,
                 generator: torch.Generator | None = None) -> torch.Tensor:
        """Greedy (or temperature) decoding with the KV cache. Returns prompt + new tokens."""
        out = self(input_ids, attention_mask=attention_mask, use_cache=True, logits_to_keep=1)
        cache = out.past_key_values
        seqs = input_ids
        mask = attention_mask
        done = torch.zeros(input_ids.shape[0], dtype=torch.bool, device=input_ids.device)
        for _ in range(max_new_tokens):
            logits = out.logits[:, -1]
            if do_sample:
                p = torch.softmax(logits / temperature, dim=-1)
                nxt = torch.multinomial(p, 1, generator=generator).squeeze(1)
            else:
                nxt = logits.argmax(dim=-1)
            if eos_token_id is not None:
                nxt = torch.where(done, torch.full_like(nxt, eos_token_id), nxt)
                done = done | (nxt == eos_token_id)
            seqs = torch.cat([seqs, nxt.unsqueeze(1)], dim=1)
            if mask is not None:
                mask = torch.cat([mask, torch.ones_like(mask[:, :1])], dim=1)
            if eos_token_id is not None and bool(done.all()):
                break
            out = self(nxt.unsqueeze(1), attention_mask=mask, past_key_values=cache, use_cache=True)
            cache = out.past_key_values
        return seqs

    # -------------------------------------------------------------- io
    def state_dict_for_save(self) -> dict[str, torch.Tensor]:
        sd = {k: v for k, v in self.state_dict().items()}
        if self.config.tie_word_embeddings:
            sd.pop("lm_head.weight", None)
        return sd

    def save_pretrained(self, path: str, max_shard_bytes: int = 5 * 1024 ** 3) -> None:
        from ..checkpoint import save_state_dict

        os.makedirs(path, exist_ok=True)
        self.config.save_pretrained(path)
        save_state_dict(self.state_dict_for_save(), path, max_shard_bytes=max_shard_bytes)

    @classmethod
    def from_pretrained(cls, path: str, dtype: torch.dtype = torch.float32, device="cpu",
                        strict: bool = True, **hf_kwargs) -> "GraniteSwitchForCausalLM":
        """Load a composed directory. ``hf_kwargs`` are what ``AutoModelForCausalLM``
        passes (``config``, ``torch_dtype`` / ``dtype``, hub options): a dtype among them
        is honoured, the rest is ignored since the checkpoint is read locally."""
        from ..checkpoint import load_state_dict

        hf_dtype = hf_kwargs.get("torch_dtype", hf_kwargs.get("dtype"))
        if isinstance(hf_dtype, torch.dtype):
            dtype = hf_dtype

        config = GraniteSwitchConfig.from_pretrained(path)
        model = cls(config)
        sd = load_state_dict(path)
        missing, unexpected = model.load_state_dict(sd, strict=False)
        missing = [m for m in missing if not (config.tie_word_embeddings and m == "lm_head.weight")]
        if strict and (missing or unexpected):
            raise RuntimeError(f"checkpoint mismatch: missing={missing[:8]} unexpected={unexpected[:8]}")
        if config.tie_word_embeddings:
            model.lm_head.weight = model.model.embed_tokens.weight
        return model.to(device=device, dtype=dtype)


def load_model(path: str, **kw) -> GraniteSwitchForCausalLM:
    """Convenience loader (reference: src/granite_switch/hf/__init__.py:26-42)."""
    return GraniteSwitchForCausalLM.from_pretrained(path, **kw)


def read_adapter_index(path: str) -> dict | None:
    p = os.path.join(path, "adapter_index.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f)
