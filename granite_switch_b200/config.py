"""``GraniteSwitchConfig``: the composed checkpoint's ``config.json`` schema.

Field names, defaults and validation rules follow the reference's
``GraniteSwitchConfig`` (reference: src/granite_switch/config.py:34-546) so a
checkpoint written by either project loads in the other. This class does not
subclass a ``transformers`` config: it is a plain attribute bag with
``from_dict`` / ``to_dict`` / ``from_pretrained`` / ``save_pretrained`` so the
runtime does not depend on a particular ``transformers`` version. Unknown keys
of ``config.json`` are kept verbatim and written back.
"""
from __future__ import annotations

import copy
import json
import os
from typing import Any

# Accepted asr_dtype values (reference: config.py:7).
ASR_DTYPES = ("auto", "float16", "bfloat16", "float32")
DEFAULT_ASR_MODEL_ID = "ibm-granite/granite-speech-5.0-470m-turboctc"
DEFAULT_ASR_MODEL_REVISION = "947f59af40db9791170a0628cf0f3f4812d720f1"
ASR_BUNDLE_DIR = "asr"

# Decoder-layer slots the reference's coded-memory switch reserves at the front
# of the model: the composer inflates num_hidden_layers by this count and every
# loader subtracts it to get the physical decoder depth (reference:
# config.py:25-31, compose_utils.py:252-255). This runtime routes with an exact
# scan and keeps no KV for these slots, but the count stays part of the format.
SWITCH_CACHE_LAYERS = 2

# Base-model fields copied from the base checkpoint (reference:
# composer/arch.py:282-330) with the defaults of a dense Granite 4 config.
_BASE_DEFAULTS: dict[str, Any] = {
    "vocab_size": 49152,
    "hidden_size": 2048,
    "intermediate_size": 8192,
    "num_hidden_layers": 32,
    "num_attention_heads": 32,
    "num_key_value_heads": 8,
    "hidden_act": "silu",
    "max_position_embeddings": 131072,
    "initializer_range": 0.02,
    "rms_norm_eps": 1e-5,
    "use_cache": True,
    "pad_token_id": None,
    "bos_token_id": None,
    "eos_token_id": None,
    "tie_word_embeddings": True,
    "rope_theta": 10000.0,
    "rope_scaling": None,
    "attention_bias": False,
    "attention_dropout": 0.0,
    "torch_dtype": "bfloat16",
    "residual_multiplier": 1.0,
    "embedding_multiplier": 1.0,
    "logits_scaling": 1.0,
    "attention_multiplier": None,
    "num_experts_per_tok": 0,
    "shared_intermediate_size": None,
    "head_dim": None,
}


class GraniteSwitchConfig:
    """Configuration of a composed Granite Switch checkpoint.

    Adapter index 0 is always the base model; index ``i >= 1`` selects the
    adapter (or probe) in slot ``i - 1``. ``adapter_token_ids`` has
    ``num_adapters`` entries, or ``num_adapters + 1`` when the first entry is a
    base-reset token that routes back to index 0.
    """

    model_type = "granite_switch"

    def __init__(
        self,
        num_adapters: int = 0,
        adapter_token_ids: list[int] | None = None,
        adapter_substitute_token_ids: list[int] | None = None,
        control_token_gain: float = 15.0,
        switch_head_dim: int = 32,
        ms_code_m: int = 6,
        ms_code_type: str = "kerdock",
        ms_memory_gain: float = 28.0,
        ms_counting_head_dim: int = 32,
        adapter_names: list[str] | None = None,
        max_lora_rank: int = 8,
        adapter_ranks: list[int] | None = None,
        lora_target_modules: list[str] | None = None,
        asr_enabled: bool = False,
        asr_model_id: str | None = None,
        asr_model_revision: str | None = None,
        asr_bundled_path: str | None = None,
        asr_device: str = "cuda",
        asr_dtype: str | None = None,
        asr_pipeline_kwargs: dict | None = None,
        asr_generate_kwargs: dict | None = None,
        asr_max_audio_clips: int = 32,
        asr_chunk_length_s: float = 120.0,
        asr_chunk_overlap_s: float = 5.0,
        asr_self_chunks: bool = False,
        cross_stream_rank: int | None = None,
        dual_stream: bool = False,
        adapter_kinds: list[str] | None = None,
        probe_label_token_ids: list[list[int] | None] | None = None,
        probe_read_layers: list[int | None] | None = None,
        fused_add_norm: bool = False,
        num_local_experts: int = 0,
        position_embedding_type: str = "rope",
        layer_types: list[str] | None = None,
        **kwargs: Any,
    ):
        extra = dict(kwargs)
        for k, v in _BASE_DEFAULTS.items():
            setattr(self, k, extra.pop(k, v))
        # transformers 5 serialises RoPE as ``rope_parameters`` and the dtype as
        # ``dtype`` (the reference's composer writes these); both stay in the
        # extra keys so they round-trip
        rp = extra.get("rope_parameters")
        if isinstance(rp, dict) and "rope_theta" not in kwargs and rp.get("rope_theta") is not None:
            self.rope_theta = float(rp["rope_theta"])
            if rp.get("rope_type") not in (None, "default") and self.rope_scaling is None:
                self.rope_scaling = {k: v for k, v in rp.items() if k != "rope_theta"}
        if extra.get("dtype") is not None and "torch_dtype" not in kwargs:
            self.torch_dtype = str(extra["dtype"]).replace("torch.", "")
        # derived / placeholder values that the reference's parent class provides
        if self.attention_multiplier is None:
            hd = self.head_dim or (self.hidden_size // self.num_attention_heads)
            self.attention_multiplier = 1.0 / float(hd) ** 0.5
        # Keys the reference writes and this runtime does not interpret.
        for k in ("architectures", "auto_map", "transformers_version", "projection_head_dim",
                  "probe_num_labels_per_slot", "max_probe_labels", "probe_control_token_ids"):
            extra.pop(k, None)
        if extra.get("unfused_qkv"):
            raise ValueError(
                "This checkpoint sets unfused_qkv=True, so it was composed with the old "
                "unfused Shadow Residual layout. Re-compose it from its PEFT adapters."
            )
        self._extra = extra

        self.num_local_experts = num_local_experts
        self.position_embedding_type = position_embedding_type
        if layer_types is None:
            layer_types = ["full_attention"] * self.num_hidden_layers
        self.layer_types = layer_types
        if self.shared_intermediate_size is None:
            self.shared_intermediate_size = 0 if num_local_experts > 0 else self.intermediate_size

        if num_adapters < 0:
            raise ValueError(f"num_adapters must be >= 0, got {num_adapters}")
        self.num_adapters = num_adapters
        self.ms_code_m = ms_code_m
        self.ms_code_type = ms_code_type
        self.ms_memory_gain = ms_memory_gain
        self.ms_counting_head_dim = ms_counting_head_dim

        allowed = (num_adapters, num_adapters + 1)
        if num_adapters > 0 and adapter_token_ids is not None:
            if len(adapter_token_ids) not in allowed:
                raise ValueError(
                    f"adapter_token_ids length ({len(adapter_token_ids)}) must be one of "
                    f"{allowed} (num_adapters={num_adapters})."
                )
            if len(set(adapter_token_ids)) != len(adapter_token_ids):
                raise ValueError(f"adapter_token_ids must be unique; got {adapter_token_ids}")
        self.adapter_token_ids = list(adapter_token_ids) if adapter_token_ids is not None else None

        if num_adapters > 0:
            if adapter_substitute_token_ids is None:
                raise ValueError(
                    "adapter_substitute_token_ids is required when num_adapters > 0: every "
                    "control token needs a substitute id whose embedding replaces it."
                )
            if len(adapter_substitute_token_ids) not in allowed:
                raise ValueError(
                    f"adapter_substitute_token_ids length ({len(adapter_substitute_token_ids)})"
                    f" must be one of {allowed} (num_adapters={num_adapters})."
                )
            if adapter_token_ids is not None and len(adapter_substitute_token_ids) != len(
                adapter_token_ids
            ):
                raise ValueError(
                    "adapter_token_ids and adapter_substitute_token_ids must have the same "
                    f"length; got {len(adapter_token_ids)} and "
                    f"{len(adapter_substitute_token_ids)}."
                )
            if any(s < 0 for s in adapter_substitute_token_ids):
                raise ValueError(
                    "adapter_substitute_token_ids must all be >= 0 (real token ids); got "
                    f"{adapter_substitute_token_ids}"
                )
            if adapter_token_ids is None:
                raise ValueError(
                    "adapter_token_ids is required when adapter_substitute_token_ids is given."
                )
        self.adapter_substitute_token_ids = (
            list(adapter_substitute_token_ids) if adapter_substitute_token_ids is not None else None
        )

        self.control_token_gain = control_token_gain
        self.switch_head_dim = switch_head_dim
        self.fused_add_norm = fused_add_norm

        self.asr_enabled = asr_enabled
        self.asr_model_id = asr_model_id
        self.asr_model_revision = asr_model_revision
        self.asr_bundled_path = asr_bundled_path
        self.asr_device = asr_device
        if asr_dtype is not None and asr_dtype not in ASR_DTYPES:
            raise ValueError(f"asr_dtype must be one of {ASR_DTYPES} or None, got {asr_dtype!r}")
        self.asr_dtype = asr_dtype
        self.asr_pipeline_kwargs = asr_pipeline_kwargs
        self.asr_generate_kwargs = asr_generate_kwargs
        if asr_max_audio_clips < 1:
            raise ValueError(f"asr_max_audio_clips must be >= 1, got {asr_max_audio_clips}")
        if asr_chunk_overlap_s >= asr_chunk_length_s:
            raise ValueError(
                f"asr_chunk_overlap_s ({asr_chunk_overlap_s}) must be < asr_chunk_length_s "
                f"({asr_chunk_length_s})"
            )
        self.asr_max_audio_clips = asr_max_audio_clips
        self.asr_chunk_length_s = asr_chunk_length_s
        self.asr_chunk_overlap_s = asr_chunk_overlap_s
        self.asr_self_chunks = asr_self_chunks

        self.dual_stream = bool(dual_stream)
        self.cross_stream_rank = cross_stream_rank
        if self.dual_stream and cross_stream_rank is None:
            raise ValueError("cross_stream_rank is required when dual_stream is True.")
        if not self.dual_stream and cross_stream_rank is not None:
            raise ValueError(
                f"cross_stream_rank must be None when dual_stream is False; got {cross_stream_rank}."
            )

        self.adapter_names = list(adapter_names) if adapter_names is not None else None
        self.projection_head_dim = (
            self.head_dim if self.head_dim is not None else self.hidden_size // self.num_attention_heads
        )

        if num_adapters > 0:
            if adapter_ranks is None:
                raise ValueError("adapter_ranks must be provided when num_adapters > 0")
            if len(adapter_ranks) != num_adapters:
                raise ValueError(
                    f"adapter_ranks length ({len(adapter_ranks)}) must equal num_adapters "
                    f"({num_adapters})"
                )
            if max(adapter_ranks) != max_lora_rank:
                raise ValueError(
                    f"max(adapter_ranks)={max(adapter_ranks)} must equal max_lora_rank={max_lora_rank}"
                )
        self.max_lora_rank = max_lora_rank
        self.adapter_ranks = list(adapter_ranks) if adapter_ranks is not None else None

        valid_kinds = ("lora", "probe")
        if adapter_kinds is None:
            adapter_kinds = ["lora"] * num_adapters
        else:
            if len(adapter_kinds) != num_adapters:
                raise ValueError(
                    f"adapter_kinds length ({len(adapter_kinds)}) must equal num_adapters "
                    f"({num_adapters})."
                )
            bad = [k for k in adapter_kinds if k not in valid_kinds]
            if bad:
                raise ValueError(f"adapter_kinds values must be one of {valid_kinds}; got {bad}")
        self.adapter_kinds = list(adapter_kinds)

        if probe_label_token_ids is not None:
            if len(probe_label_token_ids) != num_adapters:
                raise ValueError(
                    f"probe_label_token_ids length ({len(probe_label_token_ids)}) must equal "
                    f"num_adapters ({num_adapters})."
                )
            for i, (kind, ids) in enumerate(zip(self.adapter_kinds, probe_label_token_ids)):
                if kind == "probe":
                    if not ids:
                        raise ValueError(f"probe slot {i} must declare its label token ids.")
                    if any(t < 0 for t in ids):
                        raise ValueError(f"probe_label_token_ids[{i}] must all be >= 0; got {ids}")
                elif ids:
                    raise ValueError(f"non-probe slot {i} must have no label token ids; got {ids!r}.")
        elif any(k == "probe" for k in self.adapter_kinds):
            raise ValueError(
                "adapter_kinds declares a probe slot but probe_label_token_ids is unset."
            )
        self.probe_label_token_ids = probe_label_token_ids

        if probe_read_layers is not None:
            if len(probe_read_layers) != num_adapters:
                raise ValueError(
                    f"probe_read_layers length ({len(probe_read_layers)}) must equal "
                    f"num_adapters ({num_adapters})."
                )
            n_dec = self.num_hidden_layers - SWITCH_CACHE_LAYERS
            for i, (kind, layer) in enumerate(zip(self.adapter_kinds, probe_read_layers)):
                if layer is None:
                    continue
                if kind != "probe":
                    raise ValueError(f"non-probe slot {i} must have no read layer; got {layer!r}.")
                if not isinstance(layer, int) or isinstance(layer, bool) or not 0 <= layer < n_dec:
                    raise ValueError(
                        f"probe_read_layers[{i}] = {layer!r} must be an int in 0..{n_dec - 1}."
                    )
        self.probe_read_layers = probe_read_layers

        self.probe_num_labels_per_slot = [
            len(ids) if ids else 0 for ids in (probe_label_token_ids or [])
        ] or [0] * num_adapters
        self.max_probe_labels = max(self.probe_num_labels_per_slot, default=0)
        offset = len(self.adapter_token_ids or []) - num_adapters
        self.probe_control_token_ids = [
            (self.adapter_token_ids or [])[i + offset]
            for i, kind in enumerate(self.adapter_kinds)
            if kind == "probe" and self.adapter_token_ids is not None
        ]

        if lora_target_modules is None:
            lora_target_modules = []
            if num_adapters > 0:
                lora_target_modules += ["qkv_proj", "o_proj"]
                if self.shared_intermediate_size > 0:
                    lora_target_modules += ["shared_input_linear", "shared_output_linear"]
        self.lora_target_modules = list(lora_target_modules)

    # ------------------------------------------------------------------ derived
    @property
    def num_decoder_layers(self) -> int:
        """Physical decoder depth (switch cache slots excluded)."""
        if self.num_adapters > 0:
            return self.num_hidden_layers - SWITCH_CACHE_LAYERS
        return self.num_hidden_layers

    @property
    def head_dim_eff(self) -> int:
        return int(self.projection_head_dim)

    @property
    def has_base_reset(self) -> bool:
        return self.adapter_token_ids is not None and len(self.adapter_token_ids) == self.num_adapters + 1

    # ------------------------------------------------------------------ io
    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "GraniteSwitchConfig":
        """Build from a ``config.json`` dict; rejects SingleSwitch checkpoints.

        A checkpoint with adapters whose ``switch_type`` is not ``"multi"``, or
        that has neither ``switch_type`` nor ``ms_code_m``, predates the
        coded-memory switch and was sized for a different layer count
        (reference: config.py:139-178).
        """
        d = dict(d)
        if d.get("num_adapters", 0) > 0:
            st = d.get("switch_type")
            legacy = st is None and "ms_code_m" not in d
            if (st is not None and st != "multi") or legacy:
                raise ValueError(
                    "This checkpoint was built for SingleSwitch, which has been removed; it "
                    "cannot be loaded (its decoder-layer count differs). Re-compose it from its "
                    "PEFT adapters."
                )
        d.pop("switch_type", None)
        d.pop("model_type", None)
        return cls(**d)

    def to_dict(self) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for k, v in self.__dict__.items():
            if k.startswith("_"):
                continue
            out[k] = copy.deepcopy(v)
        out.update(copy.deepcopy(self._extra))
        out["model_type"] = self.model_type
        out["architectures"] = ["GraniteSwitchForCausalLM"]
        return out

    def to_json_string(self) -> str:
        return json.dumps(self.to_dict(), indent=2, sort_keys=True)

    @classmethod
    def from_pretrained(cls, path: str) -> "GraniteSwitchConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_dict(json.load(f))

    def save_pretrained(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "config.json"), "w") as f:
            f.write(self.to_json_string() + "\n")

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return f"GraniteSwitchConfig({self.to_json_string()})"

    def __eq__(self, other: object) -> bool:
        return isinstance(other, GraniteSwitchConfig) and self.to_dict() == other.to_dict()
