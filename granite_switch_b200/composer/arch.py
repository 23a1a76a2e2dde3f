"""Architecture descriptors: which module groups a base architecture offers adapters.

One :class:`ModuleGroup` per composed LoRA site: the PEFT module names that
feed it, its composed name, its slice count and the base-checkpoint weights
fused into its base layer. :func:`resolve_arch` picks the descriptor from the
base config's ``model_type`` (reference: src/granite_switch/composer/arch.py:14-483):

* ``granite`` (dense): q/k/v -> ``qkv_proj`` (3 slices), ``o_proj``, and the
  dense MLP mapped onto the shared-MLP sites (gate/up -> ``shared_input_linear``,
  2 slices; down -> ``shared_output_linear``);
* ``granitemoehybrid``: the same attention sites plus the fused shared MLP
  (PEFT ``input_linear`` split into 2 slices, ``output_linear``); frozen
  experts when ``num_local_experts > 0``;
* ``granitemoe``: attention sites only; every layer has a frozen expert bank
  and no shared MLP;
* each with ``dual_stream=True`` adds the layer-level ``cross_stream`` site
  (Shadow Residual).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ModuleGroup:
    name: str                       # composed group key
    sources: tuple[tuple[str, int | None], ...]   # (PEFT module name, slice it writes)
    prefix: str                     # composed module path inside a layer
    slices: int
    base_sources: tuple[str, ...]   # base weights concatenated (in order) into the base layer

    @property
    def peft_modules(self) -> tuple[str, ...]:
        return tuple(m for m, _ in self.sources)

    def slice_of(self, peft_module: str) -> int | None:
        """Slice a PEFT module writes; None for single-slice groups, -1 for a fused
        module that feeds every slice (A duplicated, B chunked)."""
        return dict(self.sources)[peft_module]


@dataclass(frozen=True)
class ArchSpec:
    model_type: str
    groups: tuple[ModuleGroup, ...]
    shared_mlp: bool
    experts: bool
    shadow_residual: bool

    @property
    def group_names(self) -> list[str]:
        return [g.name for g in self.groups]

    def group(self, name: str) -> ModuleGroup:
        for g in self.groups:
            if g.name == name:
                return g
        raise KeyError(f"{self.model_type} has no module group {name!r}")

    def group_of(self, peft_module: str) -> tuple[ModuleGroup, int | None]:
        for g in self.groups:
            if peft_module in g.peft_modules:
                return g, g.slice_of(peft_module)
        raise KeyError(peft_module)

    def check_adapter_modules(self, adapter: str, modules: set[str]) -> None:
        """Every module an adapter trains must be a LoRA site of this architecture."""
        known = {m for g in self.groups for m in g.peft_modules}
        bad = sorted(modules - known)
        if bad:
            raise ValueError(f"adapter {adapter!r} trains {bad}, which the {self.model_type} base "
                             f"{'(Shadow Residual) ' if self.shadow_residual else ''}does not offer as "
                             f"LoRA sites ({sorted(known)})")

    def sizes(self, cfg: dict) -> tuple[dict[str, list[int]], dict[str, int]]:
        """(output size of each slice, input size) per group for a base config."""
        h = int(cfg["hidden_size"])
        nh, nkv = int(cfg["num_attention_heads"]), int(cfg["num_key_value_heads"])
        hd = int(cfg.get("head_dim") or h // nh)
        inter = int(cfg.get("shared_intermediate_size") or cfg.get("intermediate_size") or 0)
        out = {"qkv_proj": [nh * hd, nkv * hd, nkv * hd], "o_proj": [h], "shared_input_linear": [inter, inter],
               "shared_output_linear": [h], "cross_stream": [h]}
        inp = {"qkv_proj": h, "o_proj": nh * hd, "shared_input_linear": h, "shared_output_linear": inter,
               "cross_stream": h}
        names = self.group_names
        return {g: out[g] for g in names}, {g: inp[g] for g in names}


_ATTN = (
    ModuleGroup("qkv_proj", (("q_proj", 0), ("k_proj", 1), ("v_proj", 2)), "self_attn.qkv_proj", 3,
                ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight")),
    ModuleGroup("o_proj", (("o_proj", None),), "self_attn.o_proj", 1, ("self_attn.o_proj.weight",)),
)
_DENSE_MLP = (
    ModuleGroup("shared_input_linear", (("gate_proj", 0), ("up_proj", 1)), "shared_mlp.input_linear", 2,
                ("mlp.gate_proj.weight", "mlp.up_proj.weight")),
    ModuleGroup("shared_output_linear", (("down_proj", None),), "shared_mlp.output_linear", 1,
                ("mlp.down_proj.weight",)),
)
# GraniteMoeHybrid adapters train the fused input_linear (gate|up); adapters
# trained on the split names map onto the same slices
_SHARED_MLP = (
    ModuleGroup("shared_input_linear", (("input_linear", -1), ("gate_proj", 0), ("up_proj", 1)),
                "shared_mlp.input_linear", 2, ("shared_mlp.input_linear.weight",)),
    ModuleGroup("shared_output_linear", (("output_linear", None), ("down_proj", None)), "shared_mlp.output_linear",
                1, ("shared_mlp.output_linear.weight",)),
)
_CROSS = (ModuleGroup("cross_stream", (("cross_stream", None),), "cross_stream", 1, ()),)


def _spec(model_type: str, cfg: dict, dual: bool) -> ArchSpec:
    experts = int(cfg.get("num_local_experts") or 0) > 0
    if model_type == "granite":
        groups, shared = _ATTN + _DENSE_MLP, True
    elif model_type == "granitemoehybrid":
        # with experts the shared MLP exists only when shared_intermediate_size > 0;
        # without experts it carries the dense MLP
        shared = int(cfg.get("shared_intermediate_size") or 0) > 0 if experts else True
        groups = _ATTN + (_SHARED_MLP if shared else ())
    elif model_type == "granitemoe":
        groups, shared, experts = _ATTN, False, True
    else:
        raise ValueError(f"unsupported base architecture {model_type!r}; supported: {sorted(ARCHITECTURES)}")
    if dual:
        groups = groups + _CROSS
    return ArchSpec(model_type, groups, shared, experts, dual)


ARCHITECTURES = ("granite", "granitemoe", "granitemoehybrid")


def resolve_arch(base_config: dict, dual_stream: bool = False) -> ArchSpec:
    """Descriptor for a base config (``model_type``; a composed ``*_switch`` type maps to its base).

    A config without ``model_type`` is read as dense Granite when it has no
    experts, else as GraniteMoeHybrid.
    """
    mt = base_config.get("model_type")
    if mt is None:
        mt = "granitemoehybrid" if int(base_config.get("num_local_experts") or 0) > 0 else "granite"
    mt = str(mt).replace("_switch", "")
    if mt not in ARCHITECTURES:
        raise ValueError(f"unsupported base architecture {mt!r}; supported: {list(ARCHITECTURES)}")
    return _spec(mt, base_config, dual_stream)


__all__ = ["ModuleGroup", "ArchSpec", "resolve_arch", "ARCHITECTURES"]
