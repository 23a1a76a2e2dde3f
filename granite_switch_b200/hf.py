"""``transformers`` Auto-class registration for composed Granite Switch checkpoints.

After ``import granite_switch_b200.hf`` a composed directory opens through the
usual entry points (reference: src/granite_switch/hf/__init__.py:15-23)::

    AutoConfig.from_pretrained(path)            # -> GraniteSwitchHFConfig (model_type granite_switch)
    AutoModelForCausalLM.from_pretrained(path)  # -> models.GraniteSwitchForCausalLM

The model class is this package's PyTorch model; its ``from_pretrained`` reads
the composed safetensors itself, so only the config needs a ``transformers``
class. ``GraniteSwitchHFConfig.to_native()`` returns the package's own config.
"""
from __future__ import annotations

_REGISTERED = False


def register() -> bool:
    """Register once; False when transformers is missing or refuses the registration."""
    global _REGISTERED
    if _REGISTERED:
        return True
    try:
        from transformers import AutoConfig, AutoModelForCausalLM, PretrainedConfig
    except ImportError:
        return False
    from .config import GraniteSwitchConfig
    from .models.reference import GraniteSwitchForCausalLM

    class GraniteSwitchHFConfig(PretrainedConfig):
        model_type = "granite_switch"

        def to_native(self) -> GraniteSwitchConfig:
            return GraniteSwitchConfig.from_dict(self.to_dict())

    try:
        AutoConfig.register("granite_switch", GraniteSwitchHFConfig, exist_ok=True)
        GraniteSwitchForCausalLM.config_class = GraniteSwitchHFConfig
        AutoModelForCausalLM.register(GraniteSwitchHFConfig, GraniteSwitchForCausalLM, exist_ok=True)
    except (TypeError, ValueError):
        return False
    globals()["GraniteSwitchHFConfig"] = GraniteSwitchHFConfig
    _REGISTERED = True
    return True


register()
