"""granite_switch_b200: a B200-native (sm_100a) framework for composable adapter models.

Same capabilities, public API and checkpoint format as generative-computing/granite-switch:
a composer that embeds LoRA / aLoRA / probe adapters into one Granite checkpoint, an
HF-style model class, a serving engine with continuous batching and a paged, prefix-cached
KV cache shared across adapters, and hand-written sm_100a kernels on every hot path.
"""
__version__ = "0.1.0"

from .config import GraniteSwitchConfig, SWITCH_CACHE_LAYERS  # noqa: E402,F401
