"""Composer: embed LoRA / aLoRA / probe / Shadow-Residual adapters into one checkpoint."""
from .compose import AdapterSpec, compose_checkpoint  # noqa: F401
