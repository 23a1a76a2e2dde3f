"""Models: the HF-style PyTorch class (prototyping, CPU oracle) and the native runner."""
from .reference import GraniteSwitchForCausalLM, GraniteSwitchModel, SwitchCache, load_model  # noqa: F401
