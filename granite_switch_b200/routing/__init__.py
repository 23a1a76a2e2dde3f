"""Routing: token exchange, probe split, exact latest-wins scan, codebooks."""
from .token_exchange import apply_token_exchange, build_control_to_substitute_lut  # noqa: F401
from .probe_routing import build_adapter_kind_lut, split_adapter_indices  # noqa: F401
from .scan import expert_table, route_sequence, route_flat, route_batch  # noqa: F401
