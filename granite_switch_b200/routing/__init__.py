"""Routing: token exchange, probe split, exact latest-wins scan, codebooks."""
from .token_exchange import apply_token_exchange, build_control_to_substitute_lut  # noqa: F401
from .scan import (expert_table, probe_slot_mask, route_batch, route_flat, route_sequence,  # noqa: F401
                   split_probe_stream)
