"""Hand-written sm_100a ops (one native extension) and their PyTorch oracles."""
