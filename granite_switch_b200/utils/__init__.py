"""Utilities: workload generation, device timing, clock sampling, logging."""
