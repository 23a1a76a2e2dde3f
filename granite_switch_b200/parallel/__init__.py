"""Parallelism: tensor-parallel groups, fused symmetric-memory collectives, pipeline stages."""
