"""OpenAI-compatible server, async engine front end and Prometheus metrics."""
from .async_engine import AsyncEngine  # noqa: F401
