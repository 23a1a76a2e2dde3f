"""Serving engine: requests, paged KV + prefix cache, scheduler, executors, LLM API."""
from .llm_engine import DEFAULT_MAX_WAIT_STEPS, LLM, EngineConfig, LLMEngine  # noqa: F401
from .request import Request, RequestOutput, SamplingParams  # noqa: F401
