"""Serving engine."""
from .llm import LLM, RequestOutput  # noqa: F401
from .sequence import SamplingParams  # noqa: F401
